"""The vLLM adapter on a B200: vLLM's QKV / row-parallel / merged layers
with the HiF8 methods reproduce hif8_b200.scheme bit for bit (static and
dynamic activations, 1 / 3 / 40 rows), and vLLM's VocabParallelEmbedding
with the HiF8 method matches the oracle's embedding lookup bit for bit.
Runs in a child process (tests/_vllm_adapter_cases.py)."""

from __future__ import annotations

import importlib.util
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
CASES = Path(__file__).resolve().parent / "_vllm_adapter_cases.py"


@pytest.mark.skipif(importlib.util.find_spec("vllm") is None, reason="vLLM is not installed")
@pytest.mark.timeout(600)
def test_vllm_adapter_layers_forward_gpu():
    proc = subprocess.run([sys.executable, str(CASES), "gpu"], capture_output=True, text=True, timeout=540)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "vllm adapter cases (gpu): ok" in proc.stdout
