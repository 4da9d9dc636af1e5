"""The vLLM adapter on vLLM's own parallel layers, without a GPU: quant
config registration and lookup (both prefix spellings of the Qwen3.5 text
stack, fused modules, FLOAT layers), weight loading through vLLM's
parameter loaders into the HiF8 parameter contract, the fused-module input
scale rules.  The checks run in a child process (tests/_vllm_adapter_cases.py)
so vLLM's process group stays out of this one."""

from __future__ import annotations

import importlib.util
import subprocess
import sys
from pathlib import Path

import pytest

CASES = Path(__file__).resolve().parent / "_vllm_adapter_cases.py"


@pytest.mark.skipif(importlib.util.find_spec("vllm") is None, reason="vLLM is not installed")
@pytest.mark.timeout(600)
def test_vllm_adapter_layers_cpu():
    proc = subprocess.run([sys.executable, str(CASES), "cpu"], capture_output=True, text=True, timeout=540)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "vllm adapter cases (cpu): ok" in proc.stdout
