"""The HiF8 KV-cache attention backend on a B200 through vLLM's own
``Attention.forward``: prefill, decode and mixed chunked-prefill steps with
padded rows write pages byte-identical to the oracle's and attend within the
attention tolerance of the oracle, for layer-set static scales, checkpoint
scales and dynamic row scales; padded pages give bit-identical results.
Runs in a child process (tests/_vllm_attention_cases.py)."""

from __future__ import annotations

import importlib.util
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
CASES = Path(__file__).resolve().parent / "_vllm_attention_cases.py"


@pytest.mark.skipif(importlib.util.find_spec("vllm") is None, reason="vLLM is not installed")
@pytest.mark.timeout(600)
def test_vllm_attention_backend_forward_gpu():
    proc = subprocess.run([sys.executable, str(CASES), "gpu"], capture_output=True, text=True, timeout=540)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "vllm attention cases (gpu): ok" in proc.stdout
