"""The HiF8 KV-cache attention backend for vLLM, without a GPU: the
``HIF8_KV_CACHE`` install hooks (backend registered as CUSTOM, cache dtype and
attention backend defaults, explicit other choices refused, reset), the
cache shape and vLLM's page budget on a real ``Attention`` layer, layer-index
and tensor-parallel head-scale rules, metadata from vLLM's common metadata,
and the refusals (sliding window, non-HiF8 cache dtype).  The checks run in
a child process (tests/_vllm_attention_cases.py) so vLLM's process group
stays out of this one."""

from __future__ import annotations

import importlib.util
import subprocess
import sys
from pathlib import Path

import pytest

CASES = Path(__file__).resolve().parent / "_vllm_attention_cases.py"


@pytest.mark.skipif(importlib.util.find_spec("vllm") is None, reason="vLLM is not installed")
@pytest.mark.timeout(600)
def test_vllm_attention_backend_cpu():
    proc = subprocess.run([sys.executable, str(CASES), "cpu"], capture_output=True, text=True, timeout=540)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "vllm attention cases (cpu): ok" in proc.stdout
