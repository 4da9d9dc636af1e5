"""hif8_paged_attention_noalloc (scratch in the library's own per-device
array) against hif8_paged_attention with a caller workspace, on the
configs[3] decode shapes: two calls in a row, each within the attention
tolerance of the workspace call (max-rel <= 1e-2 of max |out|).  The file
name sorts last so the test also runs after every other GPU test."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.test_kv_gpu import _make_paged

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = 1e-2


def _inputs(ctx_len, seed):
    batch, heads, kv_heads, d, block = 4, 16, 4, 256, 128
    ctx = [ctx_len - 29 * b for b in range(batch)]
    kc, vc, table = _make_paged(batch, ctx, kv_heads, d, block, seed=seed)
    q = oracle.round_bf16(np.random.default_rng(seed + 1).standard_normal((batch, heads, d)).astype(np.float32))
    return dict(
        query=torch.from_numpy(q).to(torch.bfloat16).to(DEV),
        key_cache=torch.from_numpy(kc).to(DEV),
        value_cache=torch.from_numpy(vc).to(DEV),
        block_tables=torch.from_numpy(table).to(DEV),
        seq_lens=torch.tensor(ctx, dtype=torch.int32, device=DEV),
        query_start=torch.arange(batch + 1, dtype=torch.int32, device=DEV),
        max_seq_len=max(ctx),
        scale=1.0 / math.sqrt(d),
    )


def _max_rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max()) / max(float(b.abs().max()), 1e-12)


@pytest.mark.parametrize("ctx_len", [512, 4096])
def test_noalloc_attention_matches_workspace_call(ctx_len):
    from hif8_b200 import cabi

    args = _inputs(ctx_len, seed=ctx_len + 7)
    tokens, heads, d = args["query"].shape
    assert cabi.library().hif8_paged_attention_workspace_size(tokens, heads, d, args["max_seq_len"]) > 0
    expected = torch.empty(tokens, heads, d, dtype=torch.bfloat16, device=DEV)
    cabi.paged_attention(**args, out=expected)
    first = torch.full_like(expected, float("nan"))
    second = torch.full_like(expected, float("nan"))
    cabi.paged_attention_noalloc(**args, out=first)
    cabi.paged_attention_noalloc(**args, out=second)
    torch.cuda.synchronize()
    assert _max_rel(first, expected) <= TOL
    assert _max_rel(second, expected) <= TOL


def test_noalloc_attention_rejects_oversized_scratch():
    from hif8_b200 import cabi

    lib = cabi.library()
    limit = 8 << 20
    args = _inputs(512, seed=3)
    tokens, heads, d = args["query"].shape
    # a context long enough that the split partials exceed the scratch
    long_ctx = 256 * (limit // (tokens * heads * (d + 2) * 4) + 1)
    assert lib.hif8_paged_attention_workspace_size(tokens, heads, d, long_ctx) > limit
    out = torch.zeros(tokens, heads, d, dtype=torch.bfloat16, device=DEV)
    args["max_seq_len"] = long_ctx
    with pytest.raises(cabi.Hif8Error) as err:
        cabi.paged_attention_noalloc(**args, out=out)
    assert err.value.status == cabi.HIF8_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert not out.any(), "a rejected call must enqueue nothing"
