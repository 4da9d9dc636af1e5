"""hif8_paged_attention_noalloc (split-KV scratch in the library's own
per-device array) against hif8_paged_attention with a caller workspace, on
the configs[3] decode shapes.

Both entry points run the same kernels with the same key chunking, so the
outputs must be bit-identical (torch.equal), not merely close: a scratch race
or an overrun would show up as a difference that a tolerance could hide.  Two
no-alloc calls run back to back on DIFFERENT inputs (the second with a
shorter context and so fewer split partials), each compared with its own
workspace call, so a second call that read partials left in the shared
scratch by the first would be caught.  The calls must also allocate nothing:
torch's allocator and the device's free memory stay unchanged across them.

The file name sorts last so the test also runs after every other GPU test;
it passes alone in a fresh process too (the first no-alloc call on a device
resolves the scratch address, which may load the library's device image, so
the free-memory check starts after that first call)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.test_kv_gpu import _make_paged

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


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


@pytest.mark.parametrize("ctx_len", [512, 4096])
def test_noalloc_attention_matches_workspace_call(ctx_len):
    from hif8_b200 import cabi

    lib = cabi.library()
    first_args = _inputs(ctx_len, seed=ctx_len + 7)
    second_args = _inputs(ctx_len // 2 + 64, seed=ctx_len + 11)  # other values, fewer splits
    outs = {}
    for name, args in (("first", first_args), ("second", second_args)):
        tokens, heads, d = args["query"].shape
        assert lib.hif8_paged_attention_workspace_size(tokens, heads, d, args["max_seq_len"]) > 0
        expected = torch.empty(tokens, heads, d, dtype=torch.bfloat16, device=DEV)
        cabi.paged_attention(**args, out=expected)
        outs[name] = (expected, torch.full_like(expected, float("nan")))
    torch.cuda.synchronize()

    allocated = torch.cuda.memory_allocated(DEV)
    cabi.paged_attention_noalloc(**first_args, out=outs["first"][1])
    torch.cuda.synchronize()
    free_after_first, _ = torch.cuda.mem_get_info(DEV)
    cabi.paged_attention_noalloc(**second_args, out=outs["second"][1])
    torch.cuda.synchronize()
    free_after_second, _ = torch.cuda.mem_get_info(DEV)

    for name, (expected, got) in outs.items():
        assert torch.equal(got, expected), f"{name} no-alloc call differs from its workspace call"
    assert torch.cuda.memory_allocated(DEV) == allocated, "the no-alloc calls allocated through torch"
    assert free_after_second == free_after_first, "the second no-alloc call changed the device's free memory"


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
