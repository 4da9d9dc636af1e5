"""The peer all-reduce kernel (hif8_b200::peer_allreduce_rmsnorm /
peer_allreduce) on one GPU with a world of one rank: the exchange over one or
several CTAs (column slices, per-(rank, CTA) flags, the grid barrier of the
fused norm, the epoch counter advanced by the last CTA) against a torch
reference of the
same arithmetic -- the partial rounded to BF16 once, the residual added in
BF16, RMSNorm with (1 + w) or w.  residual_out and the plain sum are
bit-exact; the normalised output within one BF16 unit (the reference sums
the squares in FP64, the kernel in FP32 in its fixed order).  The cross-GPU
exchange itself is covered by tests/test_tp_gpu.py (two GPUs) and the TP
legs of the bench."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TIMEOUT_NS = 200_000_000


def _buffer(max_rows, dim):
    from hif8_b200 import cabi

    lib = cabi.library()
    fn = lib.hif8_peer_buffer_bytes
    fn.restype, fn.argtypes = ctypes.c_size_t, [ctypes.c_int64] * 3
    buf = torch.zeros(fn(1, max_rows, dim), dtype=torch.uint8, device=DEV)
    table = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=DEV)
    return buf, table


@pytest.mark.parametrize("dim", [256, 4096, 12288, 65536])  # 65536 x 8 rows: the 16-CTA maximum
@pytest.mark.parametrize("rows", [1, 4, 8])
def test_peer_allreduce_rmsnorm_world_one(rows, dim):
    from hif8_b200 import kv_cache

    kv_cache.load_ops()
    g = torch.Generator(device=DEV).manual_seed(rows * 7 + dim)
    max_rows = 8
    buf, table = _buffer(max_rows, dim)
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    error = torch.zeros(1, dtype=torch.int32, device=DEV)
    weight = (torch.randn(dim, generator=g, device=DEV) * 0.1).to(torch.bfloat16)
    calls = 0
    for one_plus in (True, False):
        for slot in (0, 1, 0):
            local = torch.randn(rows, dim, generator=g, device=DEV) * 3
            residual = torch.randn(rows, dim, generator=g, device=DEV).to(torch.bfloat16)
            out, res_out = torch.ops.hif8_b200.peer_allreduce_rmsnorm(
                local, residual, weight, table, counter, error, max_rows, 0, 1, slot, 1e-6, one_plus, TIMEOUT_NS)
            calls += 1
            v = (local.to(torch.bfloat16).float() + residual.float()).to(torch.bfloat16)
            assert torch.equal(res_out, v), "residual_out = BF16(BF16(partial) + residual)"
            vf = v.double()
            inv = torch.rsqrt((vf * vf).sum(-1, keepdim=True) / dim + 1e-6)
            w = weight.double() + (1.0 if one_plus else 0.0)
            ref = (vf * inv * w).to(torch.bfloat16)
            torch.testing.assert_close(out.float(), ref.float(), rtol=2.0 ** -7, atol=1e-6)
    torch.cuda.synchronize()
    assert int(error) == 0 and int(counter) == calls, (int(error), int(counter))


@pytest.mark.parametrize("rows", [1, 16])
def test_peer_allreduce_sum_world_one(rows):
    from hif8_b200 import kv_cache

    kv_cache.load_ops()
    dim, max_rows = 4096, 16
    buf, table = _buffer(max_rows, dim)
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    error = torch.zeros(1, dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(rows)
    for slot in (0, 1):
        local = torch.randn(rows, dim, generator=g, device=DEV) * 5
        out = torch.ops.hif8_b200.peer_allreduce(local, table, counter, error, max_rows, 0, 1, slot, TIMEOUT_NS)
        assert torch.equal(out, local.to(torch.bfloat16))
        half = torch.randn(rows, dim, generator=g, device=DEV).to(torch.bfloat16)  # a BF16 partial, widened
        out = torch.ops.hif8_b200.peer_allreduce(half, table, counter, error, max_rows, 0, 1, 1 - slot, TIMEOUT_NS)
        assert torch.equal(out, half)
    torch.cuda.synchronize()
    assert int(error) == 0 and int(counter) == 4
