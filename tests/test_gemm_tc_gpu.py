"""Prefill GEMM (M >= 32, K % 64 == 0) on the tcgen05 tensor cores against
the FP64 oracle.

The reference computes the same product in FP32 on its CPU/NPU paths
(csrc/hif8_native.cpp:633-669, soft_hif8_gemm); the tolerance MAX_REL = 1e-2
of the largest |output| covers FP32 accumulation plus the final BF16/FP16
rounding; every output channel is also bounded against its own largest
|output| (CHANNEL_REL) and every token row's cosine similarity (MIN_COSINE),
so a wrong small channel among the 20-sigma outlier rows cannot hide under
the global scale.  The activation/weight shapes follow configs[2] of the
workload (prefill of the Qwen3.5-9B projection shapes)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._helpers import channel_rel, max_rel, row_cosine_min
from tests.test_linear_gpu import CHANNEL_REL, MIN_COSINE, _activations, _hif8_weights, _native, _to

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_REL = 1.0e-2


def _err_word(workspace, m, k) -> int:
    off = (m * k * 2 + 255) // 256 * 256
    return int(workspace[off:off + 4].cpu().view(torch.int32)[0])


@pytest.mark.parametrize("n,k", [(24576, 4096), (4096, 12288), (6144, 4096)])
@pytest.mark.parametrize("m", [32, 512, 4096])
def test_prefill_gemm_projection_shapes(m, n, k):
    """Oracle on 192 sampled channels (FP64), torch FP32 on the GPU for all."""
    from hif8_b200 import cabi

    w, w_s = _hif8_weights(n, k, seed=11, outlier_frac=1e-3)
    _, a, a_s, _ = _activations(m, k, seed=m + 3)
    w_dev, ws_dev, a_dev, as_dev = _to(w), _to(w_s), _to(a), _to(a_s)
    lib = cabi.library()
    need = lib.soft_hif8_gemm_workspace_size(m, n, k)
    assert need >= m * k * 2
    workspace = torch.full((need,), 0xAB, dtype=torch.uint8, device=DEV)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    cabi.gemm(a_dev, w_dev, as_dev, ws_dev, None, out, workspace)
    torch.cuda.synchronize()
    assert _err_word(workspace, m, k) == 0, "a pipeline wait timed out"
    got = out.float().cpu().numpy()
    cols = np.sort(np.random.default_rng(m + n).choice(n, size=192, replace=False))
    rows = np.arange(m) if m <= 512 else np.sort(np.random.default_rng(m).choice(m, size=384, replace=False))
    expected = oracle.linear(a[rows], w[cols], a_s[rows], w_s[cols])
    assert max_rel(got[np.ix_(rows, cols)], expected) <= MAX_REL
    assert channel_rel(got[np.ix_(rows, cols)], expected) <= CHANNEL_REL
    lut = torch.from_numpy(oracle.decode_table()).to(DEV)
    ref32 = (lut[a_dev.long()] * as_dev[:, None]) @ (lut[w_dev.long()] * ws_dev[:, None]).T
    ref32 = ref32.cpu().numpy()
    assert max_rel(got, ref32) <= MAX_REL
    assert channel_rel(got, ref32) <= CHANNEL_REL
    assert row_cosine_min(got, ref32) >= MIN_COSINE
    again = torch.empty_like(out)
    cabi.gemm(a_dev, w_dev, as_dev, ws_dev, None, again, workspace)
    assert torch.equal(out, again), "run-twice determinism"


@pytest.mark.parametrize("m,n,k", [(33, 64, 64), (130, 1000, 192), (300, 1000, 4096), (257, 130, 640)])
def test_prefill_gemm_ragged_tiles_bias_f16(m, n, k):
    """Token and channel tails inside a tile, K of one stage, FP16 output and
    BF16/FP16 bias (reference tests/test_npu_ops.py:296-344)."""
    ext = _native().load_extension()
    w, w_s = _hif8_weights(n, k, seed=m, outlier_frac=1e-3)
    _, a, a_s, _ = _activations(m, k, seed=n)
    bias = (np.random.default_rng(k).random(n).astype(np.float32) - 0.5)
    for out_dtype in (torch.float16, torch.bfloat16):
        for bias_dtype in (torch.float16, torch.bfloat16):
            b = _to(bias, bias_dtype)
            out = ext.soft_hif8_gemm(_to(a), _to(w), _to(a_s), _to(w_s), b, out_dtype)
            expected = oracle.linear(a, w, a_s, w_s, b.float().cpu().numpy())
            assert max_rel(out.float().cpu().numpy(), expected) <= MAX_REL, (out_dtype, bias_dtype)


def test_prefill_gemm_propagates_special_codes():
    """NaN and +-Inf activation codes reach the output of their token row
    (reference tests/test_npu_ops.py:179-214, at a tensor-core size)."""
    ext = _native().load_extension()
    one = oracle.encode_value(1.0)
    m, n, k = 48, 128, 64
    codes = [0x80, 0x6F, 0xEF] + [one] * (m - 3)
    act = np.zeros((m, k), np.uint8)
    act[:, 0] = codes
    act[:, 1] = one
    weight = np.zeros((n, k), np.uint8)
    weight[:, 0] = one
    ts = np.linspace(0.5, 2.0, m).astype(np.float32)
    dec = oracle.decode_table()
    for out_dtype in (torch.float16, torch.bfloat16):
        out = ext.soft_hif8_gemm(_to(act), _to(weight), _to(ts), _to(np.ones(n, np.float32)), None, out_dtype)
        got = out.float().cpu().numpy()
        for r in range(m):
            expected = float(dec[codes[r]]) * float(ts[r])
            if np.isnan(expected):
                assert np.isnan(got[r]).all()
            else:
                rounded = float(torch.tensor(expected, dtype=torch.float32).to(out_dtype).float())
                assert (got[r] == rounded).all(), r


def test_prefill_gemm_matches_exact_products():
    """Small-integer operands: every partial sum is exact in FP32, so the
    tensor-core result equals the oracle bit for bit after rounding."""
    ext = _native().load_extension()
    m, n, k = 96, 256, 512
    rng = np.random.default_rng(4)
    values = np.array([-2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0], np.float32)
    a = np.vectorize(oracle.encode_value)(values[rng.integers(0, 7, (m, k))]).astype(np.uint8)
    w = np.vectorize(oracle.encode_value)(values[rng.integers(0, 7, (n, k))]).astype(np.uint8)
    ts = np.ones(m, np.float32)
    cs = np.ones(n, np.float32)
    out = ext.soft_hif8_gemm(_to(a), _to(w), _to(ts), _to(cs), None, torch.float16)
    expected = oracle.linear(a, w, ts, cs).astype(np.float16)
    np.testing.assert_array_equal(out.cpu().numpy(), expected)


def test_prefill_gemm_workspace_contract():
    """The C ABI rejects a short or misaligned workspace instead of writing
    past it."""
    from hif8_b200 import cabi

    m, n, k = 64, 128, 256
    lib = cabi.library()
    need = lib.soft_hif8_gemm_workspace_size(m, n, k)
    a = torch.zeros(m, k, dtype=torch.uint8, device=DEV)
    w = torch.zeros(n, k, dtype=torch.uint8, device=DEV)
    ts = torch.ones(m, device=DEV)
    cs = torch.ones(n, device=DEV)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    big = torch.empty(need + 256, dtype=torch.uint8, device=DEV)
    with pytest.raises(cabi.Hif8Error) as short:
        cabi.gemm(a, w, ts, cs, None, out, big[:need - 1])
    assert short.value.status == cabi.HIF8_ERR_WORKSPACE
    with pytest.raises(cabi.Hif8Error) as misaligned:
        cabi.gemm(a, w, ts, cs, None, out, big[16:16 + need])
    assert misaligned.value.status == cabi.HIF8_ERR_WORKSPACE
    cabi.gemm(a, w, ts, cs, None, out, big[:need])
    torch.cuda.synchronize()
    assert torch.equal(out.float().cpu(), torch.zeros(m, n))


def test_prefill_gemm_split_k():
    """Shapes whose token x channel tiles leave most SMs idle take split-K
    (FP32 partial tiles of K ranges summed in split order by a second kernel,
    bias added once): against the FP64 oracle with BF16/FP16 output and bias,
    FP32 output through the tensor-parallel partial operator, bit-exact on
    small-integer operands, deterministic, and NaN codes still reach their
    rows."""
    from hif8_b200 import cabi

    ext = _native().load_extension()
    lib = cabi.library()
    m, n, k = 96, 512, 8192
    # the plan splits K here: the workspace holds FP32 partials beyond the BF16 copy
    assert lib.soft_hif8_gemm_workspace_size(m, n, k) > (m * k * 2 + 255) // 256 * 256 + 256 + m * n * 4
    w, w_s = _hif8_weights(n, k, seed=5, outlier_frac=1e-3)
    _, a, a_s, _ = _activations(m, k, seed=6)
    bias = (np.random.default_rng(3).random(n).astype(np.float32) - 0.5)
    for out_dtype in (torch.float16, torch.bfloat16):
        b = _to(bias, torch.bfloat16)
        out = ext.soft_hif8_gemm(_to(a), _to(w), _to(a_s), _to(w_s), b, out_dtype)
        expected = oracle.linear(a, w, a_s, w_s, b.float().cpu().numpy())
        got = out.float().cpu().numpy()
        assert max_rel(got, expected) <= MAX_REL, out_dtype
        assert channel_rel(got, expected) <= CHANNEL_REL, out_dtype
        assert row_cosine_min(got, expected) >= MIN_COSINE, out_dtype
        again = ext.soft_hif8_gemm(_to(a), _to(w), _to(a_s), _to(w_s), b, out_dtype)
        assert torch.equal(out, again), "split-K run-twice determinism"
    # FP32 partial products (the tensor-parallel operator) through the same split
    x_bits, _, _, scale = _activations(m, k, seed=6)
    x = _to(x_bits.view(np.int16)).view(torch.bfloat16)
    part = torch.ops.hif8_b200.linear_partial_f32(x, _to(w), _to(scale), _to(w_s))
    data, rows = oracle.static_quant(x_bits, scale)
    assert max_rel(part.cpu().numpy(), oracle.linear(data, w, rows, w_s)) <= 1e-4
    # small integers: every partial and their sum exact in FP32
    rng = np.random.default_rng(9)
    values = np.array([-2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0], np.float32)
    ai = np.vectorize(oracle.encode_value)(values[rng.integers(0, 7, (m, k))]).astype(np.uint8)
    wi = np.vectorize(oracle.encode_value)(values[rng.integers(0, 7, (n, k))]).astype(np.uint8)
    ai[7, 100] = 0x80  # NaN code in row 7
    ones_m, ones_n = np.ones(m, np.float32), np.ones(n, np.float32)
    out = ext.soft_hif8_gemm(_to(ai), _to(wi), _to(ones_m), _to(ones_n), None, torch.float16)
    exp = oracle.linear(ai, wi, ones_m, ones_n).astype(np.float16)
    got = out.cpu().numpy()
    assert np.isnan(got[7]).all()
    np.testing.assert_array_equal(np.delete(got, 7, axis=0), np.delete(exp, 7, axis=0))


@pytest.mark.parametrize("m,n,k", [(4096, 6144, 4096), (512, 4096, 12288), (300, 1000, 640), (257, 136, 256),
                                   (256, 64, 128)])
def test_prefill_gemm_cta_pair(m, n, k, monkeypatch):
    """The CTA-pair kernel (tcgen05.mma.cta_group::2, 256 weight rows x 256
    tokens per pair; taken with HIF8_GEMM_PAIR=1): projection shapes with and
    without split-K, ragged token and channel tails (a pair whose second CTA
    holds only rows past N, a token tile of one row) against the FP64 oracle
    and the single-CTA kernel; run-twice determinism; bit-exact on
    small-integer operands."""
    from hif8_b200 import cabi

    ext = _native().load_extension()
    w, w_s = _hif8_weights(n, k, seed=m + n, outlier_frac=1e-3)
    _, a, a_s, _ = _activations(m, k, seed=k)
    args = (_to(a), _to(w), _to(a_s), _to(w_s))
    monkeypatch.setenv("HIF8_GEMM_PAIR", "0")
    single = ext.soft_hif8_gemm(*args, None, torch.bfloat16)
    monkeypatch.setenv("HIF8_GEMM_PAIR", "1")
    lib = cabi.library()
    need = lib.soft_hif8_gemm_workspace_size(m, n, k)
    workspace = torch.full((need,), 0xAB, dtype=torch.uint8, device=DEV)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    cabi.gemm(*args, None, out, workspace)
    torch.cuda.synchronize()
    assert _err_word(workspace, m, k) == 0, "a pipeline wait timed out"
    got = out.float().cpu().numpy()
    rows = np.arange(m) if m <= 512 else np.sort(np.random.default_rng(m).choice(m, size=256, replace=False))
    cols = np.arange(n) if n <= 1000 else np.sort(np.random.default_rng(n).choice(n, size=256, replace=False))
    expected = oracle.linear(a[rows], w[cols], a_s[rows], w_s[cols])
    assert max_rel(got[np.ix_(rows, cols)], expected) <= MAX_REL
    assert channel_rel(got[np.ix_(rows, cols)], expected) <= CHANNEL_REL
    assert row_cosine_min(got[np.ix_(rows, cols)], expected) >= MIN_COSINE
    assert max_rel(got, single.float().cpu().numpy()) <= MAX_REL
    again = torch.empty_like(out)
    cabi.gemm(*args, None, again, workspace)
    assert torch.equal(out, again), "run-twice determinism"
    rng = np.random.default_rng(m)
    values = np.array([-2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0], np.float32)
    ai = np.vectorize(oracle.encode_value)(values[rng.integers(0, 7, (m, k))]).astype(np.uint8)
    wi = np.vectorize(oracle.encode_value)(values[rng.integers(0, 7, (n, k))]).astype(np.uint8)
    ones_m, ones_n = np.ones(m, np.float32), np.ones(n, np.float32)
    exact = ext.soft_hif8_gemm(_to(ai), _to(wi), _to(ones_m), _to(ones_n), None, torch.float16)
    np.testing.assert_array_equal(exact.cpu().numpy(), oracle.linear(ai, wi, ones_m, ones_n).astype(np.float16))
