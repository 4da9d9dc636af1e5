"""GPU parity of the HiF8 linear operators (soft_hif8_gemv / soft_hif8_gemm /
soft_hif8_static_fused_gemm) against the CPU oracle.

Tolerance: max |y - y_ref| / max |y_ref| <= 1e-2 against the FP64-accumulated
oracle (the reference's own bar is 2e-2, tests/test_npu_ops.py:296-344), and
the element-wise rtol/atol of the reference tests on its small shapes
(2e-2 FP16 / 8e-2 BF16, tests/test_npu_ops.py:216-294).  The projection-shape
tests also bound every output channel against its own largest |y_ref|
(CHANNEL_REL = 1e-2) and every token row's cosine similarity (>= 0.9999), so
a wrong small-magnitude channel cannot hide under the global scale."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._helpers import channel_rel, max_rel, row_cosine_min

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"
MAX_REL = 1.0e-2
CHANNEL_REL = 1.0e-2
MIN_COSINE = 0.9999


def _native():
    from hif8_b200 import native

    native.load_extension()
    return native


def _to(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return (t if dtype is None else t.to(dtype)).to(DEV)


def _hif8_weights(n, k, seed, outlier_frac=0.0):
    """configs[0]/[2] weights: N(0, 0.02) BF16, optional 20-sigma outliers,
    per-row amax / 32768 scales."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    if outlier_frac:
        count = int(n * k * outlier_frac)
        idx = torch.randint(0, n * k, (count,), generator=g)
        sign = torch.randint(0, 2, (count,), generator=g).float() * 2 - 1
        w.view(-1)[idx] = sign * 20 * 0.02
    w = w.to(torch.bfloat16).float().numpy()
    data, scale = oracle.quantize_rows_amax(w)
    return data, scale


def _activations(m, k, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).float().numpy()
    calib = torch.randn(max(m, 4), k, generator=torch.Generator().manual_seed(seed + 1000)).to(torch.bfloat16)
    input_scale = np.array([float(calib.float().abs().max()) / 32768.0], np.float32)
    bits = oracle.f32_to_bf16_bits(x)
    data, rows = oracle.static_quant(bits, input_scale)
    return bits, data, rows, input_scale


def test_reference_known_answer_2x2():
    g = np.load(GOLDEN / "linear.npz")
    native = _native()
    out = native.soft_linear(_to(g["k22_a"]), _to(g["k22_w"]), _to(g["k22_as"]), _to(g["k22_ws"]),
                             _to(g["k22_bias"], torch.bfloat16), output_dtype=torch.float16)
    torch.testing.assert_close(out.float().cpu(), torch.tensor([[1.75, -0.5], [-0.5, -1.25]]), rtol=0, atol=0)


@pytest.mark.parametrize("rows,channels,k", [(1, 17, 37), (2, 17, 37), (3, 3, 4), (5, 16, 16), (3, 17, 37),
                                             (3, 256, 16), (3, 2176, 16), (5, 16, 255), (1, 17, 1024),
                                             (2, 17, 1037), (1, 33, 2048)])
def test_small_shapes_match_reference_linear(rows, channels, k):
    """Shapes of the reference's gemm/gemv tests (tests/test_npu_ops.py:257-294, 685-716)."""
    act = np.array([[((r * 7 + c * 3) % 17 - 8) / 4.0 for c in range(k)] for r in range(rows)], np.float32)
    wts = np.array([[((r * 5 + c * 11) % 19 - 9) / 5.0 for c in range(k)] for r in range(channels)], np.float32)
    a, a_s = oracle.quantize_rows_amax(act, 1.0)
    w, w_s = oracle.quantize_rows_amax(wts, 1.0)
    bias = np.array([((c * 3) % 11 - 5) / 8.0 for c in range(channels)], np.float32)
    expected = oracle.linear_exact(a, w, a_s, w_s, bias)
    ext = _native().load_extension()
    for out_dtype, tol in ((torch.float16, 2e-2), (torch.bfloat16, 8e-2)):
        for bias_dtype in (None, torch.float16, torch.bfloat16):
            b = None if bias_dtype is None else _to(bias, bias_dtype)
            exp = expected if bias_dtype is None else expected
            if bias_dtype is None:
                exp = oracle.linear_exact(a, w, a_s, w_s, None)
            out = ext.soft_hif8_gemm(_to(a), _to(w), _to(a_s), _to(w_s), b, out_dtype)
            np.testing.assert_allclose(out.float().cpu().numpy(), exp, rtol=tol, atol=tol)
            if rows <= 2:
                out = ext.soft_hif8_gemv(_to(a), _to(w), _to(a_s), _to(w_s), b, out_dtype)
                np.testing.assert_allclose(out.float().cpu().numpy(), exp, rtol=tol, atol=tol)


def test_gemv_propagates_special_codes():
    """reference tests/test_npu_ops.py:179-214"""
    ext = _native().load_extension()
    one = oracle.encode_value(1.0)
    codes = [0x80, 0x6F, 0xEF]
    weight = _to(np.array([[one, 0] for _ in codes], np.uint8))
    token_scale = [1.5, 0.5, 2.0]
    dec = oracle.decode_table()
    for row, code in enumerate(codes):
        for out_dtype in (torch.float16, torch.bfloat16):
            act = _to(np.array([[code, one]], np.uint8))
            out = ext.soft_hif8_gemv(act, weight, _to(np.array([token_scale[row]], np.float32)),
                                     _to(np.ones(3, np.float32)), None, out_dtype)
            actual = float(out.float().cpu()[0, row])
            expected = float(dec[code]) * token_scale[row]
            if np.isnan(expected):
                assert np.isnan(actual)
            else:
                assert actual == expected


@pytest.mark.parametrize("n,k", [(24576, 4096), (4096, 12288), (6144, 4096)])
def test_decode_gemv_shapes_against_oracle(n, k):
    """M in {1,2,4,8,16} on the three projection shapes.  The
    oracle recomputes 256 sampled output channels in FP64; a torch FP32
    reference on the GPU checks every channel."""
    native = _native()
    w, w_s = _hif8_weights(n, k, seed=0)
    w_dev, ws_dev = _to(w), _to(w_s)
    rng = np.random.default_rng(n + k)
    cols = np.sort(rng.choice(n, size=256, replace=False))
    lut = torch.from_numpy(oracle.decode_table()).to(DEV)
    for m in (1, 2, 4, 8, 16):
        _, a, a_s, _ = _activations(m, k, seed=m)
        out = native.soft_linear(_to(a), w_dev, _to(a_s), ws_dev, output_dtype=torch.bfloat16)
        got = out.float().cpu().numpy()
        expected = oracle.linear(a, w[cols], a_s, w_s[cols])
        assert max_rel(got[:, cols], expected) <= MAX_REL, f"m={m}"
        assert channel_rel(got[:, cols], expected) <= CHANNEL_REL, f"m={m}"
        ref32 = (lut[_to(a).long()] * _to(a_s)[:, None]) @ (lut[w_dev.long()] * ws_dev[:, None]).T
        ref32 = ref32.cpu().numpy()
        assert max_rel(got, ref32) <= MAX_REL
        assert channel_rel(got, ref32) <= CHANNEL_REL, f"m={m}"
        assert row_cosine_min(got, ref32) >= MIN_COSINE, f"m={m}"
        again = native.soft_linear(_to(a), w_dev, _to(a_s), ws_dev, output_dtype=torch.bfloat16)
        assert torch.equal(out, again), "run-twice determinism"


@pytest.mark.parametrize("m", [32, 64, 65, 129])
def test_gemm_medium_m_with_bias_against_oracle(m):
    native = _native()
    n, k = 1024, 4096
    w, w_s = _hif8_weights(n, k, seed=5, outlier_frac=1e-3)
    _, a, a_s, _ = _activations(m, k, seed=100 + m)
    bias = (np.random.default_rng(m).random(n).astype(np.float32) - 0.5)
    for out_dtype in (torch.float16, torch.bfloat16):
        out = native.soft_linear(_to(a), _to(w), _to(a_s), _to(w_s), _to(bias, torch.bfloat16), output_dtype=out_dtype)
        bias_r = oracle.round_bf16(bias)
        expected = oracle.linear(a, w, a_s, w_s, bias_r)
        assert max_rel(out.float().cpu().numpy(), expected) <= MAX_REL
        assert channel_rel(out.float().cpu().numpy(), expected) <= CHANNEL_REL
        assert row_cosine_min(out.float().cpu().numpy(), expected) >= MIN_COSINE


def test_gemm_unaligned_tails_and_long_k():
    """reference tests/test_npu_ops.py:296-344 and 408-446 shapes"""
    ext = _native().load_extension()
    for rows, channels, k in ((1, 128, 4096), (2, 128, 12288), (12, 128, 4096), (129, 1024, 4097)):
        rng = np.random.default_rng(rows * 7 + k)
        a = rng.integers(0, 111, size=(rows, k), dtype=np.uint8)
        w = rng.integers(0, 111, size=(channels, k), dtype=np.uint8)
        ts = np.ones(rows, np.float32)
        cs = np.ones(channels, np.float32)
        out = ext.soft_hif8_gemm(_to(a), _to(w), _to(ts), _to(cs), None, torch.bfloat16)
        expected = oracle.linear(a, w, ts, cs)
        assert max_rel(out.float().cpu().numpy(), expected) <= 2e-2
        again = ext.soft_hif8_gemm(_to(a), _to(w), _to(ts), _to(cs), None, torch.bfloat16)
        assert torch.equal(out, again)


def test_static_fused_matches_quant_then_linear():
    """reference tests/test_npu_ops.py:503-563: same bytes, same kernel."""
    native = _native()
    ext = native.load_extension()
    g = torch.Generator().manual_seed(20260821)
    for rows, channels, k, with_bias in ((1, 128, 2048, False), (2, 256, 4096, True), (4, 256, 4096, True),
                                         (1, 128, 12288, True), (3, 1024, 4096, False), (2, 96, 37, True)):
        x = (torch.randn(rows, k, generator=g) * 3.0).to(torch.bfloat16).to(DEV)
        w = torch.randint(0, 111, (channels, k), generator=g, dtype=torch.uint8).to(DEV)
        fixed = torch.tensor([0.75], device=DEV)
        cs = (torch.rand(channels, generator=g) + 0.01).to(DEV)
        bias = torch.randn(channels, generator=g).to(torch.bfloat16).to(DEV) if with_bias else None
        data, row_scale = native.static_quant(x, fixed)
        expected = ext.soft_hif8_gemm(data, w, row_scale, cs, bias, torch.bfloat16)
        actual = ext.soft_hif8_static_fused_gemm(x, w, fixed, cs, bias, torch.bfloat16)
        torch.testing.assert_close(actual.float(), expected.float(), rtol=0, atol=0)


def test_static_fused_saturates_finite_outliers():
    """reference tests/test_npu_ops.py:565-605"""
    native = _native()
    ext = native.load_extension()
    k = 2048
    x = torch.zeros((1, k), dtype=torch.bfloat16)
    x[0, :6] = torch.tensor([1.0e20, -1.0e20, 32768.0, -32768.0, 65536.0, -65536.0], dtype=torch.bfloat16)
    x = x.to(DEV)
    w = torch.zeros((128, k), dtype=torch.uint8, device=DEV)
    one = oracle.encode_value(1.0)
    for c in range(6):
        w[c, c] = one
    fixed = torch.ones(1, device=DEV)
    cs = torch.ones(128, device=DEV)
    data, row_scale = native.static_quant(x, fixed)
    expected = ext.soft_hif8_gemm(data, w, row_scale, cs, None, torch.bfloat16)
    actual = ext.soft_hif8_static_fused_gemm(x, w, fixed, cs, None, torch.bfloat16)
    torch.testing.assert_close(actual.float(), expected.float(), rtol=0, atol=0, equal_nan=True)
    assert float(actual[0, 0]) == 32768.0 and float(actual[0, 1]) == -32768.0


def test_linear_through_cabi_with_host_contract():
    from hif8_b200 import cabi

    n, k, m = 6144, 4096, 4
    w, w_s = _hif8_weights(n, k, seed=9)
    _, a, a_s, _ = _activations(m, k, seed=9)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    cabi.gemm(_to(a), _to(w), _to(a_s), _to(w_s), None, out)
    torch.cuda.synchronize()
    cols = np.arange(0, n, 24)
    assert max_rel(out.float().cpu().numpy()[:, cols], oracle.linear(a, w[cols], a_s, w_s[cols])) <= MAX_REL


def test_operator_row_contracts_are_strict():
    """reference tests/test_npu_ops.py:718-752"""
    ext = _native().load_extension()
    a = torch.zeros((3, 4), dtype=torch.uint8, device=DEV)
    w = torch.zeros((2, 4), dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="M <= 2"):
        ext.soft_hif8_gemv(a, w, torch.ones(3, device=DEV), torch.ones(2, device=DEV), None, torch.float16)
    view = torch.zeros((3, 4), dtype=torch.uint8, device=DEV)[1:]
    assert view.is_contiguous() and view.storage_offset() > 0
    with pytest.raises(RuntimeError, match="storage_offset == 0"):
        ext.soft_hif8_gemv(view, w, torch.ones(2, device=DEV), torch.ones(2, device=DEV), None, torch.float16)


def test_scheme_apply_matches_oracle():
    from hif8_b200 import scheme

    n, k = 4096, 4096
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    x_bits, a, a_s, input_scale = _activations(4, k, seed=1)
    layer = scheme.Hif8StaticLinear.from_float(w.to(DEV), _to(input_scale))
    wq, wq_s = oracle.quantize_rows_amax(w.float().numpy())
    np.testing.assert_array_equal(layer.weight.cpu().numpy(), wq)
    np.testing.assert_array_equal(layer.weight_scale.cpu().numpy(), wq_s)
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16).to(DEV)
    y_fused = layer(x)
    expected = oracle.linear(a, wq, a_s, wq_s)
    assert max_rel(y_fused.float().cpu().numpy(), expected) <= MAX_REL


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 9, 15, 16, 17, 31, 32, 33, 48])
def test_routing_boundaries_in_m(m):
    """Every row count across the kernel boundaries -- fused quant + GEMV
    (<= 4 rows), quant + persistent GEMV (16-row slices), the tcgen05 GEMM
    (>= 32 rows) -- through scheme.apply, with an output width that is not a
    multiple of any row block (reference tests/test_npu_ops.py:346-406)."""
    from hif8_b200 import scheme

    n, k = 4104, 4096
    w, w_s = _hif8_weights(n, k, seed=100 + m)
    x_bits, a, a_s, input_scale = _activations(m, k, seed=200 + m)
    layer = scheme.Hif8StaticLinear(_to(w), _to(w_s).reshape(-1, 1), _to(input_scale))
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16).to(DEV)
    y = layer(x)
    assert y.shape == (m, n) and y.dtype == torch.bfloat16
    assert max_rel(y.float().cpu().numpy(), oracle.linear(a, w, a_s, w_s)) <= MAX_REL


@pytest.mark.parametrize("n", [1, 17, 100, 272, 1544])
@pytest.mark.parametrize("m", [1, 7, 16])
def test_gemv_output_width_tails(n, m):
    """Full and partial row blocks of the persistent GEMV, every last-item
    shape (reference tests/test_npu_ops.py:685-716), F16 output with bias."""
    ext = _native().load_extension()
    k = 2048
    w, w_s = _hif8_weights(n, k, seed=n + 7 * m)
    _, a, a_s, _ = _activations(m, k, seed=n + 11 * m)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(n)) * 0.1).to(torch.float16)
    out = ext.soft_hif8_gemm(_to(a), _to(w), _to(a_s), _to(w_s), bias.to(DEV), torch.float16)
    assert out.dtype == torch.float16 and out.shape == (m, n)
    expected = oracle.linear(a, w, a_s, w_s) + bias.float().numpy()[None, :]
    assert max_rel(out.float().cpu().numpy(), expected) <= MAX_REL


@pytest.mark.parametrize("n,k", [(6144, 4096), (24576, 4096), (4096, 12288), (4096, 4096), (12288, 4096),
                                 (4096, 8192)])
def test_static_fused_qwen35_generation_shapes(n, k):
    """The fused op on the 9B decoder's projection shapes at 1-4 rows, equal
    to static quant + linear (reference tests/test_npu_ops.py:607-683)."""
    native = _native()
    ext = native.load_extension()
    w, w_s = _hif8_weights(n, k, seed=n + k)
    wd, wsd = _to(w), _to(w_s)
    fixed = torch.tensor([5.0 / 32768.0], device=DEV)
    for m in (1, 2, 3, 4):
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + k)).to(torch.bfloat16).to(DEV)
        data, row_scale = native.static_quant(x, fixed)
        expected = ext.soft_hif8_gemm(data, wd, row_scale, wsd, None, torch.bfloat16)
        actual = ext.soft_hif8_static_fused_gemm(x, wd, fixed, wsd, None, torch.bfloat16)
        torch.testing.assert_close(actual.float(), expected.float(), rtol=0, atol=0)


@pytest.mark.parametrize("m", [1, 4, 8, 16, 64, 512])
def test_tensor_parallel_partial_products_fp32(m):
    """hif8_b200::linear_partial_f32 (the row-parallel partial product of a
    tensor-parallel split, kept in FP32): against the FP32 torch reference on
    every route (fused quant + GEMV for m <= 8, static quant + GEMV for
    m <= 16, the tcgen05 GEMM beyond), and the split property -- the two
    halves of the K dimension summed in FP32 and rounded once match the
    unsharded BF16 projection within one BF16 unit in the last place."""
    _native()
    n, k = 4096, 2048
    w, w_s = _hif8_weights(n, k, seed=40 + m)
    bits, a, a_s, scale = _activations(m, k, seed=41 + m)
    x = _to(bits.view(np.int16)).view(torch.bfloat16)
    w_dev, ws_dev, s_dev = _to(w), _to(w_s), _to(scale)
    full = torch.ops.hif8_b200.linear_partial_f32(x, w_dev, s_dev, ws_dev)
    assert full.dtype == torch.float32 and full.shape == (m, n)
    lut = torch.from_numpy(oracle.decode_table()).to(DEV)
    ref32 = ((lut[_to(a).long()] * _to(a_s)[:, None]) @ (lut[w_dev.long()] * ws_dev[:, None]).T).cpu().numpy()
    assert max_rel(full.cpu().numpy(), ref32) <= 1e-4, f"m={m}"
    half = k // 2
    # each rank's input columns, as a row-parallel split holds them (owned tensors)
    p0 = torch.ops.hif8_b200.linear_partial_f32(x[:, :half].clone(), w_dev[:, :half].clone(), s_dev, ws_dev)
    p1 = torch.ops.hif8_b200.linear_partial_f32(x[:, half:].clone(), w_dev[:, half:].clone(), s_dev, ws_dev)
    summed = (p0 + p1).to(torch.bfloat16)
    from hif8_b200 import scheme

    lin = scheme.Hif8StaticLinear(w_dev, ws_dev.reshape(-1, 1), s_dev)
    unsharded = scheme.apply(lin, x)
    # the two differ only in the order of the FP32 sums: within BF16 rounding
    # of the largest output, and at most one BF16 ulp on almost every element
    # (an output that is a small difference of large terms carries the FP32
    # order error as several of its own ulps)
    assert max_rel(summed.float().cpu().numpy(), unsharded.float().cpu().numpy()) <= 2.0**-8, f"m={m}"
    ulps = (summed.view(torch.int16).int() - unsharded.view(torch.int16).int()).abs()
    assert float((ulps > 1).float().mean()) <= 1e-3, f"m={m}: split partials differ by more than one BF16 ulp"


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_static_linear_op_equals_the_two_call_path(dtype):
    """hif8_b200::static_linear (scheme.apply's single operator) is the
    reference's pair of calls bit for bit: soft_hif8_static_fused_gemm for
    rows <= fused_max_rows, static quant + soft_hif8_gemm beyond (GEMV and
    tcgen05 routes), with and without bias, for 3-D and strided inputs, and
    through the C ABI."""
    from hif8_b200 import cabi

    native = _native()
    ext = native.load_extension()
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    g = torch.Generator().manual_seed(77)
    n, k = 1544, 4096
    w = torch.randint(0, 111, (n, k), generator=g, dtype=torch.uint8).to(DEV)
    cs = (torch.rand(n, generator=g) * 1e-3 + 1e-4).to(DEV)
    fixed = torch.tensor([3.0 / 32768.0], device=DEV)
    bias = torch.randn(n, generator=g).to(tdt).to(DEV)
    for m in (1, 2, 3, 4, 5, 8, 16, 17, 33, 64, 512):
        x = (torch.randn(m, k, generator=g) * 2).to(tdt).to(DEV)
        for fused_rows in (4, 0):
            for b in (None, bias):
                got = torch.ops.hif8_b200.static_linear(x, w, fixed, cs, b, fused_rows)
                if m <= fused_rows:
                    expected = ext.soft_hif8_static_fused_gemm(x, w, fixed, cs, b, tdt)
                else:
                    data, row_scale = native.static_quant(x, fixed)
                    expected = ext.soft_hif8_gemm(data, w, row_scale, cs, b, tdt)
                assert torch.equal(got, expected), (m, fused_rows, b is None)
        via_abi = torch.empty(m, n, dtype=tdt, device=DEV)
        cabi.static_linear(x, w, fixed, cs, bias, via_abi)
        assert torch.equal(via_abi, torch.ops.hif8_b200.static_linear(x, w, fixed, cs, bias, 4)), m
    x3 = (torch.randn(2, 3, 2 * k, generator=g)).to(tdt).to(DEV)[:, :, ::2]  # strided [2, 3, K]
    got = torch.ops.hif8_b200.static_linear(x3, w, fixed, cs, None, 4)
    data, row_scale = native.static_quant(x3.contiguous(), fixed)
    expected = ext.soft_hif8_gemm(data.reshape(6, k), w, row_scale, cs, None, tdt)
    assert got.shape == (2, 3, n) and torch.equal(got.reshape(6, n), expected)
    with pytest.raises(RuntimeError, match="K dimensions differ"):
        torch.ops.hif8_b200.static_linear(x3[..., :-8], w, fixed, cs, None, 4)
    # prefill rows holding specials (NaN, Inf, huge and tiny values, zeros): the
    # GEMM's fused operand pass takes the exact path for their chunks
    xs = (torch.randn(64, k, generator=g) * 2).to(tdt)
    xs[3, :6] = torch.tensor([float("nan"), float("inf"), -float("inf"), 6.0e4, -1e-7, 0.0]).to(tdt)
    xs[40] = 0
    xs = xs.to(DEV)
    data, row_scale = native.static_quant(xs, fixed)
    expected = ext.soft_hif8_gemm(data, w, row_scale, cs, bias, tdt)
    got = torch.ops.hif8_b200.static_linear(xs, w, fixed, cs, bias, 4)
    assert torch.equal(got.isnan(), expected.isnan())
    assert torch.equal(torch.nan_to_num(got), torch.nan_to_num(expected))
    for odd in (torch.tensor([2.0 ** -70], device=DEV), torch.tensor([0.25], device=DEV)):  # exact-only / power of two
        data, row_scale = native.static_quant(xs, odd)
        expected = ext.soft_hif8_gemm(data, w, row_scale, cs, None, tdt)
        got = torch.ops.hif8_b200.static_linear(xs, w, odd, cs, None, 4)
        assert torch.equal(torch.nan_to_num(got), torch.nan_to_num(expected)), float(odd)
    # contiguous views at an aligned and at an unaligned offset of a packed buffer
    for m in (2, 16):
        buf = (torch.randn(m * k + 16, generator=g) * 2).to(tdt).to(DEV)
        for off in (8, 3):
            xv = buf[off:off + m * k].view(m, k)
            got = torch.ops.hif8_b200.static_linear(xv, w, fixed, cs, bias, 4)
            assert torch.equal(got, torch.ops.hif8_b200.static_linear(xv.clone(), w, fixed, cs, bias, 4)), (m, off)
