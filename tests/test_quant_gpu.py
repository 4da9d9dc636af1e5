"""GPU parity of the static quantiser and the scaled decode against the CPU
oracle: bit-exact on golden fixtures, exhaustive BF16/FP16 sweeps and large
random tensors, through the PyTorch operators and through the C ABI."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._helpers import from_bits

pytestmark = pytest.mark.gpu
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"
DEV = "cuda:0"


def _native():
    from hif8_b200 import native

    native.load_extension()
    return native


def _quant_gpu(bits: np.ndarray, dtype: str, scale: np.ndarray, *, via_cabi: bool = False):
    tdtype = torch.bfloat16 if dtype == "bf16" else torch.float16
    x = from_bits(bits, tdtype).to(DEV)
    s = torch.from_numpy(np.asarray(scale, dtype=np.float32).reshape(-1)).to(DEV)
    if via_cabi:
        from hif8_b200 import cabi

        data = torch.empty(x.shape, dtype=torch.uint8, device=DEV)
        rows = torch.empty(x.numel() // x.shape[-1], dtype=torch.float32, device=DEV)
        cabi.static_quant(x, s, data, rows)
    else:
        data, rows = _native().static_quant(x, s)
    torch.cuda.synchronize()
    return data.cpu().numpy(), rows.cpu().numpy()


@pytest.mark.parametrize("case", ["special", "saturate", "kv_heads", "cfg0_act", "fp16", "exh_1", "exh_small",
                                  "exh_odd"])
def test_static_quant_golden(case):
    g = np.load(GOLDEN / "static_quant.npz")
    x, scale, expected = g[f"{case}__x"], g[f"{case}__scale"], g[f"{case}__out"]
    for via_cabi in (False, True):
        data, rows = _quant_gpu(x, str(g[f"{case}__dtype"]), scale, via_cabi=via_cabi)
        np.testing.assert_array_equal(data, expected)
        np.testing.assert_array_equal(rows, scale[np.arange(rows.size) % scale.size])


# Scales that stress every branch: exact-only (denormal / huge reciprocal),
# negative, zero, NaN, Inf, and ordinary calibrated magnitudes.
SWEEP_SCALES = [1.0, 0.7343872785568237, 3.0517578125e-05 * 1.37, 1.0 / 3.0, 0.1, 2.0 ** 20, 2.0 ** -126, 1e-30,
                1e-45, 3.0e38, -1.5, 0.0, float("inf"), float("nan"), 1.2e-3, 6.5e4]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_static_quant_exhaustive_patterns(dtype):
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(256, 256)
    for s in SWEEP_SCALES:
        scale = np.array([s], dtype=np.float32)
        expected, _ = oracle.static_quant(bits, scale, dtype=dtype)
        data, _ = _quant_gpu(bits, dtype, scale)
        mism = np.count_nonzero(data != expected)
        assert mism == 0, f"scale={s}: {mism} mismatching codes"


def test_static_quant_unaligned_rows_use_scalar_path():
    rng = np.random.default_rng(3)
    for k in (5, 37, 129):
        x = (rng.standard_normal((7, k)) * 100).astype(np.float32)
        bits = oracle.f32_to_bf16_bits(x)
        scale = np.array([0.37], dtype=np.float32)
        expected, _ = oracle.static_quant(bits, scale)
        data, _ = _quant_gpu(bits, "bf16", scale)
        np.testing.assert_array_equal(data, expected)


def test_static_quant_large_random_and_per_head_scales():
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(1024, 4096, generator=g) * torch.exp2(torch.randint(-20, 20, (1024, 1), generator=g).float()))
    bits = oracle.f32_to_bf16_bits(x.numpy())
    for scale in (np.array([0.0123], np.float32), np.array([0.5, 1.25, 3.0e-4, 7.0], np.float32)):
        expected, rows = oracle.static_quant(bits, scale)
        data, rows_gpu = _quant_gpu(bits, "bf16", scale)
        np.testing.assert_array_equal(data, expected)
        np.testing.assert_array_equal(rows_gpu, rows)


def test_static_quant_repeatable():
    native = _native()
    x = torch.randn(64, 4096, device=DEV, dtype=torch.bfloat16)
    s = torch.tensor([0.01], device=DEV)
    a, _ = native.static_quant(x, s)
    b, _ = native.static_quant(x, s)
    assert torch.equal(a, b)


def _decode_gpu(codes: np.ndarray, scales: np.ndarray):
    out = _native().scaled_decode(torch.from_numpy(codes).to(DEV), torch.from_numpy(scales).to(DEV))
    torch.cuda.synchronize()
    return oracle.f32_to_bf16_bits(out.float().cpu().numpy())


def _assert_bf16_equal(actual_bits, expected_bits):
    act = oracle.bf16_bits_to_f32(actual_bits)
    exp = oracle.bf16_bits_to_f32(expected_bits)
    np.testing.assert_array_equal(np.isnan(act), np.isnan(exp))
    keep = ~np.isnan(exp)
    np.testing.assert_array_equal(actual_bits[keep], expected_bits[keep])


@pytest.mark.parametrize("k", [31, 37, 256])
def test_scaled_decode_golden(k):
    g = np.load(GOLDEN / "scaled_decode.npz")
    _assert_bf16_equal(_decode_gpu(g[f"k{k}__codes"], g["scales"]), g[f"k{k}__out"])


def test_scaled_decode_every_byte_and_tiles():
    codes = np.arange(256, dtype=np.uint8).reshape(1, 256)
    _assert_bf16_equal(_decode_gpu(codes, np.array([1.5], np.float32)),
                       oracle.scaled_decode(codes, np.array([1.5], np.float32)))
    rng = np.random.default_rng(42)
    scales = np.concatenate([np.array([0.0, -0.0, 1.0, -1.0, 0.1, 1.00390625, 2.0 ** -20, 2.0 ** 20, np.inf, np.nan],
                                      np.float32), (rng.random(54) * 0.02).astype(np.float32)])
    for k in (31, 37, 256, 4096, 4128, 4133):
        codes = ((np.arange(scales.size * k).reshape(-1, k) * 73) % 256).astype(np.uint8)
        _assert_bf16_equal(_decode_gpu(codes, scales), oracle.scaled_decode(codes, scales))


def test_scaled_decode_long_context_repeated():
    rng = np.random.default_rng(17)
    codes = rng.integers(0, 256, size=(4 * 4096 * 4, 256), dtype=np.uint8)
    scales = (rng.random(codes.shape[0]) * 0.01 + 1e-5).astype(np.float32)
    expected = oracle.scaled_decode(codes, scales)
    native = _native()
    d, s = torch.from_numpy(codes).to(DEV), torch.from_numpy(scales).to(DEV)
    outs = [native.scaled_decode(d, s) for _ in range(3)]
    torch.cuda.synchronize()
    for out in outs:
        _assert_bf16_equal(oracle.f32_to_bf16_bits(out.float().cpu().numpy()), expected)


def test_scaled_decode_strided_sidecar_rows_through_cabi():
    """KV page rows decode in place: row stride head_size + 4 (reference
    tests/test_npu_ops.py:137-177)."""
    from hif8_b200 import cabi

    tokens, heads, d = 3, 2, 256
    data = (np.arange(tokens * heads * d) % 256).astype(np.uint8).reshape(tokens, heads, d)
    scales = np.array([[0.5, 0.75], [1.0, 1.25], [1.5, 2.0]], np.float32)
    packed = oracle.pack_kv_rows(data, scales)
    dev = torch.from_numpy(packed).to(DEV)
    out = torch.empty(tokens * heads, d, dtype=torch.bfloat16, device=DEV)
    cabi.scaled_decode(dev, torch.from_numpy(scales.reshape(-1)).to(DEV), out, row_stride=d + 4)
    torch.cuda.synchronize()
    expected = oracle.scaled_decode(data.reshape(-1, d), scales.reshape(-1))
    _assert_bf16_equal(oracle.f32_to_bf16_bits(out.float().cpu().numpy()), expected)
