"""GPU parity of the dynamic (W8A8HIF8_SOFT) activation path against the CPU
oracle: hif8_dynamic_quant bit-exact on the golden rows, on the reference's
own known-answer rows (tests/test_npu_ops.py:30-50) and on large random
tensors with special rows; soft_hif8_fused_gemm bit-identical to dynamic
quant followed by soft_hif8_gemm (the reference checks the same pair within
8e-2, tests/test_npu_ops.py:448-502); the scheme's apply within the linear
tolerance of the FP64 oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._helpers import bf16_bits, channel_rel, from_bits, max_rel, row_cosine_min

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"
TDTYPE = {"bf16": torch.bfloat16, "f16": torch.float16}


def _native():
    from hif8_b200 import native

    native.load_extension()
    return native


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _check_against_oracle(x: torch.Tensor, dtype: str):
    data, scale = _native().dynamic_quant(x)
    torch.cuda.synchronize()
    # the reference returns the row scales as a stride-16 view
    assert scale.shape == (x.numel() // x.shape[-1],) and scale.stride() == (16,)
    exp_data, exp_scale = oracle.dynamic_quant(_bits(x), dtype=dtype)
    np.testing.assert_array_equal(data.cpu().numpy(), exp_data)
    np.testing.assert_array_equal(scale.cpu().numpy().view(np.uint32), exp_scale.view(np.uint32))
    return data, scale


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_dynamic_quant_golden(dtype):
    g = np.load(GOLDEN / "dynamic.npz")
    x = from_bits(g[f"{dtype}_x"], TDTYPE[dtype]).to(DEV)
    data, scale = _native().dynamic_quant(x)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(data.cpu().numpy(), g[f"{dtype}_data"])
    np.testing.assert_array_equal(scale.cpu().numpy().view(np.uint32), g[f"{dtype}_scale"].view(np.uint32))


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_dynamic_quant_reference_known_answer_rows(dtype):
    rows = [[0.0, 1.0, -2.0, 4.0], [0.25, -0.5, 1.0, -4.0], [float("nan"), float("inf"), -float("inf"), 0.0],
            [2.0 ** -12, -(2.0 ** -11), 2.0 ** -10, -(2.0 ** -9)]]
    data, scale = _check_against_oracle(torch.tensor(rows, dtype=TDTYPE[dtype], device=DEV), dtype)
    # row 0: scale 4, codes of 0, 0.25, -0.5, 1; the non-finite row keeps scale 1e-12
    assert scale[0].item() == 4.0 and data[0, 0].item() == 0
    assert scale[2].item() == np.float32(1e-12)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("k", [4096, 12288, 2048 + 8, 4095, 37, 1])
def test_dynamic_quant_random_with_special_rows(dtype, k):
    """Vector path (K a multiple of 8) and scalar path (ragged K), rows of
    every kind: normal, outlier, all-zero, tiny (amax below 1e-12 for FP32
    but representable), NaN/Inf mixed with finite values, all non-finite."""
    g = torch.Generator().manual_seed(k * 7 + len(dtype))
    rows = 67
    x = torch.randn(rows, k, generator=g) * torch.logspace(-6, 4, rows).unsqueeze(1)
    x[3] = 0.0
    x[5] = x[5] * 1e-30
    if k >= 4:
        x[7, 1] = float("nan")
        x[8, k // 2] = float("inf")
        x[9, -1] = -float("inf")
    x[11] = float("nan")
    x[13, 0] = 6.0e4  # an outlier that sets the row scale
    _check_against_oracle(x.to(TDTYPE[dtype]).to(DEV), dtype)


def test_dynamic_quant_leading_dims_and_many_rows():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(3, 700, 512, generator=g) * 2.5).to(torch.bfloat16).to(DEV)
    data, scale = _check_against_oracle(x, "bf16")
    assert data.shape == x.shape and scale.numel() == 2100


def test_dynamic_quant_through_cabi_with_strided_scale():
    from hif8_b200 import cabi

    lib = cabi.library()
    g = torch.Generator().manual_seed(4)
    x = (torch.randn(33, 1024, generator=g) * 0.3).to(torch.bfloat16).to(DEV)
    data = torch.empty(x.shape, dtype=torch.uint8, device=DEV)
    scale = torch.full((33 * 5,), -1.0, device=DEV)
    status = lib.hif8_dynamic_quant(x.data_ptr(), cabi.HIF8_DTYPE_BF16, 33, 1024, data.data_ptr(), scale.data_ptr(),
                                    5, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert status == cabi.HIF8_OK
    exp_data, exp_scale = oracle.dynamic_quant(_bits(x), dtype="bf16")
    np.testing.assert_array_equal(data.cpu().numpy(), exp_data)
    got = scale.cpu().numpy().reshape(33, 5)
    np.testing.assert_array_equal(got[:, 0], exp_scale)
    assert (got[:, 1:] == -1.0).all(), "the stride gaps must stay untouched"


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_fused_gemm_matches_dynamic_quant_then_gemm(dtype):
    native = _native()
    ext = native.load_extension()
    g = torch.Generator().manual_seed(41)
    for rows, channels, k, with_bias in ((1, 128, 4096, True), (2, 128, 4096, True), (1, 128, 12288, True),
                                         (2, 4096, 4096, False), (1, 6144, 4096, True), (2, 96, 37, True),
                                         (1, 24576, 4096, False)):
        x = torch.randn(rows, k, generator=g).to(TDTYPE[dtype]).to(DEV)
        w = torch.randint(0, 111, (channels, k), generator=g, dtype=torch.uint8).to(DEV)
        cs = (torch.rand(channels, generator=g) + 0.01).to(DEV)
        bias = torch.randn(channels, generator=g).to(TDTYPE[dtype]).to(DEV) if with_bias else None
        data, token_scale = native.dynamic_quant(x)
        expected = ext.soft_hif8_gemm(data, w, token_scale.contiguous(), cs, bias, TDTYPE[dtype])
        actual = ext.soft_hif8_fused_gemm(x, w, cs, bias, TDTYPE[dtype])
        torch.cuda.synchronize()
        assert torch.equal(actual, expected), (rows, channels, k)


def test_fused_linear_rejects_more_than_two_rows():
    native = _native()
    x = torch.zeros(3, 64, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(8, 64, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError, match="M <= 2"):
        native.soft_fused_linear(x, w, torch.ones(8, device=DEV), output_dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="M <= 2"):
        native.load_extension().soft_hif8_fused_gemm(x, w, torch.ones(8, device=DEV), None, torch.bfloat16)


@pytest.mark.parametrize("fused", ["0", "1"])
@pytest.mark.parametrize("m", [1, 2, 5, 64])
def test_soft_scheme_apply_matches_oracle(monkeypatch, fused, m):
    from hif8_b200 import scheme

    monkeypatch.setenv("HIF8_SOFT_FUSED_GENERATION", fused)
    n, k = 4096, 4096
    g = torch.Generator().manual_seed(m)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    layer = scheme.Hif8SoftLinear.from_float(w.to(DEV))
    wq, wq_s = oracle.quantize_rows_amax(w.float().numpy())
    np.testing.assert_array_equal(layer.weight.cpu().numpy(), wq)
    x = (torch.randn(m, k, generator=g) * 1.7).to(torch.bfloat16)
    y = layer(x.to(DEV)).float().cpu().numpy()
    a, a_s = oracle.dynamic_quant(bf16_bits(x), dtype="bf16")
    expected = oracle.linear(a, wq, a_s, wq_s)
    assert max_rel(y, expected) <= 1e-2
    assert channel_rel(y, expected) <= 1e-2
    assert row_cosine_min(y, expected) >= 0.9999
