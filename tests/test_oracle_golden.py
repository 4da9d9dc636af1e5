"""Pin the CPU oracle against golden vectors produced by the reference's own
Python code (tests/golden/make_golden.py).  CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _load(name):
    return np.load(GOLDEN / name, allow_pickle=False)


def test_decode_tables_match_reference():
    g = _load("codec.npz")
    dec = oracle.decode_table()
    np.testing.assert_array_equal(np.isnan(dec), np.isnan(g["decode"]))
    finite = ~np.isnan(dec)
    np.testing.assert_array_equal(dec[finite], g["decode"][finite])
    np.testing.assert_array_equal(oracle.decode_bf16_table(), g["decode_bf16"])


def test_encode_lut_matches_reference():
    g = _load("codec.npz")
    np.testing.assert_array_equal(oracle.encode_lut4096(), g["lut4096"])


def test_scalar_and_tensor_encode_match_reference():
    g = _load("codec.npz")
    x = g["enc_inputs"]
    scalar = np.array([oracle.encode_value(v) for v in x], dtype=np.uint8)
    np.testing.assert_array_equal(scalar, g["enc_scalar"])
    np.testing.assert_array_equal(oracle.encode_tensor(x), g["enc_tensor"])


def test_positive_code_round_trip():
    g = _load("codec.npz")
    dec = oracle.decode_table()
    for value, code in zip(g["positive_values"], g["positive_codes"]):
        assert oracle.encode_value(value) == code
        assert dec[code] == value
        if value != 0.0:
            assert oracle.encode_value(-value) == (code | 0x80)


@pytest.mark.parametrize("case", ["special", "saturate", "kv_heads", "cfg0_act", "fp16",
                                  "exh_1", "exh_small", "exh_odd"])
def test_static_quant_matches_reference(case):
    g = _load("static_quant.npz")
    x = g[f"{case}__x"]
    out, row_scale = oracle.static_quant(x, g[f"{case}__scale"], dtype=str(g[f"{case}__dtype"]))
    np.testing.assert_array_equal(out, g[f"{case}__out"])
    s = g[f"{case}__scale"]
    np.testing.assert_array_equal(row_scale, s[np.arange(row_scale.size) % s.size])


@pytest.mark.parametrize("k", [31, 37, 256])
def test_scaled_decode_matches_reference(k):
    g = _load("scaled_decode.npz")
    out = oracle.scaled_decode(g[f"k{k}__codes"], g["scales"])
    expected = g[f"k{k}__out"]
    # NaN payloads are not part of the contract (torch's vectorised BF16
    # cast writes 0xFFFF, the scalar cast 0x7FC0); NaN-ness and every
    # non-NaN bit pattern are.
    nan_out = np.isnan(oracle.bf16_bits_to_f32(out))
    nan_exp = np.isnan(oracle.bf16_bits_to_f32(expected))
    np.testing.assert_array_equal(nan_out, nan_exp)
    np.testing.assert_array_equal(out[~nan_exp], expected[~nan_exp])
    assert np.all(out[nan_out] == 0x7FC0)


def test_kv_quant_pack_and_write_match_reference():
    g = _load("kv.npz")
    packed = oracle.pack_kv_rows(g["rt_data"], g["rt_scale"])
    np.testing.assert_array_equal(packed, g["rt_packed"])
    data, scale = oracle.unpack_kv_rows(packed, 4)
    np.testing.assert_array_equal(data, g["rt_data"])
    np.testing.assert_array_equal(scale, g["rt_scale"])
    cache = np.zeros_like(g["w_cache"])
    rejected = oracle.kv_write(g["w_src"], g["w_scale"], g["w_slots"], cache)
    assert rejected == 0
    np.testing.assert_array_equal(cache, g["w_cache"])


def test_paged_attention_matches_reference_attention():
    g = _load("kv.npz")
    out = oracle.paged_attention(g["pa_query"], g["w_cache"], g["w_cache"], g["pa_table"], g["pa_seq"],
                                 block_size=4, scale=0.25, bf16_kv=False)
    np.testing.assert_allclose(out, g["pa_out"], rtol=1e-5, atol=1e-5)


def test_linear_known_answers():
    g = _load("linear.npz")
    out = oracle.linear_exact(g["k22_a"], g["k22_w"], g["k22_as"], g["k22_ws"], g["k22_bias"])
    np.testing.assert_array_equal(out, g["k22_out"])
    np.testing.assert_array_equal(out, np.array([[1.75, -0.5], [-0.5, -1.25]]))
    # The reference keeps these row scales as Python doubles (e.g. 9/5); the
    # fixture stores them as FP32, so agreement is to FP32 scale rounding.
    out = oracle.linear_exact(g["t_a"], g["t_w"], g["t_as"], g["t_ws"], g["t_bias"])
    np.testing.assert_allclose(out, g["t_out"], rtol=1e-6, atol=1e-6)
    out2 = oracle.linear(g["t_a"], g["t_w"], g["t_as"], g["t_ws"], g["t_bias"])
    np.testing.assert_allclose(out2, out, rtol=1e-12, atol=1e-12)


def test_weight_row_quantisation_matches_reference():
    g = _load("linear.npz")
    src = oracle.bf16_bits_to_f32(g["wq_src"])
    data, scale = oracle.quantize_rows_amax(src)
    np.testing.assert_array_equal(scale, g["wq_scale"])
    np.testing.assert_array_equal(data, g["wq_data"])


def test_embedding_matches_reference_lookup():
    """The W8A8HIF8_SOFT embedding (scheme.py:120-131): the reference's own
    known answer (tests/test_embedding.py) and seeded rows with every code,
    bit-exact."""
    g = _load("embedding.npz")
    for name in ("ka", "v", "s"):
        out = oracle.embedding(g[f"{name}_w"], g[f"{name}_ws"], g[f"{name}_ids"])
        assert_bf16_equal_nan_any(out, g[f"{name}_out"])
    # the known answer's scales are BF16 values: FP32 decode x scale agrees
    dec = oracle.decode_table()
    ka = dec[g["ka_w"]] * g["ka_ws"]
    np.testing.assert_array_equal(oracle.bf16_bits_to_f32(g["ka_out"]), ka[g["ka_ids"]])


def assert_bf16_equal_nan_any(actual, expected):
    """Bit-exact BF16, except that any NaN pattern equals any other: the
    reference's CPU lookup writes NaN as 0xFFFF (ATen's vectorised float ->
    BF16 cast), this build as the canonical 0x7FC0."""
    a_nan = (actual & 0x7FFF) > 0x7F80
    e_nan = (expected & 0x7FFF) > 0x7F80
    np.testing.assert_array_equal(a_nan, e_nan)
    np.testing.assert_array_equal(np.where(a_nan, 0, actual), np.where(e_nan, 0, expected))


def test_dynamic_quant_matches_reference_rows():
    """Dynamic per-row quant: the oracle against codec.quantize_rows of the
    reference (tests/golden/dynamic.npz; the expectation of the reference's
    tests/test_npu_ops.py:30-50), BF16 and FP16 rows, special values and a
    row below the 1e-12 scale floor included."""
    d = np.load(GOLDEN / "dynamic.npz")
    for name in ("bf16", "f16"):
        data, scale = oracle.dynamic_quant(d[f"{name}_x"], dtype=name)
        np.testing.assert_array_equal(data, d[f"{name}_data"])
        np.testing.assert_array_equal(scale, d[f"{name}_scale"])
