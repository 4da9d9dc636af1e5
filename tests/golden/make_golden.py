"""Generate the golden fixtures in this folder from the REFERENCE plugin.

Run once in a container where the reference project is importable:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own CPU code (``vllm_ascend_hif8.codec``,
``torch_codec``, ``calibration``, ``kv_cache``, ``reference``) from
``<reference>/src`` and records its outputs on seeded inputs as small ``.npz``
files.  The GPU box never runs this script; tests only read the ``.npz``.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _f16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.float16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main(reference_root: str) -> None:
    sys.path.insert(0, str(Path(reference_root) / "src"))
    from vllm_ascend_hif8 import codec, torch_codec, calibration, kv_cache, reference

    # ------------------------------------------------------------- codec
    decode = np.array(codec.ASCEND_DECODE_TABLE, dtype=np.float32)
    decode_bf16 = np.array([codec.decode_ascend_bf16_bits_arithmetic(b) for b in range(256)], dtype=np.uint16)
    lut4096 = np.array(torch_codec.FLOAT32_ENCODE_LUT, dtype=np.uint8)
    positive_values = np.array(codec.POSITIVE_VALUES, dtype=np.float64)
    positive_codes = np.array(codec.POSITIVE_CODES, dtype=np.uint8)

    rng = np.random.default_rng(20261201)
    special = [0.0, -0.0, math.nan, math.inf, -math.inf, codec.UNDERFLOW_TIE,
               math.nextafter(codec.UNDERFLOW_TIE, 0.0), codec.OVERFLOW_TIE,
               math.nextafter(codec.OVERFLOW_TIE, 0.0), codec.MAX_FINITE, -codec.MAX_FINITE,
               1.0625, -1.0625, 1.0, 1.125, 2.0**-22, 2.0**-16, 1.5 * 2.0**-16, 2.0**-15, 65536.0, 1e20]
    # ties between neighbouring codes and their FP32 neighbours
    tie_values = []
    for lo, hi in zip(codec.POSITIVE_VALUES[:-1], codec.POSITIVE_VALUES[1:]):
        mid = np.float32((lo + hi) / 2.0)
        tie_values += [float(mid), float(np.nextafter(mid, np.float32(0))), float(np.nextafter(mid, np.float32(np.inf)))]
    random_bits = rng.integers(0, 2**32, size=20000, dtype=np.uint64).astype(np.uint32)
    random_vals = random_bits.view(np.float32)
    normal_vals = (rng.standard_normal(4000) * np.exp2(rng.integers(-26, 18, size=4000))).astype(np.float32)
    enc_inputs = np.concatenate([
        np.array(special, dtype=np.float32), np.array(tie_values, dtype=np.float32), random_vals, normal_vals,
    ]).astype(np.float32)
    enc_scalar = np.array([codec.encode_ascend(float(v)) for v in enc_inputs], dtype=np.uint8)
    enc_tensor = torch_codec.encode_tensor(torch.from_numpy(enc_inputs.copy())).numpy().astype(np.uint8)
    np.savez_compressed(
        HERE / "codec.npz", decode=decode, decode_bf16=decode_bf16, lut4096=lut4096,
        positive_values=positive_values, positive_codes=positive_codes,
        enc_inputs=enc_inputs, enc_scalar=enc_scalar, enc_tensor=enc_tensor,
    )

    # ------------------------------------------------------ static quant
    cases = {}
    # (reference tests/test_npu_ops.py:52-75) special rows, per-head scales
    rows = torch.tensor(
        [[0.0, 1.0, -2.0, 4.0, 1.0e20], [0.25, -0.5, 1.0, -4.0, -1.0e20],
         [float("nan"), float("inf"), -float("inf"), 0.0, 2.0],
         [2.0**-12, -(2.0**-11), 2.0**-10, -(2.0**-9), 1.0]], dtype=torch.bfloat16).reshape(2, 2, 5)
    fixed = torch.tensor([0.5, 2.0], dtype=torch.float32)
    data, _ = calibration.static_quantize_tensor(rows, fixed, group_axis=1)
    cases["special"] = (_bf16_bits(rows).reshape(4, 5), "bf16", fixed.numpy(), data.numpy().reshape(4, 5))
    # (reference tests/test_npu_ops.py:565-605) saturation of finite outliers
    sat = torch.zeros((1, 64), dtype=torch.bfloat16)
    sat[0, :6] = torch.tensor([1.0e20, -1.0e20, 32768.0, -32768.0, 65536.0, -65536.0], dtype=torch.bfloat16)
    one = torch.ones(1, dtype=torch.float32)
    data, _ = calibration.static_quantize_tensor(sat, one)
    cases["saturate"] = (_bf16_bits(sat), "bf16", one.numpy(), data.numpy())
    # (reference tests/test_hif8_kv_npu.py:380-440) realistic per-head KV scales
    g = torch.Generator().manual_seed(20260822)
    key = (torch.randn(37, 4, 256, generator=g) * 3.0).to(torch.bfloat16)
    key_scale = torch.tensor([0.9432383179664612, 0.7343872785568237, 0.9391698241233826, 1.1160656213760376])
    data, _ = calibration.static_quantize_tensor(key, key_scale, group_axis=1)
    cases["kv_heads"] = (_bf16_bits(key).reshape(-1, 256), "bf16", key_scale.numpy(), data.numpy().reshape(-1, 256))
    # random activations, scalar input_scale = absmax / 32768
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4, 4096, generator=g).to(torch.bfloat16)
    calib = torch.randn(4, 4096, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    input_scale = (calib.float().abs().amax() / 32768.0).reshape(1)
    data, _ = calibration.static_quantize_tensor(x, input_scale)
    cases["cfg0_act"] = (_bf16_bits(x), "bf16", input_scale.numpy().astype(np.float32), data.numpy())
    # FP16 input
    xh = (torch.randn(3, 37, generator=g) * 100).to(torch.float16)
    s = torch.tensor([0.37], dtype=torch.float32)
    data, _ = calibration.static_quantize_tensor(xh, s)
    cases["fp16"] = (_f16_bits(xh), "f16", s.numpy(), data.numpy())
    # exhaustive: every BF16 pattern x three scales
    all_bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    all_bf16 = torch.from_numpy(all_bits.view(np.int16).copy()).view(torch.bfloat16).reshape(256, 256)
    for name, sv in (("exh_1", 1.0), ("exh_small", 3.0517578125e-05 * 1.37), ("exh_odd", 0.7343872785568237)):
        s = torch.tensor([sv], dtype=torch.float32)
        data, _ = calibration.static_quantize_tensor(all_bf16, s)
        cases[name] = (all_bits.reshape(256, 256), "bf16", s.numpy(), data.numpy())
    payload = {}
    for name, (xb, dt, sc, out) in cases.items():
        payload[f"{name}__x"] = xb
        payload[f"{name}__dtype"] = np.array(dt)
        payload[f"{name}__scale"] = np.asarray(sc, dtype=np.float32)
        payload[f"{name}__out"] = out.astype(np.uint8)
    np.savez_compressed(HERE / "static_quant.npz", **payload)

    # ------------------------------------------------------ scaled decode
    # (reference tests/test_npu_ops.py:105-123)
    lut = torch.tensor(codec.ASCEND_DECODE_TABLE, dtype=torch.float32)
    gen = torch.Generator().manual_seed(42)
    scales = torch.cat((torch.tensor([0.0, -0.0, 1.0, -1.0, 0.1, 1.00390625, 2.0**-20, 2.0**20,
                                      float("inf"), float("nan")]), torch.rand(54, generator=gen) * 0.02))
    payload = {"scales": scales.numpy()}
    for k in (31, 37, 256):
        codes = ((torch.arange(scales.numel() * k).reshape(-1, k) * 73) % 256).to(torch.uint8)
        expected = (lut[codes.long()] * scales[:, None]).to(torch.bfloat16)
        payload[f"k{k}__codes"] = codes.numpy()
        payload[f"k{k}__out"] = _bf16_bits(expected)
    np.savez_compressed(HERE / "scaled_decode.npz", **payload)

    # ----------------------------------------------------------------- KV
    payload = {}
    values = torch.tensor([[[-2.0, -1.0, 0.0, 1.0], [0.25, 0.5, 0.75, 1.0]],
                           [[3.0, -1.0, 0.0, 2.0], [0.0, 0.0, 0.0, 0.0]]], dtype=torch.float32)
    data, scale = kv_cache.quantize_kv_rows(values)
    payload["rt_values"], payload["rt_data"], payload["rt_scale"] = values.numpy(), data.numpy(), scale.numpy()
    payload["rt_packed"] = kv_cache.pack_kv_rows(data, scale).numpy()
    # static write path: quant per head + pack + scatter by slot mapping
    gen = torch.Generator().manual_seed(7)
    tokens, heads, dim, block, nblocks = 11, 4, 32, 4, 5
    src = (torch.randn(tokens, heads, dim, generator=gen) * 2).to(torch.bfloat16)
    head_scale = torch.tensor([0.5, 0.75, 1.25, 0.3], dtype=torch.float32)
    slots = torch.tensor([3, 0, -1, 17, 8, 9, 10, -1, 19, 4, 1], dtype=torch.int64)
    q, _ = calibration.static_quantize_tensor(src.reshape(-1, dim), head_scale.repeat(tokens), group_axis=0)
    packed = kv_cache.pack_kv_rows(q.reshape(tokens, heads, dim), head_scale.repeat(tokens).reshape(tokens, heads))
    cache = torch.zeros((nblocks, block, heads, dim + 4), dtype=torch.uint8)
    kv_cache.scatter_kv_rows(cache, packed, slots, block_size=block)
    payload["w_src"], payload["w_scale"], payload["w_slots"] = _bf16_bits(src), head_scale.numpy(), slots.numpy()
    payload["w_cache"] = cache.numpy()
    # paged attention reference over that cache (K and V share it here)
    q_rows = torch.randn(3, 8, dim, generator=gen)
    table = torch.tensor([[0, 2, 4], [1, 3, 0], [4, 2, 1]], dtype=torch.int32)
    seq = [7, 12, 5]
    out = kv_cache.paged_attention_reference(q_rows, cache, cache, table, seq, block_size=block, scale=0.25)
    payload["pa_query"], payload["pa_table"] = q_rows.numpy(), table.numpy()
    payload["pa_seq"], payload["pa_out"] = np.array(seq, dtype=np.int64), out.numpy()
    np.savez_compressed(HERE / "kv.npz", **payload)

    # ------------------------------------------------------------- linear
    payload = {}
    act = codec.quantize_rows([[1.0, 0.5], [-1.0, 0.25]])
    wq = codec.quantize_rows([[1.0, 1.0], [0.5, -1.0]])
    payload["k22_a"], payload["k22_as"] = np.array(act.data, np.uint8), np.array(act.scale, np.float32)
    payload["k22_w"], payload["k22_ws"] = np.array(wq.data, np.uint8), np.array(wq.scale, np.float32)
    payload["k22_bias"] = np.array([0.25, -0.5], np.float32)
    payload["k22_out"] = np.array(reference.linear_u8_u8(act, wq, bias=[0.25, -0.5]), np.float64)
    rows_, channels, k = 3, 17, 37
    act = codec.quantize_rows([[((r * 7 + c * 3) % 17 - 8) / 4.0 for c in range(k)] for r in range(rows_)])
    wq = codec.quantize_rows([[((r * 5 + c * 11) % 19 - 9) / 5.0 for c in range(k)] for r in range(channels)])
    bias = [((c * 3) % 11 - 5) / 8.0 for c in range(channels)]
    payload["t_a"], payload["t_as"] = np.array(act.data, np.uint8), np.array(act.scale, np.float32)
    payload["t_w"], payload["t_ws"] = np.array(wq.data, np.uint8), np.array(wq.scale, np.float32)
    payload["t_bias"] = np.array(bias, np.float32)
    payload["t_out"] = np.array(reference.linear_u8_u8(act, wq, bias), np.float64)
    # weight row quantisation, scale = row amax / 32768 (configs[0] weights)
    wsrc = (torch.randn(16, 64, generator=torch.Generator().manual_seed(0)) * 0.02).to(torch.bfloat16)
    wdata, wscale = torch_codec.quantize_tensor_rows(wsrc, scale_factor=codec.MAX_FINITE)
    payload["wq_src"], payload["wq_data"], payload["wq_scale"] = _bf16_bits(wsrc), wdata.numpy(), wscale.numpy()
    np.savez_compressed(HERE / "linear.npz", **payload)
    write_embedding(codec)
    write_dynamic(codec)
    print("golden fixtures written to", HERE)


def write_embedding(codec) -> None:
    """embedding.npz: the W8A8HIF8_SOFT token-embedding lookup.  The
    reference's method (src/vllm_ascend_hif8/scheme.py:120-131) cannot be
    imported here (it needs vllm_ascend), so its four tensor operations are
    run as written there -- index_select of rows and scales, the BF16 decode
    table of codec.ASCEND_DECODE_TABLE, a BF16 product -- on the reference
    codec's table."""
    lut = torch.tensor(codec.ASCEND_DECODE_TABLE, dtype=torch.bfloat16)

    def lookup(weight, scale, ids):
        flat = ids.reshape(-1)
        rows = torch.index_select(weight, 0, flat)
        scales = torch.index_select(scale.reshape(-1), 0, flat)
        out = lut[rows.long()] * scales.to(torch.bfloat16).unsqueeze(-1)
        return out.reshape(*ids.shape, weight.shape[1])

    payload = {}
    # the known answer of the reference's tests/test_embedding.py:12-47
    values = [[-1.0, -0.5, 0.0, 0.5], [-0.5, 0.0, 0.5, 1.0], [0.25, -0.25, 0.75, -0.75]]
    w = torch.tensor([[codec.encode_ascend(v) for v in row] for row in values], dtype=torch.uint8)
    ws = torch.tensor([[2.0], [3.0], [4.0]], dtype=torch.float32)
    ids = torch.tensor([[2, 0], [1, 2]], dtype=torch.int64)
    payload["ka_w"], payload["ka_ws"], payload["ka_ids"] = w.numpy(), ws.numpy(), ids.numpy()
    payload["ka_out"] = _bf16_bits(lookup(w, ws, ids))
    # seeded rows with every code (NaN and Inf included) and FP32 row scales
    # that are not BF16 values (amax / 32768 of N(0, 0.02) rows, as exported)
    g = torch.Generator().manual_seed(7)
    for name, vocab, hidden in (("v", 96, 64), ("s", 40, 36)):
        w = torch.randint(0, 256, (vocab, hidden), generator=g, dtype=torch.int64).to(torch.uint8)
        ws = ((torch.randn(vocab, 64, generator=g) * 0.02).abs().amax(-1) / 32768.0).reshape(-1, 1)
        ids = torch.randint(0, vocab, (5, 7), generator=g, dtype=torch.int64)
        payload[f"{name}_w"], payload[f"{name}_ws"], payload[f"{name}_ids"] = w.numpy(), ws.numpy(), ids.numpy()
        payload[f"{name}_out"] = _bf16_bits(lookup(w, ws, ids))
    np.savez_compressed(HERE / "embedding.npz", **payload)


def write_dynamic(codec) -> None:
    """Dynamic per-row quant (W8A8HIF8_SOFT activations): codec.quantize_rows
    (choose_row_scale + encode_ascend of x / scale in double precision), the
    expectation of the reference's tests/test_npu_ops.py:30-50, on the rows
    of that test, seeded BF16 / FP16 rows of several magnitudes, a row of
    values below the 1e-12 scale floor, an all-zero row and rows with
    NaN / Inf."""
    g = torch.Generator().manual_seed(11)
    special = torch.tensor([[0.0, 1.0, -2.0, 4.0] * 12,
                            [0.25, -0.5, 1.0, -4.0] * 12,
                            [float("nan"), float("inf"), -float("inf"), 0.0] * 12,
                            [2.0**-12, -(2.0**-11), 2.0**-10, -(2.0**-9)] * 12])
    randn = torch.randn(12, 48, generator=g) * torch.tensor([1e-3, 1e-1, 1.0, 30.0, 1e3, 3e4] * 2).reshape(-1, 1)
    tiny = torch.randn(1, 48, generator=g) * 1e-14
    zero = torch.zeros(1, 48)
    mixed = torch.randn(2, 48, generator=g)
    mixed[0, 5] = float("inf")
    mixed[1, 17] = float("nan")
    rows = torch.cat([special, randn, tiny, zero, mixed])
    payload = {}
    for name, bits_fn, dtype in (("bf16", _bf16_bits, torch.bfloat16), ("f16", _f16_bits, torch.float16)):
        src = rows.to(dtype)
        q = codec.quantize_rows(src.float().tolist())
        payload[f"{name}_x"] = bits_fn(src)
        payload[f"{name}_data"] = np.array(q.data, dtype=np.uint8)
        payload[f"{name}_scale"] = np.array(q.scale, dtype=np.float32)
    np.savez_compressed(HERE / "dynamic.npz", **payload)


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the reference checkout> [dynamic]")
    if len(sys.argv) == 3:  # one fixture only
        sys.path.insert(0, str(Path(sys.argv[1]) / "src"))
        from vllm_ascend_hif8 import codec

        {"dynamic": write_dynamic}[sys.argv[2]](codec)
    else:
        main(sys.argv[1])
