"""GPU half of tests/_vllm_attention_cases.py: vLLM ``Attention`` layers on
the HiF8 backend run prefill, decode and mixed (chunked-prefill, padded)
steps through ``Attention.forward`` under vLLM's forward context.  After
every step the cache pages equal the oracle's write of the same rows byte
for byte, and the attention output matches the oracle's FP64 attention over
the oracle's pages (max-rel <= 1e-2 and per-row cosine >= 0.9999, the
tolerance of tests/test_kv_gpu.py), for static scales set on the layer,
static scales read from a checkpoint's hif8_metadata.json, and dynamic
per-row scales.  A cache whose pages vLLM pads (block stride above the page
size) gives bit-identical outputs and pages."""

from __future__ import annotations

import json
import math
import tempfile
from types import SimpleNamespace

import numpy as np
import torch

from _vllm_attention_cases import BS, D, HEADS, KV_HEADS, NUM_BLOCKS
from oracle import oracle

W = D + 4
# request A spans blocks 5, 9; request B blocks 12, 17 (block 0 is vLLM's null block)
TABLES = np.array([[5, 9, 0], [12, 17, 0]], dtype=np.int32)
# (query rows per request, context length per request after the step, padded rows)
STEPS = [((21, 5), (21, 5), 0), ((1, 1), (22, 6), 0), ((1, 14), (23, 20), 3)]


def _slots(query_lens, seq_lens, pad):
    out = []
    for r, (q, s) in enumerate(zip(query_lens, seq_lens)):
        for pos in range(s - q, s):
            out.append(int(TABLES[r, pos // BS]) * BS + pos % BS)
    return np.array(out + [-1] * pad, dtype=np.int64)


def _check_attention(got, expected, what):
    got = got.float().cpu().numpy()
    err = np.abs(got - expected).max() / max(np.abs(expected).max(), 1e-12)
    assert err <= 1e-2, f"{what}: max-rel error {err}"
    g = got.reshape(-1, got.shape[-1]).astype(np.float64)
    e = expected.reshape(-1, expected.shape[-1]).astype(np.float64)
    cos = (g * e).sum(-1) / (np.linalg.norm(g, axis=-1) * np.linalg.norm(e, axis=-1) + 1e-30)
    assert cos.min() > 0.9999, f"{what}: min cosine {cos.min()}"


def _oracle_write(src_bits, slots, cache, scales):
    """The oracle's page write: static per-head scales, or dynamic row
    scales (codes + FP32 scale packed, then copied into the slot)."""
    n = src_bits.shape[0]
    if scales is not None:
        oracle.kv_write(src_bits, scales, slots, cache)
        return
    codes, row_scale = oracle.dynamic_quant(src_bits.reshape(n * KV_HEADS, D))
    rows = oracle.pack_kv_rows(codes.reshape(n, KV_HEADS, D), row_scale.reshape(n, KV_HEADS))
    for i, slot in enumerate(slots[:n]):
        if slot >= 0:
            cache[slot // BS, slot % BS] = rows[i]


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _run_steps(layer, kv, scales, make_common, cfg, seed):
    from vllm.forward_context import set_forward_context

    dev = torch.device("cuda", 0)
    builder = layer.attn_backend.get_builder_cls()(layer.get_kv_cache_spec(cfg), [layer.layer_name], cfg, dev)
    kc = np.zeros((NUM_BLOCKS, BS, KV_HEADS, W), dtype=np.uint8)
    vc = np.zeros_like(kc)
    g = torch.Generator().manual_seed(seed)
    layer.kv_cache = kv
    outs = []
    for query_lens, seq_lens, pad in STEPS:
        n = int(sum(query_lens))
        rows = n + pad
        q = torch.randn(rows, HEADS * D, generator=g).to(torch.bfloat16)
        k = (torch.randn(rows, KV_HEADS * D, generator=g) * 2).to(torch.bfloat16)
        v = torch.randn(rows, KV_HEADS * D, generator=g).to(torch.bfloat16)
        slots = _slots(query_lens, seq_lens, pad)
        md = builder.build(0, make_common(query_lens, seq_lens, TABLES, slots[:n], dev))
        with set_forward_context({layer.layer_name: md}, cfg,
                                 slot_mapping={layer.layer_name: torch.from_numpy(slots).to(dev)}):
            out = layer(q.to(dev), k.to(dev), v.to(dev))
        torch.cuda.synchronize()
        _oracle_write(_bits(k[:n]).reshape(n, KV_HEADS, D), slots, kc, scales and scales[0])
        _oracle_write(_bits(v[:n]).reshape(n, KV_HEADS, D), slots, vc, scales and scales[1])
        assert np.array_equal(kv[:, 0].cpu().numpy(), kc), f"K pages differ after step {query_lens}"
        assert np.array_equal(kv[:, 1].cpu().numpy(), vc), f"V pages differ after step {query_lens}"
        qf = oracle.round_bf16(q[:n].float().numpy().reshape(n, HEADS, D))
        want = oracle.paged_attention(qf, kc, vc, TABLES, list(seq_lens), block_size=BS, scale=1.0 / math.sqrt(D),
                                      query_lens=list(query_lens))
        got = out.view(rows, HEADS, D)
        _check_attention(got[:n], want, f"{layer.layer_name} step {query_lens}")
        assert not got[n:].any(), "padded query rows must be zero"
        outs.append(out.clone())
    return outs


def _cache(padded_bytes=0):
    dev = torch.device("cuda", 0)
    page = 2 * BS * KV_HEADS * W
    stride = page + padded_bytes
    raw = torch.zeros(NUM_BLOCKS * stride, dtype=torch.uint8, device=dev)
    if not padded_bytes:
        return raw.view(NUM_BLOCKS, 2, BS, KV_HEADS, W)
    return torch.as_strided(raw, (NUM_BLOCKS, 2, BS, KV_HEADS, W), (stride, BS * KV_HEADS * W, KV_HEADS * W, W, 1))


def forward_checks(va, cfg, make_layer, make_common):
    # static scales set on the layer, dense and padded pages
    static = make_layer(va, 10)
    ks, vs = [4.0 / 32768, 2.5 / 32768], [3.0 / 32768, 5.0 / 32768]
    static.impl.set_static_kv_scales(ks, vs)
    scales = (np.array(ks, dtype=np.float32), np.array(vs, dtype=np.float32))
    dense = _run_steps(static, _cache(), scales, make_common, cfg, seed=1)
    padded_kv = _cache(padded_bytes=4096)
    padded = _run_steps(static, padded_kv, scales, make_common, cfg, seed=1)
    for a, b in zip(dense, padded):
        assert torch.equal(a, b), "a padded page layout changed the attention output"

    # static scales from a checkpoint's hif8_metadata.json (layer 11 of 12)
    with tempfile.TemporaryDirectory() as ckpt:
        meta = {"format": "W8A8HIF8_STATIC", "kv_cache": {"mode": "static_per_layer_per_head", "layers": {
            "3": {"key_scales": [1.0, 1.0], "value_scales": [1.0, 1.0]},
            "11": {"key_scales": [6.0 / 32768, 1.5 / 32768], "value_scales": [2.0 / 32768, 7.0 / 32768]}}}}
        with open(f"{ckpt}/hif8_metadata.json", "w", encoding="utf-8") as f:
            json.dump(meta, f)
        found = va.checkpoint_kv_scales(SimpleNamespace(model_config=SimpleNamespace(model=ckpt, model_weights="")))
    from_ckpt = make_layer(va, 11)
    from_ckpt.impl._checkpoint_scales = found
    layer11 = meta["kv_cache"]["layers"]["11"]
    _run_steps(from_ckpt, _cache(), (np.array(layer11["key_scales"], dtype=np.float32),
                                     np.array(layer11["value_scales"], dtype=np.float32)), make_common, cfg, seed=2)
    missing = make_layer(va, 12)
    missing.impl._checkpoint_scales = found
    try:
        missing.impl.static_kv_scales(missing, torch.device("cuda", 0))
    except ValueError as e:
        assert "no KV scales for attention layer 12" in str(e)
    else:
        raise AssertionError("a layer without checkpoint scales must be refused")

    # legacy checkpoint: dynamic per-row scales
    dynamic = make_layer(va, 13)
    assert dynamic.impl.static_kv_scales(dynamic, torch.device("cuda", 0)) is None
    _run_steps(dynamic, _cache(), None, make_common, cfg, seed=3)
