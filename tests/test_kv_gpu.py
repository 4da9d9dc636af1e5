"""GPU parity of the paged HiF8 KV path against the CPU oracle: the fused
static write is byte-exact with quant + pack + slot scatter, the dense
gather-decode is bit-exact, and attention over the HiF8 pages matches the FP64
attention over the BF16-dequantised K/V.

Attention tolerance: max |o - o_ref| <= 1e-2 * max |o_ref| and cosine
similarity > 0.9999 per query row (the reference pins its fused attention at
cosine > 0.999, tests/test_hif8_kv_npu.py:296-332)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._helpers import from_bits

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def _kv():
    from hif8_b200 import kv_cache

    kv_cache.load_ops()
    return kv_cache


def test_kv_write_golden():
    g = np.load(GOLDEN / "kv.npz")
    kv = _kv()
    src = from_bits(g["w_src"], torch.bfloat16).to(DEV)
    scale = torch.from_numpy(g["w_scale"]).to(DEV)
    cache_k = torch.zeros(g["w_cache"].shape, dtype=torch.uint8, device=DEV)
    cache_v = torch.zeros_like(cache_k)
    kv.write_static(src, src, cache_k, cache_v, torch.from_numpy(g["w_slots"]).to(DEV), scale, scale, validate=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache_k.cpu().numpy(), g["w_cache"])
    np.testing.assert_array_equal(cache_v.cpu().numpy(), g["w_cache"])


def test_kv_write_production_shape_across_page_boundary():
    """tokens = 128 + 9, 4 heads x 256, realistic per-head scales (reference
    tests/test_hif8_kv_npu.py:380-551)."""
    kv = _kv()
    tokens, heads, d, block, nblocks = 128 + 9, 4, 256, 128, 4
    gen = torch.Generator().manual_seed(20260822)
    key = (torch.randn(tokens, heads, d, generator=gen) * 3.0).to(torch.bfloat16)
    value = (torch.randn(tokens, heads, d, generator=gen) * 1.5).to(torch.bfloat16)
    ks = np.array([0.9432383179664612, 0.7343872785568237, 0.9391698241233826, 1.1160656213760376], np.float32)
    vs = np.array([0.3244977593421936, 0.416015625, 0.5311850309371948, 0.3086029291152954], np.float32)
    slots = np.arange(tokens, dtype=np.int64) + 128  # start at block 1
    slots[5] = -1
    kc = torch.zeros((nblocks, block, heads, d + 4), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    kv.write_static(key.to(DEV), value.to(DEV), kc, vc, torch.from_numpy(slots).to(DEV),
                    torch.from_numpy(ks).to(DEV), torch.from_numpy(vs).to(DEV), validate=True)
    exp_k = np.zeros(kc.shape, np.uint8)
    exp_v = np.zeros(kc.shape, np.uint8)
    kb = key.contiguous().view(torch.int16).numpy().view(np.uint16)
    vb = value.contiguous().view(torch.int16).numpy().view(np.uint16)
    assert oracle.kv_write(kb, ks, slots, exp_k) == 0
    assert oracle.kv_write(vb, vs, slots, exp_v) == 0
    np.testing.assert_array_equal(kc.cpu().numpy(), exp_k)
    np.testing.assert_array_equal(vc.cpu().numpy(), exp_v)
    # gather + decode of the request's rows is bit-exact with scaled_decode
    table = torch.tensor([[1, 2, 3]], dtype=torch.int32)
    dense = kv.gather_dense(kc, table.to(DEV), [tokens + 128 - 128])
    rows = oracle.gather_kv_rows(exp_k, np.array([1, 2, 3]), tokens, block)
    data, scale = oracle.unpack_kv_rows(rows, d)
    expected = oracle.scaled_decode(data.reshape(-1, d), scale.reshape(-1)).reshape(tokens, heads, d)
    got = dense.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, expected)


def test_kv_write_rejects_out_of_range_slots():
    kv = _kv()
    key = torch.randn(3, 2, 16, dtype=torch.bfloat16, device=DEV)
    kc = torch.zeros((2, 4, 2, 20), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    s = torch.ones(2, device=DEV)
    with pytest.raises(IndexError):
        kv.write_static(key, key, kc, vc, torch.tensor([0, 9, 1], device=DEV), s, s, validate=True)
    # the in-range rows were written, the bad one skipped
    assert int(kc[0, 0].sum()) != 0 and int(kc[0, 1].sum()) != 0


def _make_paged(batch, ctx, kv_heads, d, block, seed, second_scale_every=0):
    """Pages for `batch` requests of ctx[b] keys, scattered over a shuffled
    block table.  With second_scale_every = n, every n-th row (i % n == n - 1)
    is written with a second set of per-head scales."""
    rng = np.random.default_rng(seed)
    blocks_per = [(c + block - 1) // block for c in ctx]
    total_blocks = sum(blocks_per) + 3
    perm = rng.permutation(total_blocks)
    table = np.full((batch, max(blocks_per)), -1, np.int32)
    pos = 0
    for b in range(batch):
        table[b, :blocks_per[b]] = perm[pos:pos + blocks_per[b]]
        pos += blocks_per[b]
    ks = (0.3 + rng.random(kv_heads)).astype(np.float32) / 4.0
    vs = (0.3 + rng.random(kv_heads)).astype(np.float32) / 4.0
    kc = np.zeros((total_blocks, block, kv_heads, d + 4), np.uint8)
    vc = np.zeros_like(kc)
    for b in range(batch):
        kx = rng.standard_normal((ctx[b], kv_heads, d)).astype(np.float32)
        vx = rng.standard_normal((ctx[b], kv_heads, d)).astype(np.float32)
        slots = np.array([table[b, i // block] * block + i % block for i in range(ctx[b])], np.int64)
        if second_scale_every:
            alt = (np.arange(ctx[b]) % second_scale_every) == second_scale_every - 1
            for sel, kscale, vscale in ((~alt, ks, vs), (alt, ks * 1.75, vs * 0.6)):
                if sel.any():
                    oracle.kv_write(oracle.f32_to_bf16_bits(kx[sel]), kscale, slots[sel], kc)
                    oracle.kv_write(oracle.f32_to_bf16_bits(vx[sel]), vscale, slots[sel], vc)
        else:
            oracle.kv_write(oracle.f32_to_bf16_bits(kx), ks, slots, kc)
            oracle.kv_write(oracle.f32_to_bf16_bits(vx), vs, slots, vc)
    return kc, vc, table


def _check_attention(out, expected):
    got = out.float().cpu().numpy()
    err = np.abs(got - expected).max() / max(np.abs(expected).max(), 1e-12)
    assert err <= 1e-2, f"max-rel error {err}"
    g = got.reshape(-1, got.shape[-1]).astype(np.float64)
    e = expected.reshape(-1, expected.shape[-1]).astype(np.float64)
    cos = (g * e).sum(-1) / (np.linalg.norm(g, axis=-1) * np.linalg.norm(e, axis=-1) + 1e-30)
    assert cos.min() > 0.9999, f"min cosine {cos.min()}"


@pytest.mark.parametrize("ctx_len", [512, 4096])
def test_paged_decode_attention_config3(ctx_len):
    """batch 4, 16 query heads, 4 KV heads, head_dim 256, 128-token pages."""
    kv = _kv()
    batch, heads, kv_heads, d, block = 4, 16, 4, 256, 128
    ctx = [ctx_len - 37 * b for b in range(batch)]
    kc, vc, table = _make_paged(batch, ctx, kv_heads, d, block, seed=ctx_len)
    q = oracle.round_bf16(np.random.default_rng(1).standard_normal((batch, heads, d)).astype(np.float32))
    scale = 1.0 / math.sqrt(d)
    expected = oracle.paged_attention(q, kc, vc, table, ctx, block_size=block, scale=scale)
    out = kv.paged_attention(torch.from_numpy(q).to(torch.bfloat16).to(DEV), torch.from_numpy(kc).to(DEV),
                             torch.from_numpy(vc).to(DEV), torch.from_numpy(table).to(DEV), ctx, scale=scale)
    _check_attention(out, expected)


@pytest.mark.parametrize("group", [1, 2, 8])
def test_paged_decode_attention_groups_ragged_lengths_and_second_scale(group):
    """The decode kernel for GQA groups 1, 2 and 8 over requests of 1, 3, 67
    and 700 keys (one key, a partial round, one chunk, several chunks), with
    every fifth row written under a second per-head scale (those rows are off
    the chunk's scaled table and decode with their own scale)."""
    kv = _kv()
    kv_heads, d, block = 2, 256, 32
    heads = kv_heads * group
    ctx = [1, 3, 67, 700]
    kc, vc, table = _make_paged(len(ctx), ctx, kv_heads, d, block, seed=11 + group, second_scale_every=5)
    q = oracle.round_bf16(np.random.default_rng(3 + group).standard_normal((len(ctx), heads, d)).astype(np.float32))
    scale = 1.0 / math.sqrt(d)
    expected = oracle.paged_attention(q, kc, vc, table, ctx, block_size=block, scale=scale)
    out = kv.paged_attention(torch.from_numpy(q).to(torch.bfloat16).to(DEV), torch.from_numpy(kc).to(DEV),
                             torch.from_numpy(vc).to(DEV), torch.from_numpy(table).to(DEV), ctx, scale=scale)
    _check_attention(out, expected)


def test_paged_attention_mixed_prefill_and_decode():
    """Mixed batch: chunked prefill rows and decode rows, right-aligned causal
    mask (reference tests/test_hif8_kv_npu.py:934-1219 scenarios)."""
    kv = _kv()
    heads, kv_heads, d, block = 8, 2, 128, 16
    ctx = [5, 40, 300, 1]
    q_lens = [5, 3, 2, 1]
    kc, vc, table = _make_paged(len(ctx), ctx, kv_heads, d, block, seed=7)
    q = oracle.round_bf16(np.random.default_rng(2).standard_normal((sum(q_lens), heads, d)).astype(np.float32))
    expected = oracle.paged_attention(q, kc, vc, table, ctx, block_size=block, scale=0.125, query_lens=q_lens)
    out = kv.paged_attention(torch.from_numpy(q).to(torch.bfloat16).to(DEV), torch.from_numpy(kc).to(DEV),
                             torch.from_numpy(vc).to(DEV), torch.from_numpy(table).to(DEV), ctx,
                             query_lens=q_lens, scale=0.125)
    _check_attention(out, expected)


def test_paged_attention_matches_reference_attention_fixture():
    g = np.load(GOLDEN / "kv.npz")
    kv = _kv()
    cache = torch.from_numpy(g["w_cache"]).to(DEV)
    q = torch.from_numpy(g["pa_query"]).to(torch.bfloat16)
    out = kv.paged_attention(q.to(DEV), cache, cache, torch.from_numpy(g["pa_table"]).to(DEV),
                             [int(v) for v in g["pa_seq"]], scale=0.25)
    # the reference oracle decodes K/V in FP32 and attends in FP32 on BF16-rounded queries here
    expected = oracle.paged_attention(q.float().numpy(), g["w_cache"], g["w_cache"], g["pa_table"], g["pa_seq"],
                                      block_size=4, scale=0.25)
    _check_attention(out, expected)
    assert np.abs(out.float().cpu().numpy() - g["pa_out"]).max() < 5e-2


def test_kv_write_fp16_source_small_pages():
    """FP16 K/V rows (the reference's float16 serving dtype) written into
    16-token pages: byte-exact with the oracle's quant + pack + scatter."""
    kv = _kv()
    tokens, heads, d, block, nblocks = 53, 4, 256, 16, 6
    gen = torch.Generator().manual_seed(44)
    key = (torch.randn(tokens, heads, d, generator=gen) * 2.0).to(torch.float16)
    value = (torch.randn(tokens, heads, d, generator=gen) * 0.7).to(torch.float16)
    ks = np.array([0.61, 0.45, 0.93, 0.27], np.float32) / 8.0
    vs = np.array([0.33, 0.52, 0.41, 0.76], np.float32) / 8.0
    slots = np.random.default_rng(5).permutation(nblocks * block)[:tokens].astype(np.int64)
    slots[[3, 17]] = -1
    kc = torch.zeros((nblocks, block, heads, d + 4), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    kv.write_static(key.to(DEV), value.to(DEV), kc, vc, torch.from_numpy(slots).to(DEV),
                    torch.from_numpy(ks).to(DEV), torch.from_numpy(vs).to(DEV), validate=True)
    torch.cuda.synchronize()
    kref = np.zeros((nblocks, block, heads, d + 4), np.uint8)
    vref = np.zeros_like(kref)
    kbits = key.view(torch.int16).numpy().view(np.uint16)
    vbits = value.view(torch.int16).numpy().view(np.uint16)
    oracle.kv_write(kbits, ks, slots, kref, dtype="f16")
    oracle.kv_write(vbits, vs, slots, vref, dtype="f16")
    np.testing.assert_array_equal(kc.cpu().numpy(), kref)
    np.testing.assert_array_equal(vc.cpu().numpy(), vref)


def test_paged_decode_small_pages_and_padded_block_tables():
    """The decode kernel (head size 256, GQA group 4) on 16-token pages, one
    to 1000 keys per request, with every block-table entry past a request's
    pages pointing outside the cache: those entries are never read."""
    kv = _kv()
    heads, kv_heads, d, block = 16, 4, 256, 16
    ctx = [1, 17, 250, 1000]
    kc, vc, table = _make_paged(len(ctx), ctx, kv_heads, d, block, seed=91)
    for b, c in enumerate(ctx):
        table[b, (c + block - 1) // block:] = kc.shape[0] + 1000
    q = oracle.round_bf16(np.random.default_rng(9).standard_normal((len(ctx), heads, d)).astype(np.float32))
    scale = 1.0 / math.sqrt(d)
    expected = oracle.paged_attention(q, kc, vc, table, ctx, block_size=block, scale=scale)
    out = kv.paged_attention(torch.from_numpy(q).to(torch.bfloat16).to(DEV), torch.from_numpy(kc).to(DEV),
                             torch.from_numpy(vc).to(DEV), torch.from_numpy(table).to(DEV), ctx, scale=scale)
    _check_attention(out, expected)


def test_paged_decode_head_size_128():
    """Decode rows of head size 128 take the general kernel (GQA group 2)."""
    kv = _kv()
    heads, kv_heads, d, block = 8, 4, 128, 32
    ctx = [7, 64, 333]
    kc, vc, table = _make_paged(len(ctx), ctx, kv_heads, d, block, seed=13, second_scale_every=7)
    q = oracle.round_bf16(np.random.default_rng(4).standard_normal((len(ctx), heads, d)).astype(np.float32))
    scale = 1.0 / math.sqrt(d)
    expected = oracle.paged_attention(q, kc, vc, table, ctx, block_size=block, scale=scale)
    out = kv.paged_attention(torch.from_numpy(q).to(torch.bfloat16).to(DEV), torch.from_numpy(kc).to(DEV),
                             torch.from_numpy(vc).to(DEV), torch.from_numpy(table).to(DEV), ctx, scale=scale)
    _check_attention(out, expected)


@pytest.mark.parametrize("heads,d", [(1, 256), (2, 256), (4, 256), (8, 128), (4, 64), (3, 16), (2, 96), (5, 48)])
@pytest.mark.parametrize("scales", ["calibrated", "pow2", "special"])
def test_kv_write_head_layouts_scales_and_strided_source(heads, d, scales):
    """Every page-row-group size (the warp-per-token write stores 16-byte
    words when heads * (D + 4) is a multiple of 16, 4-byte words otherwise;
    D / 16 not a power of two takes the per-chunk kernel), power-of-two
    scales (the check-free encode), calibrated ones and non-positive /
    non-finite ones (the exact path), K and V read from a fused qkv row
    (token stride > heads * D): byte-exact with the oracle."""
    kv = _kv()
    tokens, block, nblocks = 77, 16, 8
    gen = torch.Generator().manual_seed(heads * 1000 + d + len(scales))
    qkv = (torch.randn(tokens, 3 * heads * d + 8, generator=gen) * 2.5).to(torch.bfloat16)
    qkv[0, heads * d:heads * d + 8] = torch.tensor([float("nan"), float("inf"), -float("inf"), 0.0, -0.0, 1e30,
                                                     -1e-30, 65504.0])
    key = qkv[:, heads * d:2 * heads * d].view(tokens, heads, d)
    value = qkv[:, 2 * heads * d:3 * heads * d].view(tokens, heads, d)
    if scales == "calibrated":
        ks = (key.float().abs().amax(dim=(0, 2)) / 448.0).numpy().astype(np.float32)
        vs = (value.float().abs().amax(dim=(0, 2)) / 32768.0).numpy().astype(np.float32)
    elif scales == "pow2":
        ks = (2.0 ** np.arange(-3, -3 + heads)).astype(np.float32)
        vs = (2.0 ** -np.arange(1, heads + 1)).astype(np.float32)
    else:
        ks = np.array([0.0, -0.5, float("inf"), 3.0e-39, 0.125, 1e30, 0.3, 2.0][:heads] * 2, np.float32)[:heads]
        vs = np.array([float("nan"), 1e-40, 0.25, -2.0, 7.0, 0.5, 1.0, 3.0][:heads] * 2, np.float32)[:heads]
    slots = np.random.default_rng(heads + d).permutation(nblocks * block)[:tokens].astype(np.int64)
    slots[[2, 40]] = -1
    kc = torch.zeros((nblocks, block, heads, d + 4), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    qkv_dev = qkv.to(DEV)
    kd = qkv_dev[:, heads * d:2 * heads * d].view(tokens, heads, d)
    vd = qkv_dev[:, 2 * heads * d:3 * heads * d].view(tokens, heads, d)
    assert kd.stride(0) == 3 * heads * d + 8
    kv.write_static(kd, vd, kc, vc, torch.from_numpy(slots).to(DEV), torch.from_numpy(ks).to(DEV),
                    torch.from_numpy(vs).to(DEV), validate=True)
    torch.cuda.synchronize()
    kref = np.zeros(kc.shape, np.uint8)
    vref = np.zeros_like(kref)
    oracle.kv_write(key.contiguous().view(torch.int16).numpy().view(np.uint16), ks, slots, kref)
    oracle.kv_write(value.contiguous().view(torch.int16).numpy().view(np.uint16), vs, slots, vref)
    np.testing.assert_array_equal(kc.cpu().numpy(), kref)
    np.testing.assert_array_equal(vc.cpu().numpy(), vref)


@pytest.mark.parametrize("pad_bytes", [0, 4096])
def test_block_major_pages_through_the_strided_c_abi(pad_bytes):
    """vLLM's block-major page [num_blocks, 2, block_size, kv_heads, D + 4]
    (K rows then V rows, optionally padded pages): hif8_kv_cache_write_strided
    writes each plane byte-identical to the dense write of the same rows, and
    hif8_paged_attention_strided (decode and prefill batches) returns the
    dense caches' output bit for bit."""
    from hif8_b200 import cabi

    kv = _kv()
    nb, bs, kvh, d, heads = 24, 16, 2, 256, 8
    w = d + 4
    page = 2 * bs * kvh * w
    raw = torch.zeros(nb * (page + pad_bytes), dtype=torch.uint8, device=DEV)
    pages = torch.as_strided(raw, (nb, 2, bs, kvh, w), (page + pad_bytes, bs * kvh * w, kvh * w, w, 1))
    kc = torch.zeros((nb, bs, kvh, w), dtype=torch.uint8, device=DEV)
    vc = torch.zeros_like(kc)
    gen = torch.Generator().manual_seed(77 + pad_bytes)
    table = torch.tensor([[3, 11, 5, 0], [20, 2, 0, 0], [7, 0, 0, 0]], dtype=torch.int32)
    lens = [50, 23, 9]
    slots = torch.tensor([int(table[r, p // bs]) * bs + p % bs for r, n in enumerate(lens) for p in range(n)],
                         dtype=torch.int64)
    key = (torch.randn(len(slots), kvh, d, generator=gen) * 2).to(torch.bfloat16).to(DEV)
    value = torch.randn(len(slots), kvh, d, generator=gen).to(torch.bfloat16).to(DEV)
    ks = torch.tensor([5.0 / 32768, 3.0 / 32768], device=DEV)
    vs = torch.tensor([2.0 / 32768, 4.0 / 32768], device=DEV)
    cabi.kv_cache_write(key, value, ks, vs, slots.to(DEV), pages[:, 0], pages[:, 1])
    kv.write_static(key, value, kc, vc, slots.to(DEV), ks, vs)
    torch.cuda.synchronize()
    assert torch.equal(pages[:, 0], kc) and torch.equal(pages[:, 1], vc)
    table_d, lens_d = table.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV)
    for q_lens in ([1, 1, 1], [7, 1, 4]):
        starts = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32, device=DEV)
        q = torch.randn(sum(q_lens), heads, d, generator=gen).to(torch.bfloat16).to(DEV)
        out = torch.empty_like(q)
        cabi.paged_attention(q, pages[:, 0], pages[:, 1], table_d, lens_d, starts, max(lens), 1.0 / math.sqrt(d), out)
        want = kv.paged_attention(q, kc, vc, table_d, lens, query_lens=q_lens, scale=1.0 / math.sqrt(d))
        torch.cuda.synchronize()
        assert torch.equal(out, want), f"strided pages changed the attention output ({q_lens})"
