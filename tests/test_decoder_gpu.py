"""Glue kernels of the synthetic Qwen3.5-shaped decoder against
torch FP32 restatements of transformers' Qwen3_5 text model
(models/qwen3_5/modeling_qwen3_5.py: Qwen3_5RMSNorm, Qwen3_5MLP,
Qwen3_5Attention's q/k norm + partial rotary + output gate,
Qwen3_5GatedDeltaNet with torch_recurrent_gated_delta_rule), and a reduced
decoder end to end: the HiF8 model tracks its BF16 twin, and a CUDA-graph
decode step reproduces the eager step.

Tolerances: BF16 outputs of FP32 arithmetic, compared with max-abs error
relative to the reference's max |value| (<= 2e-2; the kernels round
intermediates to BF16 where the reference model materialises BF16)."""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _ops():
    from hif8_b200 import kv_cache

    kv_cache.load_ops()
    return torch.ops.hif8_b200


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max()) / max(float(b.abs().max()), 1e-12)


def test_rmsnorm_with_residual():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(5, 4096, device=DEV, generator=g).to(torch.bfloat16)
    res = torch.randn(5, 4096, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(4096, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    out, new_res = ops.rmsnorm(x, res, w, 1e-6, True)
    r = (x + res)  # BF16 residual stream
    assert torch.equal(new_res, r)
    rf = r.float()
    ref = rf * torch.rsqrt(rf.pow(2).mean(-1, keepdim=True) + 1e-6) * (1.0 + w.float())
    assert _rel(out, ref) <= 1e-2
    out2, same = ops.rmsnorm(x, None, w, 1e-6, False)
    xf = x.float()
    assert same.data_ptr() == x.data_ptr()
    assert _rel(out2, xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()) <= 1e-2


def test_silu_mul_and_gate_mul():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(1)
    gu = torch.randn(3, 2 * 1536, device=DEV, generator=g).to(torch.bfloat16)
    out = ops.silu_mul(gu)
    ref = torch.nn.functional.silu(gu[:, :1536].float()) * gu[:, 1536:].float()
    assert _rel(out, ref) <= 1e-2
    x = torch.randn(7, 4096, device=DEV, generator=g).to(torch.bfloat16)
    gate = torch.randn(7, 4096, device=DEV, generator=g).to(torch.bfloat16)
    assert _rel(ops.gate_mul(x, gate), x.float() * torch.sigmoid(gate.float())) <= 1e-2


def _rope_ref(x, pos, rotary_dim, theta):
    half = rotary_dim // 2
    inv = theta ** (-torch.arange(half, device=x.device, dtype=torch.float32) * 2 / rotary_dim)
    ang = pos.float()[:, None, None] * inv  # [tokens, 1, half]
    cos, sin = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :half], x[..., half:rotary_dim]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, x[..., rotary_dim:]], dim=-1)


def test_attn_prep_norm_rope_gate():
    ops = _ops()
    heads, kvh, hd, rot, theta = 4, 2, 256, 64, 1.0e7
    tokens = 6
    g = torch.Generator(device=DEV).manual_seed(2)
    qkv = torch.randn(tokens, (2 * heads + 2 * kvh) * hd, device=DEV, generator=g).to(torch.bfloat16)
    pos = torch.tensor([0, 1, 5, 77, 511, 700], dtype=torch.int32, device=DEV)
    qw = (torch.randn(hd, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    kw = (torch.randn(hd, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    q, gate, k, v = ops.attn_prep(qkv, pos, qw, kw, heads, kvh, hd, rot, 1e-6, theta)
    qg = qkv.float()[:, :heads * 2 * hd].view(tokens, heads, 2 * hd)
    q_raw, g_raw = qg[..., :hd], qg[..., hd:]
    k_raw = qkv.float()[:, heads * 2 * hd:heads * 2 * hd + kvh * hd].view(tokens, kvh, hd)
    v_raw = qkv[:, heads * 2 * hd + kvh * hd:].view(tokens, kvh, hd)

    def norm(x, w):
        return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + w.float())).to(torch.bfloat16).float()

    assert _rel(q, _rope_ref(norm(q_raw, qw), pos, rot, theta)) <= 2e-2
    assert _rel(k, _rope_ref(norm(k_raw, kw), pos, rot, theta)) <= 2e-2
    assert torch.equal(gate.view(tokens, heads, hd), g_raw.to(torch.bfloat16))
    assert torch.equal(v, v_raw)


def _gdn_ref(proj, T, hk, hv, conv_w, a_log, dt_bias, norm_w, conv_state, rec_state, eps):
    """FP32 restatement of the gated delta net (conv -> SiLU -> l2norm ->
    recurrent delta rule -> gated RMSNorm) for T tokens per sequence."""
    d = 128
    B = proj.shape[0] // T
    C = 2 * hk * d + hv * d
    x = proj.float().view(B, T, -1)
    qkv, z = x[..., :C], x[..., C:C + hv * d]
    b, a = x[..., C + hv * d:C + hv * d + hv], x[..., C + hv * d + hv:]
    full = torch.cat([conv_state.transpose(1, 2), qkv], dim=1)  # [B, 3 + T, C]
    w = conv_w.float()
    y = sum(full[:, i:i + T, :] * w[:, i] for i in range(4))
    y = torch.nn.functional.silu(y)
    new_conv = full[:, -3:, :].transpose(1, 2).contiguous()
    q = y[..., :hk * d].view(B, T, hk, d)
    k = y[..., hk * d:2 * hk * d].view(B, T, hk, d)
    v = y[..., 2 * hk * d:].view(B, T, hv, d)
    q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) / math.sqrt(d)
    k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
    q = q.repeat_interleave(hv // hk, dim=2)
    k = k.repeat_interleave(hv // hk, dim=2)
    beta = torch.sigmoid(b)
    g = -a_log.float().exp() * torch.nn.functional.softplus(a + dt_bias.float())
    S = rec_state.clone()
    outs = []
    for t in range(T):
        S = S * g[:, t].exp()[..., None, None]
        kv_mem = torch.einsum("bhij,bhi->bhj", S, k[:, t])
        delta = (v[:, t] - kv_mem) * beta[:, t, :, None]
        S = S + k[:, t][..., :, None] * delta[..., None, :]
        outs.append(torch.einsum("bhij,bhi->bhj", S, q[:, t]))
    o = torch.stack(outs, dim=1)  # [B, T, hv, d]
    on = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()
    out = on * torch.nn.functional.silu(z.view(B, T, hv, d))
    return out.reshape(B * T, hv * d), new_conv, S


def _per_head_conv_state(state, hk, hv, d=128):
    """[B, 2 hk d + hv d, 3] (one history per projection channel) -> the
    kernel's [B, hv, 3, d, 3] (per value head: its key head's q and k
    channels and its own v channels)."""
    ratio = hv // hk
    heads = []
    for vh in range(hv):
        kh = vh // ratio
        q = state[:, kh * d:(kh + 1) * d]
        k = state[:, hk * d + kh * d:hk * d + (kh + 1) * d]
        v = state[:, 2 * hk * d + vh * d:2 * hk * d + (vh + 1) * d]
        heads.append(torch.stack([q, k, v], dim=1))
    return torch.stack(heads, dim=1).contiguous()


@pytest.mark.parametrize("T,B", [(1, 2), (7, 2), (1, 5)])
def test_gated_delta_net_matches_recurrent_reference(T, B):
    ops = _ops()
    hk, hv, d = 2, 4, 128
    g = torch.Generator(device=DEV).manual_seed(3 + T + B)
    C = 2 * hk * d + hv * d
    proj = torch.randn(B * T, C + hv * d + 2 * hv, device=DEV, generator=g).to(torch.bfloat16)
    conv_w = (torch.rand(C, 4, device=DEV, generator=g) - 0.5).to(torch.bfloat16)
    a_log = torch.rand(hv, device=DEV, generator=g).mul(15).add(0.1).log()
    dt_bias = torch.ones(hv, device=DEV)
    norm_w = (1 + 0.1 * torch.randn(d, device=DEV, generator=g)).to(torch.bfloat16)
    conv_state = torch.randn(B, C, 3, device=DEV, generator=g)
    rec_state = torch.randn(B, hv, d, d, device=DEV, generator=g) * 0.1
    ref_out, ref_conv, ref_S = _gdn_ref(proj, T, hk, hv, conv_w, a_log, dt_bias, norm_w, conv_state, rec_state,
                                        1e-6)
    cs, rs = _per_head_conv_state(conv_state, hk, hv), rec_state.clone()
    out = ops.gdn(proj, T, hk, hv, conv_w, a_log, dt_bias, norm_w, cs, rs, 1e-6)
    assert _rel(out, ref_out) <= 2e-2
    assert _rel(rs, ref_S) <= 1e-3
    assert torch.allclose(cs, _per_head_conv_state(ref_conv, hk, hv), rtol=0, atol=1e-6)


def _hif8_weight(n, k, seed):
    from hif8_b200 import scheme

    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn(n, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    data, scale = scheme.quantize_weight_rows(w)
    return data, scale, torch.tensor([3.0 / 32768.0], device=DEV)


@pytest.mark.parametrize("m", [1, 4])
def test_glue_linear_silu_and_gate_equal_the_separate_kernels(m):
    """SiLU-mul and sigmoid-gate fused into the GEMV prologue give the same
    bits as the glue kernel followed by the fused quant + GEMV."""
    from hif8_b200 import native

    ops = _ops()
    k, n = 1024, 768
    data, scale, fixed = _hif8_weight(n, k, 11 + m)
    g = torch.Generator(device=DEV).manual_seed(12 + m)
    gu = torch.randn(m, 2 * k, device=DEV, generator=g).to(torch.bfloat16)
    fused, _ = ops.glue_linear(gu, None, None, 1, 0.0, False, data, fixed, scale)
    ref = native.soft_static_fused_linear(ops.silu_mul(gu), data, fixed, scale, None, output_dtype=torch.bfloat16)
    assert torch.equal(fused, ref)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    gate = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    fused, _ = ops.glue_linear(x, gate, None, 2, 0.0, False, data, fixed, scale)
    ref = native.soft_static_fused_linear(ops.gate_mul(x, gate), data, fixed, scale, None, output_dtype=torch.bfloat16)
    assert torch.equal(fused, ref)


@pytest.mark.parametrize("m,n", [(1, 1024), (3, 1024), (1, 12352)])
def test_glue_linear_rmsnorm_matches_norm_then_linear(m, n):
    """Residual + RMSNorm fused into the GEMV prologue: the new residual
    stream is bit-exact; the projection matches RMSNorm followed by the fused
    quant + GEMV within 1e-2 of max |y| (the sum of squares is reduced in
    another order, so an activation can land on a neighbouring code)."""
    from hif8_b200 import native

    ops = _ops()
    k = 4096  # n = 12352: the gated-delta-net input projection of the 9B shape
    data, scale, fixed = _hif8_weight(n, k, 21 + m)
    g = torch.Generator(device=DEV).manual_seed(22 + m)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    res = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(k, device=DEV, generator=g) * 0.1).to(torch.bfloat16)
    fused, new_res = ops.glue_linear(x, res, w, 3, 1e-6, True, data, fixed, scale)
    h, ref_res = ops.rmsnorm(x, res, w, 1e-6, True)
    ref = native.soft_static_fused_linear(h, data, fixed, scale, None, output_dtype=torch.bfloat16)
    assert torch.equal(new_res, ref_res)
    assert _rel(fused, ref) <= 1e-2
    fused0, same = ops.glue_linear(x, None, w, 3, 1e-6, True, data, fixed, scale)
    h0, _ = ops.rmsnorm(x, None, w, 1e-6, True)
    assert same.data_ptr() == x.data_ptr()
    ref0 = native.soft_static_fused_linear(h0, data, fixed, scale, None, output_dtype=torch.bfloat16)
    assert _rel(fused0, ref0) <= 1e-2


def _tiny_cfg():
    from hif8_b200.decoder import DecoderConfig

    return DecoderConfig(hidden=512, intermediate=1024, layers=4, heads=4, kv_heads=2, head_dim=256,
                         lin_k_heads=2, lin_v_heads=4, vocab=1024)


def test_tiny_decoder_hif8_tracks_bf16_twin_and_graph_matches_eager():
    from hif8_b200.decoder import Decoder, calibrate

    cfg = _tiny_cfg()
    calib = calibrate(cfg, DEV, seed=5, tokens=48)
    hif8 = Decoder(cfg, "hif8", DEV, seed=5, max_batch=2, max_ctx=160, calibration=calib)
    twin = Decoder(cfg, "bf16", DEV, seed=5, max_batch=2, max_ctx=160)
    g = torch.Generator(device=DEV).manual_seed(9)
    prompt = torch.randint(0, cfg.vocab, (2, 40), device=DEV, generator=g)
    positions = torch.arange(40, dtype=torch.int32, device=DEV).repeat(2)
    lens = torch.full((2,), 40, dtype=torch.int32, device=DEV)
    with torch.no_grad():
        lh = hif8.forward(prompt.reshape(-1), positions, 2, 40, lens, hif8._slots(2, positions))
        lb = twin.forward(prompt.reshape(-1), positions, 2, 40, lens, None)
    # W8A8KV8 with at most 3 mantissa bits per code: the quantisation noise of
    # 4 random layers leaves the logits at cosine ~0.98 of the BF16 twin; a
    # wiring error (wrong slice, scale or cache row) drops it far lower
    cos = torch.nn.functional.cosine_similarity(lh, lb, dim=-1)
    assert float(cos.min()) > 0.95, f"HiF8 vs BF16 logits cosine {cos.tolist()}"

    # a decode step with the glue fused into the GEMV prologues tracks the
    # step with separate glue kernels
    hif8.reset()
    first = hif8.prefill(prompt)
    state = [t.clone() for t in hif8.conv_state + hif8.rec_state if t is not None]
    pos = torch.full((2,), 40, dtype=torch.int32, device=DEV)
    policy = hif8.fuse_glue, hif8.fuse_glue_max_rows
    with torch.no_grad():
        hif8.fuse_glue, hif8.fuse_glue_max_rows = {"rmsnorm", "silu_mul", "gate_mul"}, 8
        fused = hif8.forward(first, pos, 2, 1, pos + 1, hif8._slots(2, pos))
        for t, s0 in zip([t for t in hif8.conv_state + hif8.rec_state if t is not None], state):
            t.copy_(s0)
        hif8.fuse_glue = set()
        plain = hif8.forward(first, pos, 2, 1, pos + 1, hif8._slots(2, pos))
    hif8.fuse_glue, hif8.fuse_glue_max_rows = policy
    cos = torch.nn.functional.cosine_similarity(fused, plain, dim=-1)
    assert float(cos.min()) > 0.999, f"fused vs separate glue logits cosine {cos.tolist()}"

    # one decode step: CUDA graph replay == eager step, from the same state
    # (batch 1 runs the fused residual + RMSNorm GEMV prologues)
    for model, batch in ((hif8, 2), (hif8, 1), (twin, 2)):
        graph, tokens, pos = model.decode_graph(batch)
        model.reset()
        first = model.prefill(prompt[:batch])
        state = [t.clone() for t in model.conv_state + model.rec_state if t is not None]
        tokens.copy_(first)
        pos.fill_(40)
        graph.replay()
        torch.cuda.synchronize()
        graph_tokens = tokens.clone()
        for t, s in zip([t for t in model.conv_state + model.rec_state if t is not None], state):
            t.copy_(s)
        e_tokens = first.clone()
        e_pos = torch.full((batch,), 40, dtype=torch.int32, device=DEV)
        with torch.no_grad():
            model._decode_step(batch, e_tokens, e_pos)
        assert torch.equal(graph_tokens, e_tokens), (model.mode, batch)
        model.release_graphs()
