"""Checks of the vLLM adapter (hif8_b200.vllm_adapter) on real vLLM layers,
run as a separate process by tests/test_vllm_adapter_cpu.py (mode ``cpu``:
construction, weight loading, parameter contracts) and
tests/test_vllm_adapter_gpu.py (mode ``gpu``: the same plus forward passes
through vLLM's layers against hif8_b200.scheme and the embedding against
the oracle).  vLLM's model-parallel state (gloo, world size 1) lives only in
this process.  Exits non-zero on the first failed check."""

from __future__ import annotations

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "gcc-hif8-quantized-from-qwen3.5-9b_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

STATIC, SOFT = "W8A8HIF8_STATIC", "W8A8HIF8_SOFT"
HIDDEN, HEAD, HEADS, KV_HEADS, INTER, VOCAB = 256, 64, 4, 2, 512, 128


def _desc():
    d = {}
    for c in ("q_proj", "k_proj", "v_proj", "o_proj"):
        d[f"model.language_model.layers.0.self_attn.{c}.weight"] = STATIC
    for c in ("gate_proj", "up_proj", "down_proj"):
        d[f"model.language_model.layers.0.mlp.{c}.weight"] = STATIC
    for c in ("in_proj_qkv", "in_proj_z", "out_proj"):
        d[f"model.language_model.layers.1.linear_attn.{c}.weight"] = SOFT
    d["model.language_model.layers.1.linear_attn.in_proj_b.weight"] = "FLOAT"
    d["model.language_model.layers.1.linear_attn.in_proj_a.weight"] = "FLOAT"
    d["model.language_model.layers.2.self_attn.q_proj.weight"] = STATIC   # mixed fused module
    d["model.language_model.layers.2.self_attn.k_proj.weight"] = SOFT
    d["model.language_model.layers.2.self_attn.v_proj.weight"] = STATIC
    d["model.language_model.embed_tokens.weight"] = SOFT
    return d


def _expect_raises(exc, fn, match):
    try:
        fn()
    except exc as e:
        assert match in str(e), f"expected {match!r} in {e!r}"
        return
    raise AssertionError(f"expected {exc.__name__} ({match})")


def main(mode: str) -> None:
    from vllm.config import DeviceConfig, VllmConfig, set_current_vllm_config
    from vllm.distributed import init_distributed_environment, initialize_model_parallel
    from vllm.model_executor.layers.linear import (
        MergedColumnParallelLinear,
        QKVParallelLinear,
        RowParallelLinear,
        UnquantizedLinearMethod,
    )
    from vllm.model_executor.layers.quantization import get_quantization_config
    from vllm.model_executor.layers.vocab_parallel_embedding import VocabParallelEmbedding

    from hif8_b200 import scheme
    from hif8_b200 import vllm_adapter as va

    va.register()
    va.register()  # idempotent
    assert get_quantization_config("hif8") is va.Hif8Config
    gpu = mode == "gpu"
    dev = torch.device("cuda", 0) if gpu else torch.device("cpu")
    if gpu:
        torch.cuda.set_device(0)
        torch.set_default_device(dev)
    g = torch.Generator().manual_seed(7)
    cfg = va.Hif8Config.from_config(_desc())
    assert va.Hif8Config.get_config_filenames() == ["quant_model_description.json"]
    port = 29700 + os.getpid() % 200
    with set_current_vllm_config(VllmConfig(device_config=DeviceConfig(device="cuda"))):
        init_distributed_environment(world_size=1, rank=0, distributed_init_method=f"tcp://127.0.0.1:{port}",
                                     local_rank=0, backend="gloo")
        initialize_model_parallel(1, 1)
        pre = "language_model.model.layers"  # vLLM's module tree of Qwen3.5

        def weights(n, k):
            return (torch.randint(0, 111, (n, k), dtype=torch.uint8, generator=g, device="cpu"),
                    (torch.rand(n, 1, generator=g, device="cpu") * 1e-3 + 1e-4))

        # q/k/v fused, static, one input scale stored under q_proj only
        qkv = QKVParallelLinear(HIDDEN, HEAD, HEADS, KV_HEADS, bias=False, params_dtype=torch.bfloat16,
                                quant_config=cfg, prefix=f"{pre}.0.self_attn.qkv_proj")
        assert isinstance(qkv.quant_method, va.Hif8StaticLinearMethod)
        parts = {}
        for sid, n in (("q", HEADS * HEAD), ("k", KV_HEADS * HEAD), ("v", KV_HEADS * HEAD)):
            w, ws = weights(n, HIDDEN)
            parts[sid] = (w, ws)
            qkv.weight.weight_loader(qkv.weight, w, sid)
            qkv.weight_scale.weight_loader(qkv.weight_scale, ws, sid)
        qkv.input_scale.weight_loader(qkv.input_scale, torch.tensor([0.0625]), "q")
        qkv.quant_method.process_weights_after_loading(qkv)
        want_w = torch.cat([parts[s][0] for s in "qkv"])
        want_s = torch.cat([parts[s][1] for s in "qkv"]).reshape(-1)
        assert qkv.weight.dtype == torch.uint8 and torch.equal(qkv.weight.cpu(), want_w)
        assert torch.equal(qkv.weight_scale.cpu(), want_s) and qkv.weight_scale.shape == (want_w.shape[0],)
        assert qkv.input_scale.shape == (1,) and float(qkv.input_scale) == 0.0625

        # gate/up fused: equal component scales accepted, different ones refused
        def gate_up(scales):
            lin = MergedColumnParallelLinear(HIDDEN, [INTER, INTER], bias=False, params_dtype=torch.bfloat16,
                                             quant_config=cfg, prefix=f"{pre}.0.mlp.gate_up_proj")
            for sid in (0, 1):
                w, ws = weights(INTER, HIDDEN)
                lin.weight.weight_loader(lin.weight, w, sid)
                lin.weight_scale.weight_loader(lin.weight_scale, ws, sid)
                lin.input_scale.weight_loader(lin.input_scale, torch.tensor([scales[sid]]), sid)
            lin.quant_method.process_weights_after_loading(lin)
            return lin

        gu = gate_up((0.25, 0.25))
        assert float(gu.input_scale) == 0.25 and gu.weight.shape == (2 * INTER, HIDDEN)
        _expect_raises(ValueError, lambda: gate_up((0.25, 0.5)), "different input scales")

        # row-parallel o_proj: input scale loaded as is; a missing one is refused
        def o_proj(scale):
            lin = RowParallelLinear(HEADS * HEAD, HIDDEN, bias=False, params_dtype=torch.bfloat16, quant_config=cfg,
                                    prefix=f"{pre}.0.self_attn.o_proj")
            w, ws = weights(HIDDEN, HEADS * HEAD)
            lin.weight.weight_loader(lin.weight, w)
            lin.weight_scale.weight_loader(lin.weight_scale, ws)
            if scale is not None:
                lin.input_scale.weight_loader(lin.input_scale, torch.tensor([scale]))
            lin.quant_method.process_weights_after_loading(lin)
            return lin

        o = o_proj(0.125)
        assert float(o.input_scale) == 0.125
        _expect_raises(ValueError, lambda: o_proj(None), "missing input_scale")

        # dynamic (W8A8HIF8_SOFT) fused gated-delta-net input; FLOAT b/a stays unquantized
        qkvz = MergedColumnParallelLinear(HIDDEN, [3 * HIDDEN, HIDDEN], bias=False, params_dtype=torch.bfloat16,
                                          quant_config=cfg, prefix=f"{pre}.1.linear_attn.in_proj_qkvz")
        assert isinstance(qkvz.quant_method, va.Hif8SoftLinearMethod) and not hasattr(qkvz, "input_scale")
        for sid, n in ((0, 3 * HIDDEN), (1, HIDDEN)):
            w, ws = weights(n, HIDDEN)
            qkvz.weight.weight_loader(qkvz.weight, w, sid)
            qkvz.weight_scale.weight_loader(qkvz.weight_scale, ws, sid)
        qkvz.quant_method.process_weights_after_loading(qkvz)
        ba = MergedColumnParallelLinear(HIDDEN, [8, 8], bias=False, params_dtype=torch.bfloat16, quant_config=cfg,
                                        prefix=f"{pre}.1.linear_attn.in_proj_ba")
        assert isinstance(ba.quant_method, UnquantizedLinearMethod)
        _expect_raises(ValueError, lambda: QKVParallelLinear(HIDDEN, HEAD, HEADS, KV_HEADS, bias=False,
                                                             params_dtype=torch.bfloat16, quant_config=cfg,
                                                             prefix=f"{pre}.2.self_attn.qkv_proj"),
                       "mixes HiF8 quant types")

        # HiF8 token embedding
        emb = VocabParallelEmbedding(VOCAB, HIDDEN, params_dtype=torch.bfloat16, quant_config=cfg,
                                     prefix="language_model.model.embed_tokens")
        assert isinstance(emb.quant_method, va.Hif8EmbeddingMethod)
        table, tscale = weights(VOCAB, HIDDEN)
        emb.weight_loader(emb.weight, table)
        emb.weight_loader(emb.weight_scale, tscale)
        emb.quant_method.process_weights_after_loading(emb)
        assert emb.weight.dtype == torch.uint8 and torch.equal(emb.weight[:VOCAB].cpu(), table)

        if gpu:
            _forward_checks(qkv, o, qkvz, emb, table, tscale, scheme)
    print(f"vllm adapter cases ({mode}): ok")


def _forward_checks(qkv, o, qkvz, emb, table, tscale, scheme):
    from oracle import oracle

    dev = qkv.weight.device
    g = torch.Generator().manual_seed(11)
    for rows in (1, 3, 40):
        x = (torch.randn(rows, HIDDEN, generator=g, device="cpu") * 2).to(torch.bfloat16).to(dev)
        ref = scheme.Hif8StaticLinear(qkv.weight.clone(), qkv.weight_scale.reshape(-1, 1).clone(),
                                      qkv.input_scale.clone())
        y, _ = qkv(x)
        assert torch.equal(y, ref(x)), f"qkv forward differs from scheme.apply at {rows} rows"
        xo = (torch.randn(rows, HEADS * HEAD, generator=g, device="cpu")).to(torch.bfloat16).to(dev)
        ref_o = scheme.Hif8StaticLinear(o.weight.clone(), o.weight_scale.reshape(-1, 1).clone(), o.input_scale.clone())
        yo, _ = o(xo)
        assert torch.equal(yo, ref_o(xo)), f"o_proj forward differs at {rows} rows"
        ref_d = scheme.Hif8SoftLinear(qkvz.weight.clone(), qkvz.weight_scale.reshape(-1, 1).clone())
        yd, _ = qkvz(x)
        assert torch.equal(yd, ref_d(x)), f"dynamic in_proj_qkvz forward differs at {rows} rows"
    ids = torch.tensor([0, 5, VOCAB - 1, 77, 5], device=dev)
    got = emb(ids)
    want = oracle.embedding(table.numpy(), tscale.numpy().reshape(-1), ids.cpu().numpy())
    assert got.dtype == torch.bfloat16
    np.testing.assert_array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16), want)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "cpu")
