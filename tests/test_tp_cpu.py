"""Tensor-parallel host logic of the synthetic decoder on CPU: every rank's
slices of the column-parallel (q/k/v/gate, gated-delta-net input, gate/up,
LM head) and row-parallel (o, out, down) projections reassemble into the
TP=1 tensors, KV heads are shared correctly when ranks outnumber them, and
the vocab-parallel greedy argmax agrees with the full argmax across two gloo
ranks."""

from __future__ import annotations

import json
import os
import types

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _cfg():
    from hif8_b200.decoder import DecoderConfig

    return DecoderConfig(hidden=128, intermediate=256, layers=4, heads=8, kv_heads=2, head_dim=256, rotary_dim=64,
                         lin_k_heads=4, lin_v_heads=8, vocab=64)


def _models(tp):
    from hif8_b200.decoder import Decoder

    return [Decoder(_cfg(), "bf16", "cpu", seed=3, tp_rank=r, tp_size=tp, max_batch=1, max_ctx=32)
            for r in range(tp)]


@pytest.mark.parametrize("tp", [2, 4])
def test_tp_slices_reassemble_the_full_weights(tp):
    cfg = _cfg()
    full = _models(1)[0]
    parts = _models(tp)
    D, d = cfg.head_dim, cfg.lin_dim
    for i, L in enumerate(full.layers):
        Ls = [m.layers[i] for m in parts]
        if L["full"]:
            q_rows = cfg.heads * 2 * D
            q_loc = q_rows // tp
            assert torch.equal(torch.cat([x["qkv"].weight[:q_loc] for x in Ls]), L["qkv"].weight[:q_rows])
            kv_loc = parts[0].kv_local * D
            k_full = L["qkv"].weight[q_rows:q_rows + cfg.kv_heads * D]
            k_parts = [x["qkv"].weight[q_loc:q_loc + kv_loc] for x in Ls]
            if tp <= cfg.kv_heads:
                assert torch.equal(torch.cat(k_parts), k_full)
            else:  # ranks 2j and 2j + 1 share KV head j
                for r, kp in enumerate(k_parts):
                    j = r // (tp // cfg.kv_heads)
                    assert torch.equal(kp, k_full[j * D:(j + 1) * D])
            assert torch.equal(torch.cat([x["o"].weight for x in Ls], dim=1), L["o"].weight)
        else:
            kd, vd = cfg.lin_k_heads * d, cfg.lin_v_heads * d
            sizes = [kd, kd, vd, vd, cfg.lin_v_heads, cfg.lin_v_heads]
            full_blocks = torch.split(L["lin_in"].weight, sizes)
            part_blocks = [torch.split(x["lin_in"].weight, [s // tp for s in sizes]) for x in Ls]
            for b, fb in enumerate(full_blocks):
                assert torch.equal(torch.cat([pb[b] for pb in part_blocks]), fb)
            assert torch.equal(torch.cat([x["lin_out"].weight for x in Ls], dim=1), L["lin_out"].weight)
            assert torch.equal(torch.cat([x["a_log"] for x in Ls]), L["a_log"])
        inter = cfg.intermediate // tp
        assert torch.equal(torch.cat([x["gate_up"].weight[:inter] for x in Ls]),
                           L["gate_up"].weight[:cfg.intermediate])
        assert torch.equal(torch.cat([x["gate_up"].weight[inter:] for x in Ls]),
                           L["gate_up"].weight[cfg.intermediate:])
        assert torch.equal(torch.cat([x["down"].weight for x in Ls], dim=1), L["down"].weight)
    assert torch.equal(torch.cat([m.lm_head for m in parts]), full.lm_head)


def test_kv_heads_shared_when_ranks_outnumber_them():
    from hif8_b200.decoder import Decoder, DecoderConfig

    cfg = DecoderConfig(hidden=128, intermediate=256, layers=4, heads=8, kv_heads=2, head_dim=256, rotary_dim=64,
                        lin_k_heads=8, lin_v_heads=16, vocab=64)
    parts = [Decoder(cfg, "bf16", "cpu", seed=3, tp_rank=r, tp_size=8, max_batch=1, max_ctx=32) for r in range(8)]
    assert [m.kv0 for m in parts] == [0, 0, 0, 0, 1, 1, 1, 1]
    assert all(m.kv_local == 1 and m.heads == 1 for m in parts)


def _argmax_rank(rank, world, port, logits_full, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hif8_b200.decoder import Decoder

        vocab_local = logits_full.shape[-1] // world
        me = types.SimpleNamespace(rank=rank, tp=world, group=None, vocab_local=vocab_local)
        local = logits_full[:, rank * vocab_local:(rank + 1) * vocab_local].contiguous()
        idx = Decoder.argmax(me, local)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as fh:
            json.dump(idx.tolist(), fh)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_vocab_parallel_argmax_over_gloo(tmp_path):
    world = 2
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(3, 64, generator=g)
    logits[1, 50] = 9.0  # the winner on rank 1
    logits[2, 3] = 9.0   # the winner on rank 0
    port = 29500 + os.getpid() % 1000
    mp.spawn(_argmax_rank, args=(world, port, logits, str(tmp_path)), nprocs=world, join=True)
    expected = logits.argmax(dim=-1).tolist()
    for r in range(world):
        assert json.loads((tmp_path / f"rank{r}.json").read_text()) == expected
