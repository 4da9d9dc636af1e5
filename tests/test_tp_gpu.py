"""Two-GPU tensor-parallel decode of a reduced synthetic decoder against the
single-GPU (TP-1) model with the same seeded weights and the same static
scales.

Every rank builds the TP-1 model too and computes its logits for a seeded
prompt and 6 teacher-forced decode steps; the TP-2 model must reproduce them
on its vocabulary slice within max-rel 2e-2 of the largest |logit| (the
only numerical difference is the summation of the row-parallel partials:
each rank's partial is rounded to BF16 before the sum), both with the NCCL
all-reduce and with the decode-step all-reduce fused into the following
residual + RMSNorm over peer memory.  The greedy tokens of every step must
agree, and the CUDA-graph replay of a decode step must reproduce the eager
step.  Ranks run as two processes (one per GPU) with a short process-group
timeout; the peer waits are bounded in the kernel.  Skipped where fewer than
two GPUs are visible."""

from __future__ import annotations

import os
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
STEPS = 6
MAX_REL = 2e-2


def _cfg():
    from hif8_b200.decoder import DecoderConfig

    return DecoderConfig(hidden=512, intermediate=1024, layers=4, heads=4, kv_heads=2, head_dim=256,
                         lin_k_heads=2, lin_v_heads=4, vocab=1024)


def _compare(logits, tokens, ref_logits, ref_tokens, rank, vocab_local):
    """(worst max-rel over the steps, steps whose greedy tokens all agree)."""
    worst, agree = 0.0, 0
    for lg, tk, rl, rt in zip(logits, tokens, ref_logits, ref_tokens):
        ref_slice = rl[:, rank * vocab_local:(rank + 1) * vocab_local]
        rel = float((lg - ref_slice).abs().max()) / max(float(rl.abs().max()), 1e-12)
        worst = max(worst, rel)
        agree += int(torch.equal(tk, rt))
    return worst, agree


def _rank(rank, world, port, out_dir):
    import faulthandler
    import json

    faulthandler.dump_traceback_later(300, exit=True)  # a stuck rank reports its stack and ends
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        from hif8_b200.decoder import Decoder, calibrate, forced_logits

        cfg = _cfg()
        calib = calibrate(cfg, dev, seed=5, tokens=48, tp_rank=rank, tp_size=world)
        g = torch.Generator(device=dev).manual_seed(9)
        prompt = torch.randint(0, cfg.vocab, (2, 40), device=dev, generator=g)

        # the TP-1 model of the same weights and scales, on this rank's GPU
        single = Decoder(cfg, "hif8", dev, seed=5, max_batch=2, max_ctx=160, calibration=calib)
        ref_logits, ref_tokens = forced_logits(single, prompt, steps=STEPS)
        ref_logits = [t.clone() for t in ref_logits]
        del single
        torch.cuda.empty_cache()

        model = Decoder(cfg, "hif8", dev, seed=5, tp_rank=rank, tp_size=world, max_batch=2, max_ctx=160,
                        calibration=calib)
        vl = model.vocab_local
        logits, tokens = forced_logits(model, prompt, ref_tokens, steps=STEPS)  # NCCL all-reduce
        nccl_rel, nccl_agree = _compare(logits, tokens, ref_logits, ref_tokens, rank, vl)
        model.enable_peer_allreduce()
        logits, tokens = forced_logits(model, prompt, ref_tokens, steps=STEPS)  # fused peer reduce
        peer_rel, peer_agree = _compare(logits, tokens, ref_logits, ref_tokens, rank, vl)

        # graph replay == eager with the fused reduce
        model.reset()
        first = model.prefill(prompt)
        state = [t.clone() for t in model.conv_state + model.rec_state if t is not None]
        graph, gtokens, gpos = model.decode_graph(2)
        for t, s in zip([t for t in model.conv_state + model.rec_state if t is not None], state):
            t.copy_(s)
        gtokens.copy_(first)
        gpos.fill_(40)
        graph.replay()
        torch.cuda.synchronize()
        graph_tokens = gtokens.clone()
        for t, s in zip([t for t in model.conv_state + model.rec_state if t is not None], state):
            t.copy_(s)
        e_tokens, e_pos = first.clone(), torch.full((2,), 40, dtype=torch.int32, device=dev)
        with torch.no_grad():
            model._decode_step(2, e_tokens, e_pos)
        model.peer.check()
        same = bool(torch.equal(graph_tokens, e_tokens))
        result = {"nccl_rel": nccl_rel, "nccl_agree": nccl_agree, "peer_rel": peer_rel, "peer_agree": peer_agree,
                  "graph_equals_eager": same, "steps": STEPS + 1}
        print(f"rank {rank}: {result}", flush=True)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as fh:
            json.dump(result, fh)
        del graph, gtokens, gpos  # a graph holding NCCL calls must be freed before the process group
        model.release_graphs()
        torch.cuda.synchronize()
        dist.barrier()
        model.peer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(480)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_decoder_matches_single_gpu_model(tmp_path):
    import json

    world = 2
    port = 29600 + os.getpid() % 1000
    # results come back through files: no manager process forked from this
    # (CUDA-initialised) process
    mp.spawn(_rank, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        res = json.loads((tmp_path / f"rank{r}.json").read_text())
        for path in ("nccl", "peer"):
            assert res[f"{path}_rel"] <= MAX_REL, f"rank {r}: TP-2 ({path}) vs TP-1 logits max-rel {res[f'{path}_rel']}"
            assert res[f"{path}_agree"] == res["steps"], f"rank {r}: TP-2 ({path}) greedy tokens differ from TP-1"
        assert res["graph_equals_eager"], f"rank {r}: graph replay differs from the eager step"
