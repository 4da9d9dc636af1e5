"""Two-GPU tensor-parallel decode of a reduced synthetic decoder: the decode
step with the row-parallel all-reduce fused into the following residual +
RMSNorm over peer memory (PeerReducer) matches the NCCL all-reduce step,
and its CUDA-graph replay reproduces the eager step.  Ranks run as two
processes (one per GPU) with a short process-group timeout; the peer waits
are bounded in the kernel.  Skipped where fewer than two GPUs are visible."""

from __future__ import annotations

import os
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg():
    from hif8_b200.decoder import DecoderConfig

    return DecoderConfig(hidden=512, intermediate=1024, layers=4, heads=4, kv_heads=2, head_dim=256,
                         lin_k_heads=2, lin_v_heads=4, vocab=1024)


def _rank(rank, world, port, out_dir):
    import faulthandler
    import json

    faulthandler.dump_traceback_later(240, exit=True)  # a stuck rank reports its stack and ends
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        from hif8_b200.decoder import Decoder, calibrate

        cfg = _cfg()
        calib = calibrate(cfg, dev, seed=5, tokens=48, tp_rank=rank, tp_size=world)
        model = Decoder(cfg, "hif8", dev, seed=5, tp_rank=rank, tp_size=world, max_batch=2, max_ctx=160,
                        calibration=calib)
        g = torch.Generator(device=dev).manual_seed(9)
        prompt = torch.randint(0, cfg.vocab, (2, 40), device=dev, generator=g)
        model.reset()
        first = model.prefill(prompt)
        state = [t.clone() for t in model.conv_state + model.rec_state if t is not None]
        pos = torch.full((2,), 40, dtype=torch.int32, device=dev)
        with torch.no_grad():
            ref = model.forward(first, pos, 2, 1, pos + 1, model._slots(2, pos))  # NCCL all-reduce
        for t, s in zip([t for t in model.conv_state + model.rec_state if t is not None], state):
            t.copy_(s)
        model.enable_peer_allreduce()
        with torch.no_grad():
            fused = model.forward(first, pos, 2, 1, pos + 1, model._slots(2, pos))
        model.peer.check()
        rel = float((fused - ref).abs().max()) / max(float(ref.abs().max()), 1e-12)
        # graph replay == eager with the fused reduce
        graph, tokens, gpos = model.decode_graph(2)
        for t, s in zip([t for t in model.conv_state + model.rec_state if t is not None], state):
            t.copy_(s)
        tokens.copy_(first)
        gpos.fill_(40)
        graph.replay()
        torch.cuda.synchronize()
        graph_tokens = tokens.clone()
        for t, s in zip([t for t in model.conv_state + model.rec_state if t is not None], state):
            t.copy_(s)
        e_tokens, e_pos = first.clone(), torch.full((2,), 40, dtype=torch.int32, device=dev)
        with torch.no_grad():
            model._decode_step(2, e_tokens, e_pos)
        model.peer.check()
        same = bool(torch.equal(graph_tokens, e_tokens))
        print(f"rank {rank}: fused vs NCCL max-rel {rel:.3e}, graph == eager {same}", flush=True)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as fh:
            json.dump([rel, same], fh)
        del graph, tokens, gpos  # a graph holding NCCL calls must be freed before the process group
        model.release_graphs()
        torch.cuda.synchronize()
        dist.barrier()
        model.peer.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(420)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_fused_allreduce_matches_nccl_and_graph_matches_eager(tmp_path):
    import json

    world = 2
    port = 29600 + os.getpid() % 1000
    # results come back through files: no manager process forked from this
    # (CUDA-initialised) process
    mp.spawn(_rank, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        rel, same = json.loads((tmp_path / f"rank{r}.json").read_text())
        assert rel <= 2e-2, f"rank {r}: fused vs NCCL logits max-rel {rel}"
        assert same, f"rank {r}: graph replay differs from the eager step"
