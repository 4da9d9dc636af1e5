"""Benchmark of the B200 HiF8 static W8A8 decode hot path.

One step = the decode projection sweep of configs[1]: for every token count
M in {1, 2, 4, 8, 16} and every projection shape (N, K) in
{(24576, 4096) gate/up, (4096, 12288) down, (6144, 4096) qkv}, one W8A8HIF8
static linear call ``y = linear(x)`` exactly as the quant scheme issues it
(static activation quant with the fixed input_scale + HiF8 linear; rows <= 4
take the fused quant+linear kernel).  Every call has its own weight, so a step
streams 15 distinct weights (880 MB, larger than the 126 MB L2) and no weight
is re-read from L2 between steps.

Metric: HiF8 GEMV HBM GB/s = algorithmic bytes / device time, algorithmic
bytes per call = N*K weight bytes + 4N channel scales + 2MK BF16 activation
+ 2MN BF16 output + 4 (input scale).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (torchrun, one rank per GPU, NCCL) the headline is the same
problem split tensor-parallel over the ranks (gate/up and qkv by output
channel, down by input channel + NCCL all-reduce): strong scaling, value =
the sweep's bytes / the slowest rank's time, so value_N / (N * value_1) is
the strong-scaling efficiency.  Before it is timed every call is checked
against the unsharded layer of the same quantised weight, and the
configs[4] decoder tensor-parallel over the N GPUs against its single-GPU
model (``tp_parity``); a failed check ends the run with exit code 3.
Beside it: ``replica_sweep`` (every rank runs the full sweep on its own
weights, no collective: weak scaling) and ``decode`` (the decoder's tok/s).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_ROOT = ROOT / "gcc-hif8-quantized-from-qwen3.5-9b_b200"
for _p in (str(ROOT), str(PKG_ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

M_VALUES = (1, 2, 4, 8, 16)
SHAPES = (("gate_up", 24576, 4096), ("down", 4096, 12288), ("qkv", 6144, 4096))
METRIC = "HiF8 GEMV HBM GB/s vs peak (M=1-16); W8A8KV8 decode tok/s at 1/2/4/8 B200"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0
TP_SWEEP_TOL = 1e-2    # north-star tolerance of a TP split (only the summation order changes)
# logits cosine vs TP-1 after 32 random-init layers: measured at TP 2, 0.9985-0.9989 for the BF16 twin
# (rounding-level differences amplified layer by layer) and 0.95-0.97 for HiF8 (a one-ulp difference can
# move a static code by a whole step); the bounds leave margin for other TP degrees
DECODER_TP_COS_BF16 = 0.99
DECODER_TP_COS_HIF8 = 0.85


def call_bytes(m: int, n: int, k: int) -> int:
    return n * k + 4 * n + 2 * m * k + 2 * m * n + 4


def step_bytes() -> int:
    return sum(call_bytes(m, n, k) for m in M_VALUES for _, n, k in SHAPES)


def workload_config(world: int, parallelism: str | None = None) -> dict:
    return {
        "workload": "configs[1] decode GEMV sweep: M in {1,2,4,8,16} x (N,K) in {(24576,4096) gate_up, "
                    "(4096,12288) down, (6144,4096) qkv}; one static-quant + HiF8 linear call each",
        "calls_per_step": len(M_VALUES) * len(SHAPES),
        "algorithmic_bytes_per_step": step_bytes(),
        "weights": "N(0,0.02) BF16 -> HiF8 u8, per-channel scale = row amax / 32768 (quantised over full rows, "
                   "then sharded); seeded",
        "activations": "N(0,1) BF16, fixed input_scale = calibration absmax / 32768",
        "l2": "inputs larger than L2: 15 distinct weights (880 MB) streamed per step",
        "parallelism": parallelism or ("single GPU" if world == 1 else f"tp{world}"),
        "graph": "one step captured as a CUDA graph, replayed per timed step",
    }


# ------------------------------------------------------------- utilities ---

def load_peak_hbm() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_profile_traffic() -> dict | None:
    path = ROOT / "profiles" / "gemv_traffic.json"
    try:
        return json.loads(path.read_text())
    except Exception:
        return None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.window = (0.0, 0.0)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)  # the sampler is producing lines before the timed region starts
        except Exception:
            self.proc = None
        return self

    def mark_start(self):
        self.window = (time.time(), self.window[1])

    def mark_end(self):
        self.window = (self.window[0], time.time())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        from datetime import datetime

        sm, smax, reasons = [], [], set()
        start, end = self.window
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                stamp = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                sm_mhz, max_mhz = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            if start and not (start - 0.02 <= stamp <= end + 0.02):
                continue
            sm.append(sm_mhz)
            smax.append(max_mhz)
            for name, flag in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                  parts[6:10]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------- CPU baseline ---

def time_cpu_baseline(budget_s: float = 20.0) -> dict:
    """Time the oracle port (the reference's CPU path restated: static quant
    in C, decode LUT + FP32 matmul in numpy/BLAS) on a bounded sample of the
    sweep: each projection shape at M = 1 and M = 16."""
    import numpy as np

    from oracle import oracle

    rng = np.random.default_rng(0)
    sample = [(m, name, n, k) for name, n, k in SHAPES for m in (1, 16)]
    done_bytes, spent = 0, 0.0
    runs = 0
    weights = {}
    for name, n, k in SHAPES:
        w = (rng.standard_normal((n, k), dtype=np.float32) * 0.02)
        weights[name] = oracle.quantize_rows_amax(w)
    start_all = time.perf_counter()
    while spent < budget_s and runs < 4:
        for m, name, n, k in sample:
            wq, ws = weights[name]
            x = oracle.f32_to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
            scale = np.array([4.5 / 32768.0], np.float32)
            t0 = time.perf_counter()
            a, a_s = oracle.static_quant(x, scale)
            y = oracle.linear_f32(a, wq, a_s, ws)
            oracle.f32_to_bf16_bits(y)
            spent += time.perf_counter() - t0
            done_bytes += call_bytes(m, n, k)
        runs += 1
        if time.perf_counter() - start_all > 3 * budget_s:
            break
    return {"value": done_bytes / spent / 1e9, "unit": UNIT, "cores": oracle.cpu_threads(), "kind": "port",
            "sample": f"{runs} pass(es) over M in {{1,16}} x the 3 projection shapes (static quant + decode + "
                      f"FP32 matmul, numpy BLAS threads); {spent:.1f} s"}


def run_reference(args) -> None:
    """--impl reference: the reference's CPU path (oracle port) on the host
    cores, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle

    rng = np.random.default_rng(0)
    # one step = the whole sweep on CPU is ~minutes; each step times a bounded
    # sample (every shape at M = 1 and 16) and reports GB/s over it
    weights = {name: oracle.quantize_rows_amax(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
               for name, n, k in SHAPES}
    xs = {(m, name): oracle.f32_to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
          for name, n, k in SHAPES for m in (1, 16)}
    scale = np.array([4.5 / 32768.0], np.float32)

    def one_step() -> tuple[float, int]:
        t0 = time.perf_counter()
        nbytes = 0
        for name, n, k in SHAPES:
            wq, ws = weights[name]
            for m in (1, 16):
                a, a_s = oracle.static_quant(xs[(m, name)], scale)
                oracle.f32_to_bf16_bits(oracle.linear_f32(a, wq, a_s, ws))
                nbytes += call_bytes(m, n, k)
        return time.perf_counter() - t0, nbytes

    for _ in range(args.warmup):
        one_step()
    total_t, total_b = 0.0, 0
    for _ in range(args.steps):
        t, b = one_step()
        total_t += t
        total_b += b
    value = total_b / total_t / 1e9
    cores = oracle.cpu_threads()
    sample = "per step: static quant + decode + FP32 matmul for every shape at M in {1,16} (oracle port)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total_t / max(args.steps, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(1) | {"reference_sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- our arm ---

def build_layers(world: int, rank: int, device, replica: int = 0, keep_reference: bool = False):
    """Seeded weights and activations for every call of the sweep; this rank's
    tensor-parallel shard when world > 1 (replica: a different seed set for an
    independent full copy).

    Every rank generates the same global weight of a call and quantises it
    ONCE over its full rows (bytes + per-row scale), as an exported
    checkpoint holds it; a column-parallel rank keeps its rows (and their
    scales), a row-parallel rank its input columns with the full rows'
    scales -- so the shards' results sum to the unsharded layer's result.
    ``keep_reference`` also keeps the unsharded layer and activation of every
    call (the TP-1 computation the parity check compares against)."""
    import torch

    from hif8_b200 import scheme

    calls = []
    for m in M_VALUES:
        for idx, (name, n, k) in enumerate(SHAPES):
            row_parallel = name == "down"
            seed = 1000 * m + idx + 104729 * replica
            g = torch.Generator(device=device).manual_seed(seed)
            n_loc = n if (world == 1 or row_parallel) else n // world
            k_loc = k // world if (world > 1 and row_parallel) else k
            w = torch.randn(n, k, device=device, generator=g, dtype=torch.float32).mul_(0.02).to(torch.bfloat16)
            calib = torch.randn(16, k, device=device, generator=g).to(torch.bfloat16)
            input_scale = (calib.float().abs().amax() / 32768.0).reshape(1).to(torch.float32)
            data, scale = scheme.quantize_weight_rows(w)
            del w
            x_full = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
            if world == 1:
                shard, shard_scale, x = data, scale, x_full
            elif row_parallel:  # clone: an owned tensor (the op wants storage offset 0)
                shard, shard_scale = data[:, rank * k_loc:(rank + 1) * k_loc].clone(), scale
                x = x_full[:, rank * k_loc:(rank + 1) * k_loc].clone()
            else:
                shard = data[rank * n_loc:(rank + 1) * n_loc].clone()
                shard_scale = scale[rank * n_loc:(rank + 1) * n_loc].clone()
                x = x_full
            layer = scheme.Hif8StaticLinear(shard, shard_scale.reshape(-1, 1), input_scale)
            call = {"m": m, "name": name, "n": n, "k": k, "layer": layer, "x": x, "row_parallel": row_parallel,
                    "n_loc": n_loc, "k_loc": k_loc}
            if keep_reference and world > 1:
                call["reference"] = (scheme.Hif8StaticLinear(data, scale.reshape(-1, 1), input_scale), x_full)
            calls.append(call)
            del data, scale
    torch.cuda.synchronize()
    return calls


def tp_apply(c, x, tp: bool):
    """One call of the sweep: scheme.apply, or -- for a row-parallel call
    under tensor parallelism -- this rank's FP32 partial product (summed over
    the ranks before its one BF16 rounding)."""
    import torch

    from hif8_b200 import scheme

    layer = c["layer"]
    if tp and c["row_parallel"]:
        return torch.ops.hif8_b200.linear_partial_f32(x, layer.weight, layer.input_scale, layer.weight_scale)
    return scheme.apply(layer, x)


class RowParallelReduce:
    """The all-reduce after a row-parallel call of the tensor-parallel sweep:
    the push exchange over NVLink peer memory (``PeerReducer.sum``: one
    launch, every rank sums the partials in rank order) or NCCL.  Call sites
    alternate between the reducer's two slots."""

    def __init__(self, device, rank: int, world: int, kind: str):
        self.kind = kind
        self.peer = None
        if kind == "peer":
            from hif8_b200.decoder import PeerReducer

            self.peer = PeerReducer(device, rank, world, max_rows=max(M_VALUES), dim=4096)
        self.site = 0

    def begin_step(self):
        self.site = 0

    def __call__(self, y):
        """All-reduce of an FP32 partial; the BF16 sum (one rounding)."""
        import torch
        import torch.distributed as dist

        if self.peer is None:
            dist.all_reduce(y)
            return y.to(torch.bfloat16)
        out = self.peer.sum(y, self.site % 2)
        self.site += 1
        return out

    def close(self):
        if self.peer is not None:
            import torch
            import torch.distributed as dist

            self.peer.check()
            torch.cuda.synchronize()
            dist.barrier()
            self.peer.close()
            self.peer = None


def tp_sweep_parity(calls, world: int, rank: int, device, reduce) -> dict:
    """Every call of the tensor-parallel sweep against the unsharded (TP-1)
    layer of the same quantised weight: column-parallel shards against their
    rows of the TP-1 output, row-parallel results (after the all-reduce)
    against the whole TP-1 output.  Errors are max |tp - ref| / max |ref|
    (global) and the same per output channel; the worst over calls and
    ranks is returned (every rank takes the same collective steps)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from hif8_b200 import scheme

    worst = torch.zeros(2, dtype=torch.float64, device=device)
    reduce.begin_step()
    for c in calls:
        ref_layer, x_full = c["reference"]
        ref = scheme.apply(ref_layer, x_full).float()
        y = tp_apply(c, c["x"], True)
        if c["row_parallel"]:
            y = reduce(y)
        else:
            ref = ref[:, rank * c["n_loc"]:(rank + 1) * c["n_loc"]]
        y = y.float()
        diff = (y - ref).abs()
        glob = float(diff.max()) / max(float(ref.abs().max()), 1e-12)
        floor = max(float(ref.abs().max()) * 1e-3, 1e-30)
        chan = float((diff.amax(dim=0) / ref.abs().amax(dim=0).clamp(min=floor)).max())
        worst = torch.maximum(worst, torch.tensor([glob, chan], dtype=torch.float64, device=device))
    dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    glob, chan = (float(v) for v in worst.tolist())
    ok = bool(np.isfinite(glob) and glob <= TP_SWEEP_TOL and chan <= TP_SWEEP_TOL)
    return {"max_rel": glob, "channel_max_rel": chan, "tol": TP_SWEEP_TOL, "pass": ok,
            "reduce": reduce.kind,
            "against": "the unsharded (TP-1) layer of the same quantised weight, every call of the sweep"}


def decoder_tp_parity(device, world: int, rank: int, calib: dict, steps: int = 8) -> dict:
    """The configs[4] decoder tensor-parallel over the ranks (peer-memory
    decode reduce, as measured) against the TP-1 model of the same seeded
    weights and static scales, which every rank also builds on its own GPU:
    logits of a seeded 64-token prompt's prefill and of ``steps``
    teacher-forced decode steps at batch 1 and 4, compared on this rank's
    vocabulary slice, for the HiF8 model and for its BF16 twin.

    The split itself changes only the order of FP32 sums (the row-parallel
    partials, and the column-parallel GEMMs that cuBLAS tiles differently for
    the twin).  That is a rounding-level difference per projection, but 32
    random-init layers amplify it: measured at TP 2, the BF16 twin -- no
    quantisation at all -- ends at logits cosine 0.9985 (max-rel 5 %) against
    its TP-1 model, and in the HiF8 model an output that moves by one BF16
    ulp can also move a static HiF8 code of the next projection's input by a
    whole code step (cosine 0.95-0.97).  The exact per-projection check is
    the sweep parity, and the 4-layer decoder is held to 2e-2 and identical
    tokens in tests/test_tp_gpu.py; here the pass criteria are cosine >=
    DECODER_TP_COS_BF16 (twin) and >= DECODER_TP_COS_HIF8 (HiF8) at every
    step, and every step's max-rel, cosine and greedy-token agreement is
    reported."""
    import torch
    import torch.distributed as dist

    from hif8_b200.decoder import Decoder, DecoderConfig, forced_logits

    cfg = DecoderConfig()
    g = torch.Generator(device=device).manual_seed(123)
    prompts = {b: torch.randint(0, cfg.vocab, (b, 64), device=device, generator=g) for b in (1, 4)}
    out = {"against": "the TP-1 model of the same seeded weights and static scales (prefill + "
                      f"{steps} teacher-forced decode steps, batch 1 and 4)"}
    ok = True
    for mode in ("bf16", "hif8"):
        single = Decoder(cfg, mode, device, seed=0, max_batch=4, max_ctx=128,
                         calibration=calib if mode == "hif8" else None)
        refs = {b: forced_logits(single, p, steps=steps) for b, p in prompts.items()}
        del single
        torch.cuda.empty_cache()
        model = Decoder(cfg, mode, device, seed=0, tp_rank=rank, tp_size=world, max_batch=4, max_ctx=128,
                        calibration=calib if mode == "hif8" else None)
        model.enable_peer_allreduce()
        vl = model.vocab_local
        # per step: max-rel (max over ranks), cosine (min over ranks), tokens equal (min over ranks)
        rel, cos, same = [], [], []
        for b, p in prompts.items():
            ref_logits, ref_tokens = refs[b]
            logits, tokens = forced_logits(model, p, ref_tokens, steps=steps)
            for lg, tk, rl, rt in zip(logits, tokens, ref_logits, ref_tokens):
                rs = rl[:, rank * vl:(rank + 1) * vl]
                rel.append(float((lg - rs).abs().max()) / max(float(rl.abs().max()), 1e-12))
                cos.append(float(torch.nn.functional.cosine_similarity(lg.flatten(), rs.flatten(), dim=0)))
                same.append(1.0 if torch.equal(tk, rt) else 0.0)
        model.peer.check()
        torch.cuda.synchronize()
        dist.barrier()
        model.peer.close()
        del model
        torch.cuda.empty_cache()
        t = torch.tensor([rel, [-c for c in cos], [-x for x in same]], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        rel, cos, same = t[0].tolist(), [-c for c in t[1].tolist()], [-x for x in t[2].tolist()]
        n = steps + 1  # per batch: prefill + decode steps
        res = {"logits_max_rel": [round(x, 5) for x in rel], "cosine": [round(x, 6) for x in cos],
               "greedy_equal": [int(x) for x in same], "steps_per_batch": n, "batches": [1, 4]}
        res["pass"] = min(cos) >= (DECODER_TP_COS_BF16 if mode == "bf16" else DECODER_TP_COS_HIF8)
        ok &= res["pass"]
        out["bf16_twin" if mode == "bf16" else "hif8_w8a8kv8"] = res
    out["pass"] = ok
    out["tol"] = {"bf16_twin_min_cosine": DECODER_TP_COS_BF16, "hif8_min_cosine": DECODER_TP_COS_HIF8}
    return out


def time_sweep(calls, args, device, world: int, local_rank: int, *, tp: bool, profile: bool, reduce=None):
    """One step = every call of ``calls`` (static quant + HiF8 linear through
    scheme.apply; row-parallel results all-reduced when ``tp``), captured as
    a CUDA graph; W warm-up replays, then K timed replays between barriers.
    Returns (max over ranks of the timed device ms, the clock sampler)."""
    import torch
    import torch.distributed as dist

    from hif8_b200 import scheme

    def step():
        outs = []
        if tp:
            reduce.begin_step()
        for c in calls:
            y = tp_apply(c, c["x"], tp)
            if tp and c["row_parallel"]:
                y = reduce(y)
            outs.append(y)
        return outs

    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        step()  # warm the private pool on the capture stream
        torch.cuda.synchronize(device)
        with torch.cuda.graph(graph, stream=stream):
            graph_outs = step()
    torch.cuda.current_stream(device).wait_stream(stream)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        # profiler start/stop bracket the timed steps for `ncu --profile-from-start off`
        if profile:
            torch.cuda.profiler.start()
        clocks.mark_start()
        start.record(cur)
        for _ in range(args.steps):
            graph.replay()
        end.record(cur)
        torch.cuda.synchronize()
        clocks.mark_end()
        if profile:
            torch.cuda.profiler.stop()
    if world > 1:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    del graph, graph_outs  # graphs holding NCCL calls go before the process group
    return elapsed_ms, clocks


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))
    from hif8_b200 import native

    native.load_extension()
    extra = {}
    parity_ok = True
    if world == 1:
        # The headline sweep on one GPU: the full configs[1] problem.
        calls = build_layers(1, 0, device)
        elapsed_ms, clocks = time_sweep(calls, args, device, world, local_rank, tp=False, profile=True)
        value = step_bytes() * args.steps / (elapsed_ms * 1e-3) / 1e9
        launches_per_step = sum(1 if c["m"] <= 4 else 2 for c in calls)
        parallelism = "single GPU"
    else:
        # N > 1: the headline is the SAME problem (the configs[1] sweep)
        # split tensor-parallel over the ranks (column: gate_up, qkv; row:
        # down + all-reduce) -- strong scaling, so value_N / (N * value_1) is
        # the strong-scaling efficiency.  Checked against the unsharded
        # layers before it is timed; a failed check ends the run non-zero.
        calls = build_layers(world, rank, device, keep_reference=True)
        reduce = RowParallelReduce(device, rank, world, args.tp_allreduce)
        extra["tp_parity"] = {"sweep": tp_sweep_parity(calls, world, rank, device, reduce)}
        parity_ok &= extra["tp_parity"]["sweep"]["pass"]
        for c in calls:
            c.pop("reference")
        torch.cuda.empty_cache()
        elapsed_ms, clocks = time_sweep(calls, args, device, world, local_rank, tp=True, profile=True, reduce=reduce)
        value = step_bytes() * args.steps / (elapsed_ms * 1e-3) / 1e9
        launches_per_step = sum(1 if c["m"] <= 4 else 2 for c in calls) + (
            sum(1 for c in calls if c["row_parallel"]) if reduce.kind == "peer" else 0)
        parallelism = (f"tp{world} (column: gate_up, qkv; row: down + all-reduce "
                       f"{'over NVLink peer memory (push exchange kernel)' if reduce.kind == 'peer' else 'NCCL'})")

    # -------------------------- dominant kernel: the GEMV, timed alone ---
    roofline = gemv_roofline(calls, args, device, world)

    # -------------------------------------------- e2e: public API, host I/O
    e2e = measure_e2e(calls, args, device, world, tp=world > 1, reduce=reduce if world > 1 else None)
    serial = measure_e2e(calls, args, device, world, tp=world > 1, reduce=reduce if world > 1 else None,
                         pipelined=False)
    e2e["serial"] = {"value": serial["value"], "ms_per_step": serial["ms_per_step"],
                     "how": "upload, compute and read-back in order on one stream"}
    if world > 1:
        reduce.close()

    if world > 1:
        # beside the headline: N independent full-size replicas (weak)
        calls.clear()
        torch.cuda.empty_cache()
        rep_calls = build_layers(1, 0, device, replica=rank)
        rep_ms, _ = time_sweep(rep_calls, args, device, world, local_rank, tp=False, profile=False)
        extra["replica_sweep"] = {"value": world * step_bytes() * args.steps / (rep_ms * 1e-3) / 1e9, "unit": UNIT,
                                  "scaling": "weak", "ms_per_step": rep_ms / args.steps,
                                  "what": "every rank runs the full configs[1] sweep on its own weights, "
                                          "no collective"}
        rep_calls.clear()
        torch.cuda.empty_cache()

    # ------------------- the other hot-path kernels (one GPU, timed alone) ---
    if world == 1 and not args.no_extra:
        extra["prefill_gemm"] = measure_prefill_gemm(device)
        extra["paged_attention"] = measure_paged_attention(device)
        extra["hbm_kernels"] = measure_hbm_kernels(device)
    if not args.no_decode:
        calls.clear()
        torch.cuda.empty_cache()
        extra["decode"] = measure_decoder(device, world, rank, check_parity=world > 1)
        if "tp_parity" in extra["decode"]:
            extra.setdefault("tp_parity", {})["decoder"] = extra["decode"].pop("tp_parity")
            parity_ok &= extra["tp_parity"]["decoder"]["pass"]

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        if not parity_ok:
            sys.exit(3)
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": workload_config(world, parallelism),
        "gpu_launches": launches_per_step * args.steps, "clocks": clocks.summary(), "roofline": roofline,
        "e2e": e2e, **extra,
    }
    if "decode" in extra:
        line["decode_tok_s"] = {b: extra["decode"]["hif8_w8a8kv8"][b]["tok_s"] for b in ("batch1", "batch4")}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = time_cpu_baseline(args.cpu_budget)
    print(json.dumps(line), flush=True)
    if not parity_ok:
        print("[bench] tensor-parallel parity check FAILED (tp_parity in the line)", file=sys.stderr)
        sys.exit(3)


def load_peak_bf16() -> tuple[float, str]:
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(peaks["bf16_tflops"]), "measured burst (MEASURED_PEAKS.json bf16_tflops, cuBLAS 8192^3)"
    except Exception:
        return 1590.0, "fallback 1590 TF/s"


def _timed_alone(fn, device, reps: int = 5) -> float:
    """Median device time (ms) of fn() over reps launches, each after a
    read-based L2 eviction, CUDA events on the current stream."""
    import torch

    flush = torch.ones(128 * 1024 * 1024, dtype=torch.float32, device=device)
    cur = torch.cuda.current_stream(device)
    times = []
    for _ in range(reps):
        flush.sum()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(cur)
        fn()
        e.record(cur)
        e.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)


def measure_prefill_gemm(device) -> dict:
    """M in {512, 4096} x the projection shapes, weights with 0.1%
    outliers at 20 sigma; soft_hif8_gemm (activation decode pre-pass + the
    tcgen05 GEMM) timed alone against the measured dense BF16 peak."""
    import torch

    from hif8_b200 import native, scheme

    ext = native.load_extension()
    g = torch.Generator(device=device).manual_seed(2)
    peak, kind = load_peak_bf16()
    per = []
    flops_total, ms_total = 0.0, 0.0
    for name, n, k in SHAPES:
        w = torch.randn(n, k, device=device, generator=g) * 0.02
        count = n * k // 1000
        idx = torch.randint(0, n * k, (count,), device=device, generator=g)
        sign = torch.randint(0, 2, (count,), device=device, generator=g).float() * 2 - 1
        w.view(-1)[idx] = sign * 20 * 0.02
        wq, ws = scheme.quantize_weight_rows(w.to(torch.bfloat16))
        del w
        lin = scheme.Hif8StaticLinear(wq, ws.reshape(-1, 1), torch.tensor([4.5 / 32768.0], device=device))
        for m in (512, 4096):
            x = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
            a, ts = native.static_quant(x, torch.tensor([4.5 / 32768.0], device=device))
            ext.soft_hif8_gemm(a, wq, ts, ws, None, torch.bfloat16)
            t = _timed_alone(lambda: ext.soft_hif8_gemm(a, wq, ts, ws, None, torch.bfloat16), device)
            # the projection as scheme.apply runs it from BF16 input: the static
            # quant fused into the GEMM's operand pass (beside: quant + GEMM)
            scheme.apply(lin, x)
            t_apply = _timed_alone(lambda: scheme.apply(lin, x), device)
            t_pair = _timed_alone(lambda: ext.soft_hif8_gemm(*native.static_quant(x, lin.input_scale)[:1], wq,
                                                             ts, ws, None, torch.bfloat16), device)
            flops = 2.0 * m * n * k
            per.append({"m": m, "shape": name, "us": round(t * 1e3, 1), "tflops": round(flops / (t * 1e-3) / 1e12, 1),
                        "frac": round(flops / (t * 1e-3) / 1e12 / peak, 3),
                        "apply_us": round(t_apply * 1e3, 1), "quant_then_gemm_us": round(t_pair * 1e3, 1)})
            flops_total += flops
            ms_total += t
    achieved = flops_total / (ms_total * 1e-3) / 1e12
    return {"bound": "tensor", "kernel": "gemm_hif8_tc_kernel (tcgen05, TMEM A operand) + decode_to_bf16",
            "achieved": round(achieved, 1), "peak": peak, "unit": "TF/s", "frac": round(achieved / peak, 3),
            "peak_kind": kind, "algorithmic": "2*M*N*K FLOPs per call", "per_call": per,
            "apply": "apply_us: scheme.apply from BF16 input (static quant fused into the GEMM's BF16 operand pass); "
                     "quant_then_gemm_us: hif8_static_quant then soft_hif8_gemm",
            "timing": "median of 5 calls per config, each after a read-based L2 eviction, CUDA events"}


def measure_paged_attention(device) -> dict:
    """decode step of batch 4 at contexts 512 and 4096, 16 query /
    4 KV heads, head_dim 256, 128-token HiF8 pages (shuffled block table);
    the attention kernels timed alone against the measured HBM peak."""
    import math

    import torch

    from hif8_b200 import kv_cache

    kv_cache.load_ops()
    peak, kind = load_peak_hbm()
    g = torch.Generator(device=device).manual_seed(3)
    batch, heads, kv_heads, d, block = 4, 16, 4, 256, 128
    per = []
    for ctx in (512, 4096):
        blocks_per = ctx // block
        total = batch * blocks_per
        table = torch.randperm(total, device=device, generator=g).view(batch, blocks_per).to(torch.int32)
        kc = torch.randint(0, 256, (total, block, kv_heads, d + 4), dtype=torch.uint8, device=device, generator=g)
        vc = torch.randint(0, 256, (total, block, kv_heads, d + 4), dtype=torch.uint8, device=device, generator=g)
        scale_bytes = torch.tensor([0.01] * (total * block * kv_heads), dtype=torch.float32,
                                   device=device).view(torch.uint8).view(total, block, kv_heads, 4)
        kc[..., d:] = scale_bytes
        vc[..., d:] = scale_bytes
        kc[..., :d] &= 0x7F  # finite magnitudes only (no NaN code)
        vc[..., :d] &= 0x7F
        kc[..., :d] = torch.where(kc[..., :d] == 0x6F, torch.zeros_like(kc[..., :d]), kc[..., :d])
        vc[..., :d] = torch.where(vc[..., :d] == 0x6F, torch.zeros_like(vc[..., :d]), vc[..., :d])
        q = torch.randn(batch, heads, d, device=device, generator=g).to(torch.bfloat16)
        lens = torch.full((batch,), ctx, dtype=torch.int32, device=device)
        starts = torch.arange(batch + 1, dtype=torch.int32, device=device)
        fn = lambda: torch.ops.hif8_b200.paged_attention(q, kc, vc, table, lens, starts, ctx, 1.0 / math.sqrt(d), True)
        fn()
        t = _timed_alone(fn, device)
        nbytes = 2 * batch * ctx * kv_heads * (d + 4) + 2 * 2 * batch * heads * d
        per.append({"ctx": ctx, "batch": batch, "us": round(t * 1e3, 2), "gbs": round(nbytes / (t * 1e-3) / 1e9, 1),
                    "frac": round(nbytes / (t * 1e-3) / 1e9 / peak, 3)})
    return {"bound": "hbm", "kernel": "paged_attention_kernel + attention_combine_kernel", "unit": "GB/s",
            "peak": peak, "peak_kind": kind, "algorithmic": "K and V pages read once (B*ctx*kv_heads*(D+4)*2) + Q + out",
            "per_config": per, "timing": "median of 5 decode steps, each after a read-based L2 eviction, CUDA events"}


HBM_KERNEL_CASES = {
    # name: (kernel, the size where HBM is the bound, the decode-size case)
    "quant": ("static_quant_vec16", "x [4096, 12288] BF16 (configs[2] prefill, down input), scale = calibration "
                                    "absmax / 32768",
              "x [16, 12288] BF16"),
    "kv_write": ("kv_write_warp_kernel", "16384 tokens x 4 KV heads x 256, K and V, BF16 source, per-head scale = "
                                         "calibration absmax / 32768, random slots",
                 "4 tokens (a batch-4 decode step)"),
    "embedding": ("embedding_gather", "16384 ids of a [248320, 4096] HiF8 table",
                  "4 ids (a batch-4 decode step)"),
    "scaled_decode": ("scaled_decode_vec", "data [65536, 256] u8 (configs[3]: batch 4 x ctx 4096 x 4 KV heads)",
                      "data [16, 256] u8"),
}


def _hbm_kernel_inputs(name: str, big: bool, device):
    """(callable, algorithmic bytes) of one hbm_kernels case."""
    import torch

    from hif8_b200 import checkpoint, kv_cache, native

    g = torch.Generator(device=device).manual_seed(4)
    if name == "quant":
        m, k = (4096, 12288) if big else (16, 12288)
        x = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
        # the configs' rule: global absmax of a seeded calibration batch / 32768
        calib = torch.randn(64, k, device=device, generator=g).to(torch.bfloat16)
        scale = (calib.float().abs().amax() / 32768.0).reshape(1)
        # BF16 in, u8 out, FP32 row scale out, the fixed scale in
        return (lambda: native.static_quant(x, scale)), 3 * m * k + 4 * m + 4
    if name == "kv_write":
        tokens, heads, d, block = (16384 if big else 4), 4, 256, 128
        layout = kv_cache.Hif8KVCacheLayout(max(tokens // block, 1) * 2, block, heads, d)
        kc, vc = layout.allocate(device)
        key = torch.randn(tokens, heads, d, device=device, generator=g).to(torch.bfloat16)
        val = torch.randn(tokens, heads, d, device=device, generator=g).to(torch.bfloat16)
        # per-head static scales by the configs' rule: calibration absmax / 32768
        ks = (key[:64].float().abs().amax(dim=(0, 2)) / 32768.0).contiguous()
        vs = (val[:64].float().abs().amax(dim=(0, 2)) / 32768.0).contiguous()
        slots = torch.randperm(layout.num_blocks * block, device=device, generator=g)[:tokens].contiguous()
        fn = lambda: torch.ops.hif8_b200.kv_cache_write(key, val, ks, vs, slots, kc, vc, None)
        # per token and plane: heads x (2 D source bytes + D + 4 page bytes); + the 8-byte slot
        return fn, tokens * (2 * heads * (2 * d + d + 4) + 8)
    if name == "embedding":
        vocab, hidden = 248320, 4096
        ids_n = 16384 if big else 4
        data = torch.randint(0, 0x6F, (vocab, hidden), dtype=torch.uint8, device=device, generator=g)
        scale = torch.rand(vocab, device=device, generator=g) * 1e-4 + 1e-5
        emb = checkpoint.Hif8Embedding(data, scale)
        ids = torch.randint(0, vocab, (ids_n,), device=device, generator=g)
        # per id: the HiF8 row, its FP32 scale, the BF16 output row, the 8-byte id
        return (lambda: emb(ids)), ids_n * (hidden + 4 + 2 * hidden + 8)
    if name == "scaled_decode":
        rows, d = (65536, 256) if big else (16, 256)
        data = torch.randint(0, 0x6F, (rows, d), dtype=torch.uint8, device=device, generator=g)
        scale = torch.rand(rows, device=device, generator=g) + 0.25
        # u8 in, FP32 row scale in, BF16 out
        return (lambda: native.scaled_decode(data, scale)), rows * d * 3 + 4 * rows
    raise ValueError(name)


def measure_hbm_kernels(device) -> dict:
    """Roofline of the other HBM-bound kernels of the path (static quant, KV
    page write, HiF8 embedding gather): each timed alone at a size where HBM
    is the bound (median of 5 launches, each after a read-based L2
    eviction, CUDA events) against the measured HBM peak, with its
    decode-size latency beside it."""
    import torch

    peak, kind = load_peak_hbm()
    out = {"peak": peak, "unit": "GB/s", "peak_kind": kind,
           "timing": "median of 5 launches, each after a read-based L2 eviction, CUDA events"}
    for name, (kernel, big_desc, small_desc) in HBM_KERNEL_CASES.items():
        fn, nbytes = _hbm_kernel_inputs(name, True, device)
        fn()
        t = _timed_alone(fn, device)
        achieved = nbytes / (t * 1e-3) / 1e9
        sfn, sbytes = _hbm_kernel_inputs(name, False, device)
        sfn()
        ts = _timed_alone(sfn, device)
        out[name] = {"kernel": kernel, "bound": "hbm", "size": big_desc, "bytes": nbytes, "us": round(t * 1e3, 2),
                     "achieved": round(achieved, 1), "frac": round(achieved / peak, 3),
                     "decode_size": small_desc, "decode_us": round(ts * 1e3, 2)}
        del fn, sfn
        torch.cuda.empty_cache()
    return out


def measure_decoder(device, world: int, rank: int, check_parity: bool = False) -> dict:
    """the random-init Qwen3.5-9B-shaped hybrid decoder, 512
    prompt / 256 generated tokens at batch 1 and 4, tensor-parallel over the
    bench's GPUs; the W8A8KV8 HiF8 model and its BF16 twin.  Decode steps are
    CUDA-graph replays timed with CUDA events (max over ranks).  With
    ``check_parity`` the tensor-parallel HiF8 model is first compared with
    its single-GPU model (``tp_parity`` in the result)."""
    import torch
    import torch.distributed as dist

    from hif8_b200.decoder import Decoder, DecoderConfig, calibrate, measure_decode

    cfg = DecoderConfig()
    calib = calibrate(cfg, device, seed=0, tokens=64, tp_rank=rank, tp_size=world)
    out = {"model": "Qwen3.5-9B-shaped hybrid decoder (32 layers: 8 gated full-attention, 24 gated delta net; "
                    "hidden 4096, MLP 12288, vocab 248320), random init",
           "prompt": 512, "generated": 256, "tp": world, "timing": "CUDA-graph decode steps, CUDA events, max over ranks",
           "allreduce": "single GPU" if world == 1 else "row-parallel partials summed over peer memory inside the "
                                                       "following residual + RMSNorm kernel (prefill: NCCL)"}
    if check_parity:
        out["tp_parity"] = decoder_tp_parity(device, world, rank, calib)
    for mode in ("hif8", "bf16"):
        model = Decoder(cfg, mode, device, seed=0, tp_rank=rank, tp_size=world, max_batch=4, max_ctx=768,
                        calibration=calib if mode == "hif8" else None)
        if world > 1:
            model.enable_peer_allreduce()  # decode-step all-reduce fused into the following RMSNorm
        res = {}
        for batch in (1, 4):
            r = measure_decode(model, batch)
            ms = torch.tensor([r["ms_per_step"]], device=device, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            res[f"batch{batch}"] = {"tok_s": round(batch / (float(ms) * 1e-3), 1), "ms_per_step": round(float(ms), 3)}
        model.release_graphs()
        if model.peer is not None:
            model.peer.check()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            model.peer.close()
        del model
        torch.cuda.empty_cache()
        out["hif8_w8a8kv8" if mode == "hif8" else "bf16_twin"] = res
    out["speedup_vs_bf16"] = {b: round(out["hif8_w8a8kv8"][b]["tok_s"] / out["bf16_twin"][b]["tok_s"], 3)
                              for b in ("batch1", "batch4")}
    return out


def gemv_roofline(calls, args, device, world) -> dict:
    """Roofline of the dominant kernel (the GEMV), measured in the timed
    step's setting: the 15 GEMV launches of the sweep (M <= 4: the fused
    quant + GEMV kernel on BF16 input; M = 8, 16: the GEMV on the bytes and
    row scales of hif8_static_quant, computed once outside) are captured back
    to back as one CUDA graph and replayed K times between two CUDA events
    on the launching stream; achieved = algorithmic bytes of the 15 launches
    x K / the elapsed time, i.e. bytes per launch / average launch duration.
    The sweep's 15 distinct weights (880 MB) exceed L2, so every launch reads
    its weight from HBM.  Reported beside it: per-launch durations from
    timing events recorded around every launch inside a graph (event nodes
    serialise the launches, so these read slightly long) and the same
    launches timed alone after a read-based L2 eviction."""
    import torch

    from hif8_b200 import native

    ext = native.load_extension()
    cur = torch.cuda.current_stream(device)

    def algo_bytes(c):
        m, n_loc, k_loc = c["m"], c["n_loc"], c["k_loc"]
        # u8 weight + FP32 channel scale + u8 activation + FP32 row scale +
        # BF16 out; the fused M <= 4 kernel reads BF16 activations instead
        act = 2 * m * k_loc if m <= 4 else m * k_loc + 4 * m
        return n_loc * k_loc + 4 * n_loc + act + 2 * m * n_loc

    def capture(fn):
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream(device)
        stream.wait_stream(cur)
        with torch.cuda.stream(stream):
            fn()
            torch.cuda.synchronize(device)
            with torch.cuda.graph(graph, stream=stream):
                fn()
        cur.wait_stream(stream)
        return graph

    quant = [native.static_quant(c["x"], c["layer"].input_scale) if c["m"] > 4 else None for c in calls]

    def gemv(c, q):
        layer = c["layer"]
        if q is None:
            native.soft_static_fused_linear(c["x"], layer.weight, layer.input_scale, layer.weight_scale, None,
                                            output_dtype=torch.bfloat16)
        else:
            ext.soft_hif8_gemm(q[0], layer.weight, q[1], layer.weight_scale, None, torch.bfloat16)

    # ------------------------------------- the 15 launches back to back ---
    reps = max(args.steps, 5)
    graph = capture(lambda: [gemv(c, q) for c, q in zip(calls, quant)])
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(cur)
    for _ in range(reps):
        graph.replay()
    end.record(cur)
    torch.cuda.synchronize()
    stream_ms = start.elapsed_time(end) / reps
    del graph

    # ----------------------- per-launch events inside a graph (detail) ---
    evs = [(torch.cuda.Event(enable_timing=True, external=True),
            torch.cuda.Event(enable_timing=True, external=True)) for _ in calls]

    def step():
        for c, q, (s, e) in zip(calls, quant, evs):
            s.record()
            gemv(c, q)
            e.record()

    in_graph = None
    try:
        graph = capture(step)
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        sums = [0.0] * len(calls)
        for _ in range(reps):
            graph.replay()
            torch.cuda.synchronize()
            for i, (s, e) in enumerate(evs):
                sums[i] += s.elapsed_time(e)
        del graph
        in_graph = [t / reps for t in sums]
    except RuntimeError as exc:  # event-record nodes unsupported: no per-launch detail
        print(f"[bench] in-graph GEMV events unavailable ({exc})", file=sys.stderr)
        torch.cuda.synchronize()

    # --------------------------------------------- isolated, L2 evicted ---
    # L2 is evicted by READING a 512 MB buffer: writing one would leave dirty
    # lines whose write-back competes with the timed launch.
    flush = torch.ones(128 * 1024 * 1024, dtype=torch.float32, device=device)
    iso = []
    for c, q in zip(calls, quant):
        times = []
        for _ in range(5):
            flush.sum()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(cur)
            gemv(c, q)
            e.record(cur)
            e.synchronize()
            times.append(s.elapsed_time(e))
        iso.append(statistics.median(times))
    del flush

    # compact rows (one short list per launch) so the whole JSON line stays short
    per = []
    total_b = sum(algo_bytes(c) for c in calls)
    for i, c in enumerate(calls):
        b = algo_bytes(c)
        per.append([c["m"], c["name"], b, round(iso[i] * 1e3, 2),
                    round(in_graph[i] * 1e3, 2) if in_graph is not None else None])
    peak, kind = load_peak_hbm()
    achieved = total_b / (stream_ms * 1e-3) / 1e9
    iso_achieved = total_b / (sum(iso) * 1e-3) / 1e9
    prof = load_profile_traffic()
    traffic = None
    if prof and prof.get("world") == world:
        traffic = prof.get("traffic_bytes_per_launch")
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic, "algorithmic_bytes_mean_per_launch": total_b / len(calls),
            "launch_us_mean": stream_ms * 1e3 / len(calls),
            "peak_kind": f"{kind} (MEASURED_PEAKS.json hbm_gbs, copy)" if kind == "measured" else "fallback 6650 GB/s",
            "kernel": "gemv_hif8_kernel (persistent split-K, LUT decode, mma.sync)",
            "algorithmic_bytes_per_launch": "N*K + 4N + 2N*M + (M <= 4: 2MK BF16 activation; else MK + 4M u8 "
                                            "activation + row scale)",
            "timing": f"the 15 GEMV launches of the sweep as one CUDA graph, {reps} replays between CUDA events "
                      "on the launching stream",
            "event_timing": "per_launch event_us: events recorded around each launch inside a graph (serialising)",
            "isolated": {"achieved": iso_achieved, "frac": iso_achieved / peak,
                         "timing": "median of 5 launches per config, each after a read-based L2 eviction"},
            "per_launch_fields": ["m", "shape", "algorithmic bytes", "isolated_us", "event_us"],
            "per_launch": per}


def measure_e2e(calls, args, device, world, tp: bool = False, reduce=None, pipelined: bool = True) -> dict:
    """The same sweep through the public API (hif8_b200.scheme, eager) with
    host buffers inside the timed region: every step copies its 15
    activations from one packed pinned host buffer to the device (one H2D
    transfer), runs the 15 ``scheme.apply`` calls, gathers the 15 outputs
    into one device buffer and reads it back into pinned host memory (one D2H
    transfer).  ``pipelined`` (the headline): the copies run on a copy stream
    and overlap the neighbouring steps' compute, as a serving loop overlaps
    its transfers -- step i's upload is issued once step i-2 has finished
    with its input buffer (two buffers), and its read-back as soon as its
    outputs are gathered; the timed region opens before the first upload and
    closes after the last read-back.  Without it, every step uploads, computes
    and reads back in order on one stream.  With ``tp`` the calls are this
    rank's tensor-parallel shards (row-parallel results all-reduced inside
    the step) and value is the sweep's bytes over the slowest rank's time;
    without it, one independent replica per rank (value aggregates the
    ranks)."""
    import torch
    import torch.distributed as dist

    sizes = [c["x"].numel() for c in calls]
    offs = [sum(sizes[:i]) for i in range(len(sizes))]
    host_in = torch.cat([c["x"].reshape(-1).cpu() for c in calls]).pin_memory()
    out_sizes = [c["m"] * (c["n_loc"] if not c["row_parallel"] else c["n"]) for c in calls]
    slots = 2 if pipelined else 1
    dev_in = [torch.empty(host_in.numel(), dtype=host_in.dtype, device=device) for _ in range(slots)]
    dev_x = [[buf[o:o + n].view(c["x"].shape) for o, n, c in zip(offs, sizes, calls)] for buf in dev_in]
    dev_out = [torch.empty(sum(out_sizes), dtype=torch.bfloat16, device=device) for _ in range(slots)]
    host_out = [torch.empty(sum(out_sizes), dtype=torch.bfloat16).pin_memory() for _ in range(slots)]
    cur = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device) if pipelined else cur
    uploaded = [torch.cuda.Event() for _ in range(slots)]
    computed = [torch.cuda.Event() for _ in range(slots)]

    def compute(slot):
        outs = []
        if tp:
            reduce.begin_step()
        for c, x in zip(calls, dev_x[slot]):
            y = tp_apply(c, x, tp)
            if tp and c["row_parallel"]:
                y = reduce(y)
            outs.append(y.reshape(-1))
        torch.cat(outs, out=dev_out[slot])

    def run(steps, start=None):
        if not pipelined:
            for _ in range(steps):
                dev_in[0].copy_(host_in, non_blocking=True)
                compute(0)
                host_out[0].copy_(dev_out[0], non_blocking=True)
            return
        if start is not None:
            copy.wait_event(start)
        else:
            copy.wait_stream(cur)
        with torch.cuda.stream(copy):
            for i in range(min(2, steps)):
                dev_in[i].copy_(host_in, non_blocking=True)
                uploaded[i].record(copy)
        for i in range(steps):
            slot = i % 2
            cur.wait_event(uploaded[slot])
            compute(slot)
            computed[slot].record(cur)
            copy.wait_event(computed[slot])
            with torch.cuda.stream(copy):
                host_out[slot].copy_(dev_out[slot], non_blocking=True)
                if i + 2 < steps:
                    dev_in[slot].copy_(host_in, non_blocking=True)
                    uploaded[slot].record(copy)
        cur.wait_stream(copy)

    run(max(args.warmup, 1))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(cur)
    run(args.steps, start)
    end.record(cur)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    last = (args.steps - 1) % slots
    if not torch.equal(host_out[last], dev_out[last].cpu()):
        raise RuntimeError("e2e: the read-back differs from the step's device outputs")
    for hy, c in zip(host_out[last].split(out_sizes), calls):  # the read-back values are the step's results
        if not torch.isfinite(hy.float()).all():
            raise RuntimeError(f"e2e: non-finite output for {c['name']} M={c['m']}")
    h2d = host_in.numel() * 2
    d2h = host_out[0].numel() * 2
    problems = 1 if tp else world  # TP: one problem split over the ranks; else one per rank
    how = ("copies on a copy stream overlapping the neighbouring steps' compute (two input buffers)" if pipelined
           else "upload, compute and read-back in order on one stream")
    return {"value": problems * step_bytes() * args.steps / (ms * 1e-3) / 1e9, "unit": UNIT,
            "h2d_bytes_per_step": world * h2d, "d2h_bytes_per_step": world * d2h, "ms_per_step": ms / args.steps,
            "transfers_per_step": {"h2d": 1, "d2h": 1},
            "path": "hif8_b200.scheme.apply (one hif8_b200::static_linear operator per call -> C ABI), pinned host "
                    "buffers, outputs gathered on the device and read back in one transfer; " + how +
                    (f"; tensor-parallel shards + {reduce.kind} all-reduce" if tp else "")}


def run_profile_case(spec: str, launches: int) -> None:
    """Small cases for ncu captures, nothing else of the bench:
    ``decode:<batch>`` runs one eager decode step of the configs[4] model;
    ``gemv:<shape>:<m>`` / ``gemm:<shape>:<m>`` run the linear kernel of one
    call ``launches`` times (two warm-up launches first); ``gemv:sweep`` runs
    each of the 15 configs[1] calls once after a read-based L2 eviction, M <= 4
    through the fused quant + GEMV kernel as in the timed step."""
    import torch

    from hif8_b200 import native, scheme

    parts = spec.split(":")
    if parts[0] == "decode-tp" and len(parts) == 2:
        # one CUDA-graph decode step of the configs[4] model tensor-parallel
        # over the torchrun ranks, kernels recorded by torch.profiler (CUPTI)
        # on rank 0; prints the kernel time per name (device time, the step
        # replayed as in the bench)
        import torch.distributed as dist
        from datetime import timedelta

        from hif8_b200.decoder import Decoder, DecoderConfig, calibrate

        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        if world > 1:
            dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        batch = int(parts[1])
        cfg = DecoderConfig()
        calib = calibrate(cfg, dev, seed=0, tokens=64, tp_rank=rank, tp_size=world)
        model = Decoder(cfg, "hif8", dev, seed=0, tp_rank=rank, tp_size=world, max_batch=batch, max_ctx=768,
                        calibration=calib)
        if world > 1:
            model.enable_peer_allreduce()
        g = torch.Generator(device=dev).manual_seed(1)
        prompt = torch.randint(0, cfg.vocab, (batch, 512), device=dev, generator=g)
        graph, tokens, pos = model.decode_graph(batch)
        with torch.no_grad():
            tokens.copy_(model.prefill(prompt))
        pos.fill_(512)
        for _ in range(5):
            graph.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            graph.replay()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        if rank == 0:
            rows = {}
            for ev in prof.events():
                if ev.device_type == torch.autograd.DeviceType.CUDA and ev.device_time > 0:
                    r = rows.setdefault(ev.name[:60], [0, 0.0])
                    r[0] += 1
                    r[1] += ev.device_time
            total = sum(v[1] for v in rows.values())
            print(f"decode step, batch {batch}, tp {world}: {sum(v[0] for v in rows.values())} launches, "
                  f"{total:.1f} us of kernel time (rank 0, torch.profiler)")
            for name, (n, t) in sorted(rows.items(), key=lambda kv: -kv[1][1]):
                print(f"{name:60s} {n:6d} {t:10.1f} {100 * t / total:6.1f}%")
        del graph  # a graph holding NCCL calls goes before the process group
        model.release_graphs()
        if model.peer is not None:
            model.peer.check()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            model.peer.close()
        if world > 1:
            dist.destroy_process_group()
        return
    if parts[0] == "decode" and len(parts) == 2:
        # one eager decode step of the configs[4] model at batch B between
        # cudaProfilerStart/Stop (for `ncu --profile-from-start off`)
        from hif8_b200.decoder import Decoder, DecoderConfig, calibrate

        dev = torch.device("cuda", 0)
        batch = int(parts[1])
        cfg = DecoderConfig()
        calib = calibrate(cfg, dev, seed=0, tokens=64)
        model = Decoder(cfg, "hif8", dev, seed=0, max_batch=batch, max_ctx=768, calibration=calib)
        g = torch.Generator(device=dev).manual_seed(1)
        first = model.prefill(torch.randint(0, cfg.vocab, (batch, 512), device=dev, generator=g))
        pos = torch.full((batch,), 512, dtype=torch.int32, device=dev)
        with torch.no_grad():
            for _ in range(2):
                model._decode_step(batch, first.clone(), pos.clone())
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            model._decode_step(batch, first.clone(), pos.clone())
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
        print(f"profile case {spec}: one decode step ok")
        return
    if parts[0] == "attn" and len(parts) == 2:
        import math

        dev = torch.device("cuda", 0)
        native.load_extension()
        from hif8_b200 import kv_cache

        kv_cache.load_ops()
        g = torch.Generator(device=dev).manual_seed(3)
        ctx = int(parts[1])
        batch, heads, kv_heads, d, block = 4, 16, 4, 256, 128
        total = batch * ((ctx + block - 1) // block)
        table = torch.randperm(total, device=dev, generator=g).view(batch, -1).to(torch.int32)
        kc = torch.randint(0, 0x60, (total, block, kv_heads, d + 4), dtype=torch.uint8, device=dev, generator=g)
        vc = torch.randint(0, 0x60, (total, block, kv_heads, d + 4), dtype=torch.uint8, device=dev, generator=g)
        sb = torch.full((total, block, kv_heads), 0.01, device=dev).view(torch.uint8).view(total, block, kv_heads, 4)
        kc[..., d:] = sb
        vc[..., d:] = sb
        q = torch.randn(batch, heads, d, device=dev, generator=g).to(torch.bfloat16)
        lens = torch.full((batch,), ctx, dtype=torch.int32, device=dev)
        starts = torch.arange(batch + 1, dtype=torch.int32, device=dev)
        for _ in range(2 + launches):
            torch.ops.hif8_b200.paged_attention(q, kc, vc, table, lens, starts, ctx, 1.0 / math.sqrt(d), True)
        torch.cuda.synchronize()
        print(f"profile case {spec}: {2 + launches} launches ok")
        return
    if parts[0] == "hbm" and len(parts) in (2, 3):
        # hbm:<quant|kv_write|embedding>[:small]: two warm-up launches, then
        # `launches` launches of that kernel at the bench's HBM-bound size
        dev = torch.device("cuda", 0)
        native.load_extension()
        fn, _ = _hbm_kernel_inputs(parts[1], len(parts) == 2, dev)
        for _ in range(2 + launches):
            fn()
        torch.cuda.synchronize()
        print(f"profile case {spec}: {2 + launches} launches ok")
        return
    if parts[0] not in ("gemv", "gemm") or len(parts) not in (2, 3):
        raise SystemExit(f"unknown profile case {spec!r}")
    dev = torch.device("cuda", 0)
    ext = native.load_extension()
    g = torch.Generator(device=dev).manual_seed(0)
    fixed = torch.tensor([4.5 / 32768.0], device=dev)

    def weight(n, k):
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        return scheme.quantize_weight_rows(w)

    if parts[1] == "sweep":
        flush = torch.ones(128 * 1024 * 1024, dtype=torch.float32, device=dev)
        weights = {name: weight(n, k) for name, n, k in SHAPES}
        for m in M_VALUES:
            for name, n, k in SHAPES:
                wq, ws = weights[name]
                x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
                a, ts = native.static_quant(x, fixed)
                flush.sum()
                if m <= 4:  # the fused quant + GEMV launch of scheme.apply
                    native.soft_static_fused_linear(x, wq, fixed, ws, None, output_dtype=torch.bfloat16)
                else:
                    ext.soft_hif8_gemm(a, wq, ts, ws, None, torch.bfloat16)
        torch.cuda.synchronize()
        print(f"profile case {spec}: {len(M_VALUES) * len(SHAPES)} launches ok")
        return
    n, k = {name: (n, k) for name, n, k in SHAPES}[parts[1]]
    m = int(parts[2])
    wq, ws = weight(n, k)
    x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
    a, ts = native.static_quant(x, fixed)
    for _ in range(2 + launches):
        ext.soft_hif8_gemm(a, wq, ts, ws, None, torch.bfloat16)
    torch.cuda.synchronize()
    print(f"profile case {spec}: {2 + launches} launches ok")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of CPU baseline work")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-extra", action="store_true", help="skip the prefill GEMM and attention measurements")
    parser.add_argument("--no-decode", action="store_true", help="skip the configs[4] decoder tok/s measurement")
    parser.add_argument("--profile-case", default=None,
                        help="run one small kernel case for ncu (e.g. gemv:gate_up:1) and exit")
    parser.add_argument("--profile-launches", type=int, default=3)
    parser.add_argument("--tp-allreduce", choices=("peer", "nccl"), default="peer",
                        help="all-reduce of the tensor-parallel sweep's row-parallel calls (N > 1)")
    args = parser.parse_args()
    if args.profile_case:
        run_profile_case(args.profile_case, args.profile_launches)
        return
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        parser.error(f"--gpus {args.gpus} does not match WORLD_SIZE {world}; launch N>1 under torchrun")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
