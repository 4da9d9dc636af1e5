"""Synthetic Qwen3.5-9B-shaped hybrid decoder on the HiF8 static W8A8KV8 path
(configs[4] of the workload) and its BF16 twin.

Architecture of transformers' Qwen3_5 text model (models/qwen3_5/
modeling_qwen3_5.py, config defaults): 32 layers, hidden 4096, SiLU MLP of
12288, every 4th layer gated full attention (16 query / 4 KV heads of 256,
q/k RMSNorm, rotary embedding on 64 of 256 dims, sigmoid output gate), the
others gated-delta-net linear attention (16 key / 32 value heads of 128,
causal conv of 4), vocabulary 248320 with a BF16 LM head.  Weights are
random (N(0, 0.02) projections, seeded per tensor), so every rank of a
tensor-parallel group regenerates the same global tensor and keeps its
slice.

The HiF8 model runs every projection through the plugin path (static
activation quant with a calibrated input scale + HiF8 GEMV/GEMM,
``scheme.apply``) and keeps full-attention K/V in the packed HiF8 page cache
with calibrated per-head scales; its token embedding is HiF8 rows with FP32
row scales, as the exported checkpoint stores it (W8A8HIF8_SOFT, decoded on
lookup).  The BF16 twin runs the same layers with BF16 weights (cuBLAS), a
BF16 embedding and a dense BF16 KV cache.  Both share the fused glue
kernels (``torch.ops.hif8_b200.{rmsnorm, silu_mul, gate_mul, attn_prep,
gdn}``).  Tensor parallelism: q/k/v/gate, the gated-delta-net input
projection and gate/up are column-parallel, o_proj / out_proj / down are
row-parallel followed by an NCCL all-reduce, the LM head is vocab-parallel
with an all-gathered argmax.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

MAX_FINITE = 32768.0


@dataclass
class DecoderConfig:
    hidden: int = 4096
    intermediate: int = 12288
    layers: int = 32
    full_every: int = 4
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 1.0e7
    lin_k_heads: int = 16
    lin_v_heads: int = 32
    lin_dim: int = 128
    conv: int = 4
    vocab: int = 248320
    eps: float = 1e-6
    page: int = 128
    init_std: float = 0.02

    def is_full(self, layer: int) -> bool:
        return (layer + 1) % self.full_every == 0


class _Gen:
    """Deterministic per-tensor random init: the same global tensor on every
    rank, whatever the parallel layout."""

    def __init__(self, seed: int, device):
        self.seed = seed
        self.device = device

    def normal(self, tag: str, shape, std: float):
        import torch

        g = torch.Generator(device=self.device).manual_seed(self._key(tag))
        return (torch.randn(*shape, device=self.device, generator=g) * std).to(torch.bfloat16)

    def uniform(self, tag: str, shape, lo: float, hi: float):
        import torch

        g = torch.Generator(device=self.device).manual_seed(self._key(tag))
        return torch.rand(*shape, device=self.device, generator=g) * (hi - lo) + lo

    def _key(self, tag: str) -> int:
        h = self.seed * 1000003
        for ch in tag:
            h = (h * 131 + ord(ch)) % (1 << 61)
        return h


class _Linear:
    """One projection: BF16 weight (twin) or HiF8 static layer (per-row
    scale = row amax / weight_factor).  ``cols`` = (start, count) keeps only
    those input columns of the weight (a row-parallel shard): the HiF8 bytes
    are quantised over the FULL row first and then sliced, with the full
    row's scale, as a tensor-parallel load of one exported checkpoint
    shards it -- so the shards' partial products sum to the unsharded
    layer's result."""

    def __init__(self, weight_bf16, mode: str, input_scale=None, weight_factor: float = MAX_FINITE, cols=None):
        import torch

        self.mode = mode
        self.out_features = weight_bf16.shape[0]
        c0, cn = cols if cols is not None else (0, weight_bf16.shape[1])
        if mode == "bf16":
            self.weight = weight_bf16[:, c0:c0 + cn].contiguous()
        else:
            from . import scheme

            data, scale = scheme.quantize_weight_rows(weight_bf16, weight_factor)
            self.weight = data[:, c0:c0 + cn].contiguous() if cols is not None else data
            self.weight_scale = scale.reshape(-1).contiguous()
            self.input_scale = (input_scale if input_scale is not None
                                else torch.ones(1, device=weight_bf16.device)).reshape(1).float().contiguous()

    def __call__(self, x):
        import torch

        if self.mode == "bf16":
            return torch.nn.functional.linear(x, self.weight)
        from . import scheme

        return scheme.apply(self, x)

    def partial(self, x):
        """This rank's partial product of a row-parallel projection, before
        the all-reduce: FP32 for the HiF8 layer (summed over the ranks
        before its one BF16 rounding, so the sum equals the unsharded
        projection up to the FP32 summation order); likewise FP32 for the twin
        (cuBLAS with BF16 operands and an FP32 result)."""
        import torch

        if self.mode == "bf16":
            x2 = x.reshape(-1, x.shape[-1])
            return torch.mm(x2, self.weight.t(), out_dtype=torch.float32)
        from . import scheme

        scale = self.input_scale
        factor = scheme.static_scale_factor()
        if factor != 1.0:
            scale = scale * factor
        return torch.ops.hif8_b200.linear_partial_f32(x.reshape(-1, x.shape[-1]).contiguous(), self.weight, scale,
                                                      self.weight_scale)


class PeerReducer:
    """Tensor-parallel all-reduce of a decode step's row-parallel partials,
    fused with the residual add + RMSNorm that follows every one of them
    (``torch.ops.hif8_b200.peer_allreduce_rmsnorm``) or alone (``sum``):
    each rank's buffer is mapped by its peers over NVLink through exchanged
    CUDA IPC handles; every rank pushes its partial into every rank's
    buffer, signals and waits on epoch flags (bounded) and sums the partials
    in rank order from its own memory."""

    def __init__(self, device, rank: int, world: int, max_rows: int, dim: int, group=None,
                 timeout_ns: int = 200_000_000):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import cabi

        lib = cabi.library()
        lib.hif8_peer_alloc.restype = ctypes.c_int
        lib.hif8_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
        lib.hif8_peer_open.restype = ctypes.c_int
        lib.hif8_peer_open.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        lib.hif8_peer_close.restype = ctypes.c_int
        lib.hif8_peer_close.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.hif8_peer_buffer_bytes.restype = ctypes.c_size_t
        lib.hif8_peer_buffer_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64]
        self._lib = lib
        self.rank, self.world, self.max_rows, self.dim, self.timeout_ns = rank, world, max_rows, dim, timeout_ns
        nbytes = lib.hif8_peer_buffer_bytes(world, max_rows, dim)
        torch.cuda.set_device(device)
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        cabi.check("hif8_peer_alloc", lib.hif8_peer_alloc(nbytes, ctypes.byref(own), handle))
        self._own = own.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        bases, self._opened = [], []
        for q in range(world):
            if q == rank:
                bases.append(self._own)
                continue
            peer = ctypes.c_void_p()
            buf = (ctypes.c_ubyte * 64).from_buffer_copy(handles[q])
            cabi.check("hif8_peer_open", lib.hif8_peer_open(buf, ctypes.byref(peer)))
            bases.append(peer.value)
            self._opened.append(peer.value)
        self.table = torch.tensor(bases, dtype=torch.int64, device=device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.error = torch.zeros(1, dtype=torch.int32, device=device)
        dist.barrier(group=group)  # every rank's buffer is mapped before the first signal

    def __call__(self, local, residual, weight, eps: float, slot: int):
        import torch

        return torch.ops.hif8_b200.peer_allreduce_rmsnorm(local.contiguous(), residual, weight, self.table,
                                                          self.counter, self.error, self.max_rows, self.rank,
                                                          self.world, slot, eps, True, self.timeout_ns)

    def sum(self, local, slot: int):
        """The all-reduced sum of every rank's ``local`` (BF16 rows x dim)."""
        import torch

        return torch.ops.hif8_b200.peer_allreduce(local.contiguous(), self.table, self.counter, self.error,
                                                  self.max_rows, self.rank, self.world, slot, self.timeout_ns)

    def check(self):
        if int(self.error.item()) != 0:
            raise RuntimeError("a peer all-reduce wait timed out")

    def close(self):
        for ptr in self._opened:
            self._lib.hif8_peer_close(ptr, 1)
        self._opened = []
        if self._own:
            self._lib.hif8_peer_close(self._own, 0)
            self._own = None


class Decoder:
    """The model on one rank.  ``mode`` is "hif8" or "bf16"."""

    def __init__(self, cfg: DecoderConfig, mode: str, device, *, seed: int = 0, tp_rank: int = 0, tp_size: int = 1,
                 group=None, max_batch: int = 4, max_ctx: int = 768, calibration: dict | None = None):
        import torch

        from . import kv_cache

        kv_cache.load_ops()
        if mode not in ("hif8", "bf16"):
            raise ValueError(f"mode must be hif8 or bf16, got {mode!r}")
        c = cfg
        for name, total in (("heads", c.heads), ("lin_k_heads", c.lin_k_heads), ("lin_v_heads", c.lin_v_heads),
                            ("intermediate", c.intermediate), ("vocab", c.vocab)):
            if total % tp_size:
                raise ValueError(f"{name}={total} does not split over {tp_size} ranks")
        self.cfg, self.mode, self.device = cfg, mode, torch.device(device)
        self.rank, self.tp, self.group = tp_rank, tp_size, group
        self.max_batch, self.max_ctx = max_batch, max_ctx
        calib = calibration or {}
        gen = _Gen(seed, self.device)
        r, tp = tp_rank, tp_size
        H, D = c.hidden, c.head_dim
        self.heads = c.heads // tp
        self.kv_rep = max(1, tp // c.kv_heads)              # ranks sharing one KV head
        self.kv_local = max(1, c.kv_heads // tp)
        kv0 = (r // self.kv_rep) * self.kv_local if tp > c.kv_heads else r * self.kv_local
        self.kv0 = kv0  # first KV head of this rank
        self.hk, self.hv, dl = c.lin_k_heads // tp, c.lin_v_heads // tp, c.lin_dim
        self.inter = c.intermediate // tp
        self.vocab_local = c.vocab // tp

        def scale_for(tag):
            a = calib.get(tag)
            return None if a is None else torch.tensor([a], device=self.device)

        weight_factor = float(calib.get("weight_factor", MAX_FINITE))

        def lin(tag, w, cols=None):
            return _Linear(w, mode, scale_for(tag), weight_factor, cols)

        def rows(w, start, count):
            return w[start:start + count]

        self.layers = []
        for i in range(c.layers):
            L = {"full": c.is_full(i)}
            L["in_w"] = gen.normal(f"{i}.in_norm", (H,), 0.02)
            L["post_w"] = gen.normal(f"{i}.post_norm", (H,), 0.02)
            if L["full"]:
                wq = gen.normal(f"{i}.q", (c.heads * 2 * D, H), c.init_std)
                wk = gen.normal(f"{i}.k", (c.kv_heads * D, H), c.init_std)
                wv = gen.normal(f"{i}.v", (c.kv_heads * D, H), c.init_std)
                wo = gen.normal(f"{i}.o", (H, c.heads * D), c.init_std)
                w_qkv = torch.cat([rows(wq, r * self.heads * 2 * D, self.heads * 2 * D),
                                   rows(wk, kv0 * D, self.kv_local * D), rows(wv, kv0 * D, self.kv_local * D)])
                L["qkv"] = lin(f"{i}.qkv", w_qkv)
                L["o"] = lin(f"{i}.o", wo, (r * self.heads * D, self.heads * D))
                del wq, wk, wv, wo, w_qkv
                L["q_norm"] = gen.normal(f"{i}.q_norm", (D,), 0.02)
                L["k_norm"] = gen.normal(f"{i}.k_norm", (D,), 0.02)
                ks = calib.get(f"{i}.k_scale")
                vs = calib.get(f"{i}.v_scale")
                L["k_scale"] = (torch.tensor(ks[kv0:kv0 + self.kv_local], device=self.device) if ks
                                else torch.ones(self.kv_local, device=self.device))
                L["v_scale"] = (torch.tensor(vs[kv0:kv0 + self.kv_local], device=self.device) if vs
                                else torch.ones(self.kv_local, device=self.device))
            else:
                kd, vd = c.lin_k_heads * dl, c.lin_v_heads * dl
                w_in = gen.normal(f"{i}.lin_in", (2 * kd + 2 * vd + 2 * c.lin_v_heads, H), c.init_std)
                q0, k0, v0, z0 = 0, kd, 2 * kd, 2 * kd + vd
                b0, a0 = 2 * kd + 2 * vd, 2 * kd + 2 * vd + c.lin_v_heads
                lq, lk, lv = self.hk * dl, self.hk * dl, self.hv * dl
                w_loc = torch.cat([rows(w_in, q0 + r * lq, lq), rows(w_in, k0 + r * lk, lk), rows(w_in, v0 + r * lv, lv),
                                   rows(w_in, z0 + r * lv, lv), rows(w_in, b0 + r * self.hv, self.hv),
                                   rows(w_in, a0 + r * self.hv, self.hv)])
                L["lin_in"] = lin(f"{i}.lin_in", w_loc)
                del w_in, w_loc
                conv = gen.uniform(f"{i}.conv", (2 * kd + vd, c.conv), -0.5, 0.5).to(torch.bfloat16)
                L["conv_w"] = torch.cat([rows(conv, q0 + r * lq, lq), rows(conv, k0 + r * lk, lk),
                                         rows(conv, v0 + r * lv, lv)]).contiguous()
                a_log = gen.uniform(f"{i}.A", (c.lin_v_heads,), 1e-3, 16.0).log()
                L["a_log"] = a_log[r * self.hv:(r + 1) * self.hv].clone()
                L["dt_bias"] = torch.ones(self.hv, device=self.device)
                L["gdn_norm"] = (1.0 + gen.normal(f"{i}.gdn_norm", (dl,), 0.02).float()).to(torch.bfloat16)
                w_out = gen.normal(f"{i}.lin_out", (H, vd), c.init_std)
                L["lin_out"] = lin(f"{i}.lin_out", w_out, (r * lv, lv))
                del w_out
            w_gate = gen.normal(f"{i}.gate", (c.intermediate, H), c.init_std)
            w_up = gen.normal(f"{i}.up", (c.intermediate, H), c.init_std)
            L["gate_up"] = lin(f"{i}.gate_up", torch.cat([rows(w_gate, r * self.inter, self.inter),
                                                          rows(w_up, r * self.inter, self.inter)]))
            del w_gate, w_up
            w_down = gen.normal(f"{i}.down", (H, c.intermediate), c.init_std)
            L["down"] = lin(f"{i}.down", w_down, (r * self.inter, self.inter))
            del w_down
            self.layers.append(L)
        embed = gen.normal("embed", (c.vocab, H), c.init_std)
        if mode == "hif8":
            # the exported checkpoint's W8A8HIF8_SOFT token embedding: HiF8
            # rows with FP32 row scales (the projections' calibrated row
            # factor), requested rows decoded on lookup
            from . import checkpoint, scheme

            data, scale = scheme.quantize_weight_rows(embed, weight_factor)
            self.embed = checkpoint.Hif8Embedding(data, scale)
            del embed
        else:
            self.embed = embed
        self.final_w = gen.normal("final_norm", (H,), 0.02)
        head = gen.normal("lm_head", (c.vocab, H), c.init_std)
        self.lm_head = head[r * self.vocab_local:(r + 1) * self.vocab_local].clone()  # frees the full head
        del head
        self._alloc_state()
        self.calib_amax: dict | None = None  # set to a dict to record calibration samples (BF16 twin)
        self._graphs: dict[int, tuple] = {}
        self.peer: PeerReducer | None = None  # decode-step all-reduce over peer memory (enable_peer_allreduce)
        self._fused_reduce = False
        # Glue kernels fused into the prologue of the GEMV they feed on decode
        # steps ("rmsnorm", "silu_mul", "gate_mul").  Every CTA of the fused
        # GEMV recomputes the glue for its K slice, so only the residual +
        # RMSNorm of single-row steps pays off (measured on B200 at the 9B
        # shape: batch 1 +3.7 % tok/s; at batch 4 and for the elementwise glue
        # the fused prologue costs as much as or more than the launch it saves).
        self.fuse_glue = {"rmsnorm"}
        self.fuse_glue_max_rows = 1
        self._fuse_glue = False
        self._site = 0

    def enable_peer_allreduce(self):
        """Decode steps (one token per sequence) all-reduce the row-parallel
        partials inside the following residual + RMSNorm kernel, over peer
        memory, instead of NCCL."""
        if self.tp > 1 and self.peer is None:
            self.peer = PeerReducer(self.device, self.rank, self.tp, self.max_batch, self.cfg.hidden, self.group)

    # ---------------------------------------------------------------- state --
    def _alloc_state(self):
        import torch

        c, B, dev = self.cfg, self.max_batch, self.device
        # per value head: the convolution history of its q, k and v channels
        self.conv_state = [torch.zeros(B, self.hv, 3, c.lin_dim, c.conv - 1, device=dev) if not L["full"] else None
                           for L in self.layers]
        self.rec_state = [torch.zeros(B, self.hv, c.lin_dim, c.lin_dim, device=dev) if not L["full"] else None
                          for L in self.layers]
        if self.mode == "hif8":
            self.blocks_per_seq = (self.max_ctx + c.page - 1) // c.page
            nb = B * self.blocks_per_seq
            shape = (nb, c.page, self.kv_local, c.head_dim + 4)
            self.k_cache = [torch.zeros(shape, dtype=torch.uint8, device=dev) if L["full"] else None
                            for L in self.layers]
            self.v_cache = [torch.zeros(shape, dtype=torch.uint8, device=dev) if L["full"] else None
                            for L in self.layers]
            self.block_table = torch.arange(nb, dtype=torch.int32, device=dev).view(B, self.blocks_per_seq)
        else:
            shape = (B, self.max_ctx, self.kv_local, c.head_dim)
            self.k_cache = [torch.zeros(shape, dtype=torch.bfloat16, device=dev) if L["full"] else None
                            for L in self.layers]
            self.v_cache = [torch.zeros(shape, dtype=torch.bfloat16, device=dev) if L["full"] else None
                            for L in self.layers]

    def reset(self):
        for t in self.conv_state + self.rec_state:
            if t is not None:
                t.zero_()

    # --------------------------------------------------------------- blocks --
    def _all_reduce(self, y):
        """Sum of the row-parallel partials (BF16 result): NCCL, or deferred
        to the next norm when the step fuses it (returns the partial
        unchanged then)."""
        if self.tp > 1 and not self._fused_reduce:
            import torch
            import torch.distributed as dist

            dist.all_reduce(y, group=self.group)
            if y.dtype != torch.bfloat16:
                y = y.to(torch.bfloat16)  # the one rounding of the FP32 sum
        return y

    def _row_proj(self, tag, lin, x):
        """A row-parallel projection (o, out, down): the plain projection on
        one GPU, this rank's partial product under tensor parallelism."""
        if self.tp == 1:
            return self._proj(tag, lin, x)
        if self.calib_amax is not None:
            self._record(tag, x)
        return lin.partial(x)

    def _norm(self, x, residual, weight):
        """(1 + w) RMSNorm of x + residual; with a fused reduce x is this
        rank's partial and the all-reduce happens inside the norm kernel."""
        import torch

        if self._fused_reduce and residual is not None:
            slot = self._site % 2
            self._site += 1
            return self.peer(x, residual, weight, self.cfg.eps, slot)
        return torch.ops.hif8_b200.rmsnorm(x, residual, weight, self.cfg.eps, True)

    def _record(self, tag, x):
        """Calibration: keep a bounded sample of the values seen at ``tag``."""
        flat = x.detach().reshape(-1)
        if flat.numel() > _CALIB_SAMPLES:
            step = flat.numel() // _CALIB_SAMPLES
            flat = flat[::step][:_CALIB_SAMPLES]
        self.calib_amax.setdefault(tag, []).append(flat.clone())

    def _proj(self, tag, lin, x):
        if self.calib_amax is not None:
            self._record(tag, x)
        return lin(x)

    def _glue(self, kind: int, x, aux, lin, norm_w=None):
        """Decode-step projection with its glue (1 silu_mul, 2 gate_mul, 3
        residual + RMSNorm) fused into the quantisation prologue of the GEMV:
        (out, new residual)."""
        import torch

        return torch.ops.hif8_b200.glue_linear(x, aux, norm_w, kind, self.cfg.eps, True, lin.weight, lin.input_scale,
                                               lin.weight_scale)

    def _norm_proj(self, tag, x, residual, norm_w, lin):
        """First projection of a block on RMSNorm(x + residual): one fused
        launch on decode steps without a peer reduce, else norm then
        projection.  Returns (projection, new residual)."""
        if self._fuse_glue and "rmsnorm" in self.fuse_glue and not self._fused_reduce:
            return self._glue(3, x, residual, lin, norm_w)
        h, residual = self._norm(x, residual, norm_w)
        return self._proj(tag, lin, h), residual

    def _attention(self, i, L, qkv, batch: int, T: int, positions, seq_lens, slots):
        """qkv projection [batch * T, ...] -> attention output [batch * T, hidden]."""
        import torch

        c = self.cfg
        q, gate, k, v = torch.ops.hif8_b200.attn_prep(qkv, positions, L["q_norm"], L["k_norm"], self.heads,
                                                      self.kv_local, c.head_dim, c.rotary_dim, c.eps, c.rope_theta)
        if self.calib_amax is not None:  # per global KV head
            for j in range(self.kv_local):
                self._record(f"{i}.k.{self.kv0 + j}", k[:, j])
                self._record(f"{i}.v.{self.kv0 + j}", v[:, j])
        scale = 1.0 / math.sqrt(c.head_dim)
        if self.mode == "hif8":
            torch.ops.hif8_b200.kv_cache_write(k, v, L["k_scale"], L["v_scale"], slots, self.k_cache[i],
                                               self.v_cache[i], None)
            q_start = torch.arange(0, batch * T + 1, T, dtype=torch.int32, device=self.device)
            attn = torch.ops.hif8_b200.paged_attention(q, self.k_cache[i], self.v_cache[i],
                                                       self.block_table[:batch].contiguous(), seq_lens, q_start,
                                                       self.max_ctx, scale, True)
        else:
            kc, vc = self.k_cache[i], self.v_cache[i]
            b_idx = torch.arange(batch, device=self.device).repeat_interleave(T)
            kc.index_put_((b_idx, positions.long()), k)
            vc.index_put_((b_idx, positions.long()), v)
            qh = q.view(batch, T, self.heads, c.head_dim).transpose(1, 2)
            keys = kc[:batch].transpose(1, 2)
            vals = vc[:batch].transpose(1, 2)
            kpos = torch.arange(self.max_ctx, device=self.device)
            qpos = positions.view(batch, T).long()
            mask = (kpos.view(1, 1, 1, -1) <= qpos.view(batch, 1, T, 1))
            attn = torch.nn.functional.scaled_dot_product_attention(qh, keys, vals, attn_mask=mask, scale=scale,
                                                                    enable_gqa=True)
            attn = attn.transpose(1, 2).reshape(batch * T, self.heads, c.head_dim)
        attn = attn.reshape(batch * T, -1).contiguous()
        if self._fuse_glue and "gate_mul" in self.fuse_glue and self.tp == 1:
            return self._all_reduce(self._glue(2, attn, gate, L["o"])[0])
        out = torch.ops.hif8_b200.gate_mul(attn, gate)
        return self._all_reduce(self._row_proj(f"{i}.o", L["o"], out))

    def _gdn(self, i, L, proj, batch: int, T: int):
        import torch

        core = torch.ops.hif8_b200.gdn(proj, T, self.hk, self.hv, L["conv_w"], L["a_log"], L["dt_bias"],
                                       L["gdn_norm"], self.conv_state[i][:batch], self.rec_state[i][:batch],
                                       self.cfg.eps)
        return self._all_reduce(self._row_proj(f"{i}.lin_out", L["lin_out"], core))

    def _mlp(self, i, L, gu):
        import torch

        if self._fuse_glue and "silu_mul" in self.fuse_glue and self.tp == 1:
            return self._all_reduce(self._glue(1, gu, None, L["down"])[0])
        act = torch.ops.hif8_b200.silu_mul(gu)
        return self._all_reduce(self._row_proj(f"{i}.down", L["down"], act))

    def forward(self, tokens, positions, batch: int, T: int, seq_lens, slots):
        """tokens / positions [batch * T] (sequence-major) -> logits of each
        sequence's last token [batch, vocab_local] (FP32)."""
        import torch

        c = self.cfg
        self._fused_reduce = self.peer is not None and T == 1 and batch <= self.max_batch
        # decode steps fuse the glue kernels into the GEMV prologues
        self._fuse_glue = (self.mode == "hif8" and T == 1 and batch <= self.fuse_glue_max_rows
                           and self.calib_amax is None)
        self._site = 0
        x = self.embed(tokens) if self.mode == "hif8" else self.embed.index_select(0, tokens)
        residual = None
        for i, L in enumerate(self.layers):
            if L["full"]:
                qkv, residual = self._norm_proj(f"{i}.qkv", x, residual, L["in_w"], L["qkv"])
                x = self._attention(i, L, qkv, batch, T, positions, seq_lens, slots)
            else:
                proj, residual = self._norm_proj(f"{i}.lin_in", x, residual, L["in_w"], L["lin_in"])
                x = self._gdn(i, L, proj, batch, T)
            gu, residual = self._norm_proj(f"{i}.gate_up", x, residual, L["post_w"], L["gate_up"])
            x = self._mlp(i, L, gu)
        if T > 1:
            last = torch.arange(batch, device=self.device) * T + (T - 1)
            x, residual = x.index_select(0, last).contiguous(), residual.index_select(0, last).contiguous()
        h, _ = self._norm(x, residual, self.final_w)
        self._fused_reduce = False
        self._fuse_glue = False
        return torch.nn.functional.linear(h, self.lm_head).float()

    def argmax(self, logits):
        """Greedy token over the full (vocab-parallel) vocabulary."""
        import torch

        val, idx = logits.max(dim=-1)
        idx = idx + self.rank * self.vocab_local
        if self.tp == 1:
            return idx
        import torch.distributed as dist

        both = torch.stack([val, idx.float()], dim=-1)  # vocab < 2^24: exact in FP32
        gathered = [torch.empty_like(both) for _ in range(self.tp)]
        dist.all_gather(gathered, both, group=self.group)
        g = torch.stack(gathered)  # [tp, batch, 2]
        best = g[..., 0].argmax(dim=0)
        return g[..., 1].gather(0, best.unsqueeze(0)).squeeze(0).long()

    # ------------------------------------------------------------- serving --
    def _slots(self, batch: int, positions):
        import torch

        if self.mode != "hif8":
            return None
        b_idx = torch.arange(batch, device=self.device).repeat_interleave(positions.numel() // batch)
        blk = self.block_table[b_idx, (positions // self.cfg.page).long()].long()
        return blk * self.cfg.page + (positions % self.cfg.page).long()

    def prefill(self, prompt):
        """prompt [batch, T] int64 -> first generated token [batch]."""
        import torch

        batch, T = prompt.shape
        positions = torch.arange(T, dtype=torch.int32, device=self.device).repeat(batch)
        seq_lens = torch.full((batch,), T, dtype=torch.int32, device=self.device)
        logits = self.forward(prompt.reshape(-1), positions, batch, T, seq_lens, self._slots(batch, positions))
        return self.argmax(logits)

    def _decode_step(self, batch: int, tokens, pos):
        import torch

        seq_lens = pos + 1
        logits = self.forward(tokens, pos, batch, 1, seq_lens, self._slots(batch, pos))
        tokens.copy_(self.argmax(logits))
        pos.add_(1)

    def decode_graph(self, batch: int):
        """A CUDA graph of one decode step for ``batch`` sequences; it reads
        and advances its own token / position buffers."""
        import torch

        if batch in self._graphs:
            return self._graphs[batch]
        tokens = torch.zeros(batch, dtype=torch.int64, device=self.device)
        pos = torch.zeros(batch, dtype=torch.int32, device=self.device)
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        saved = [t.clone() for t in self.conv_state + self.rec_state if t is not None]
        with torch.cuda.stream(stream):
            self._decode_step(batch, tokens, pos)  # warm the allocator pool on the capture stream
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                self._decode_step(batch, tokens, pos)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        for t, s in zip([t for t in self.conv_state + self.rec_state if t is not None], saved):
            t.copy_(s)
        self._graphs[batch] = (graph, tokens, pos)
        return self._graphs[batch]

    def release_graphs(self):
        self._graphs.clear()


_CALIB_SAMPLES = 1 << 16


def best_static_scale(samples) -> float:
    """The fixed scale with the least mean squared error of
    decode(static_quant(x / s)) * s over ``samples``: candidates from
    amax / 32768 upwards in quarter octaves (the exact-codebook search of the
    reference's calibration.py:470-510, on a plain MSE objective)."""
    import torch

    from . import native

    x = samples.reshape(1, -1).to(torch.bfloat16).contiguous()
    xf = x.float()
    amax = float(xf.abs().max())
    if not math.isfinite(amax) or amax == 0.0:
        return 1.0
    best, best_s = None, amax / MAX_FINITE
    for i in range(0, 4 * 18 + 1):
        s = amax / MAX_FINITE * 2.0 ** (i / 4.0)
        data, row_scale = native.static_quant(x, torch.tensor([s], device=x.device))
        err = float((native.scaled_decode(data, row_scale).float() - xf).pow(2).mean())
        if best is None or err < best:
            best, best_s = err, s
    return best_s


def best_weight_factor(weight) -> float:
    """The per-row factor f (scale = row amax / f) with the least squared
    error over a sample of rows of ``weight``."""
    import torch

    from . import native, scheme

    rows = weight[:: max(1, weight.shape[0] // 256)][:256].contiguous()
    best, best_f = None, MAX_FINITE
    for i in range(0, 2 * 14 + 1):
        f = MAX_FINITE / 2.0 ** (i / 2.0)
        data, scale = scheme.quantize_weight_rows(rows, f)
        deq = native.scaled_decode(data, scale.reshape(-1).contiguous()).float()
        err = float((deq - rows.float()).pow(2).mean())
        if best is None or err < best:
            best, best_f = err, f
    return best_f


def calibrate(cfg: DecoderConfig, device, *, seed: int = 0, tokens: int = 64, tp_rank: int = 0, tp_size: int = 1,
              group=None) -> dict:
    """Static HiF8 scales from the BF16 twin run on a seeded calibration
    prompt: every projection's input scale, the per-KV-head K and V scales,
    and the weights' per-row scale factor, each by least squared error
    against the HiF8 codebook."""
    import torch

    twin = Decoder(cfg, "bf16", device, seed=seed, tp_rank=tp_rank, tp_size=tp_size, group=group, max_batch=1,
                   max_ctx=max(tokens, 64))
    twin.calib_amax = {}
    g = torch.Generator(device=device).manual_seed(seed + 17)
    prompt = torch.randint(0, cfg.vocab, (1, tokens), device=device, generator=g)
    with torch.no_grad():
        twin.prefill(prompt)
    samples = {tag: torch.cat(v) for tag, v in twin.calib_amax.items()}
    for i in range(cfg.layers):  # every rank lists every KV head (empty where not local)
        if cfg.is_full(i):
            for h in range(cfg.kv_heads):
                for kind in ("k", "v"):
                    samples.setdefault(f"{i}.{kind}.{h}", torch.zeros(0, device=device, dtype=torch.bfloat16))
    weight_factor = best_weight_factor(twin.layers[0]["gate_up"].weight)
    del twin
    if tp_size > 1:  # every rank's samples of a tag -> one pooled sample
        import torch.distributed as dist

        # one weight factor for the whole model: each rank measured it on its
        # own shard, and ranks quantising with different factors would not sum
        # to the single-GPU model (rank 0's choice is broadcast)
        wf = torch.tensor([weight_factor], dtype=torch.float64, device=device)
        dist.broadcast(wf, src=0, group=group)
        weight_factor = float(wf.item())

        pooled = {}
        for tag in sorted(samples):
            t = samples[tag].float()
            n = torch.tensor([t.numel()], device=device)
            dist.all_reduce(n, op=dist.ReduceOp.MAX, group=group)
            padded = torch.zeros(int(n), device=device)
            padded[:t.numel()] = t
            parts = [torch.empty_like(padded) for _ in range(tp_size)]
            dist.all_gather(parts, padded, group=group)
            pooled[tag] = torch.cat(parts)
        samples = pooled
    calib: dict = {"weight_factor": weight_factor}
    kv: dict = {}
    for tag, t in samples.items():
        s = best_static_scale(t)
        parts = tag.split(".")
        if len(parts) == 3 and parts[1] in ("k", "v"):
            kv.setdefault(f"{parts[0]}.{parts[1]}_scale", {})[int(parts[2])] = s
        else:
            calib[tag] = s
    for tag, per_head in kv.items():
        calib[tag] = [per_head[h] for h in sorted(per_head)]
    torch.cuda.empty_cache()
    return calib


def forced_logits(model: Decoder, prompt, next_tokens=None, steps: int = 8):
    """Logits of the prefill of ``prompt`` [batch, T] and of ``steps``
    single-token decode steps (eager, the decode path: fused reductions and
    glue as the CUDA-graph step uses them).  Decode step s is fed
    ``next_tokens[s]`` when given (teacher forcing, so two models can be
    compared step by step without a flipped near-tie changing everything
    after it), else this model's own greedy token.  Returns (list of this
    rank's FP32 logits [batch, vocab_local], list of greedy tokens [batch])."""
    import torch

    batch, T = prompt.shape
    model.reset()
    logits, tokens = [], []
    with torch.no_grad():
        positions = torch.arange(T, dtype=torch.int32, device=model.device).repeat(batch)
        seq_lens = torch.full((batch,), T, dtype=torch.int32, device=model.device)
        lg = model.forward(prompt.reshape(-1), positions, batch, T, seq_lens, model._slots(batch, positions))
        for s in range(steps + 1):
            logits.append(lg.clone())
            tokens.append(model.argmax(lg))
            if s == steps:
                break
            tok = next_tokens[s] if next_tokens is not None else tokens[-1]
            pos = torch.full((batch,), T + s, dtype=torch.int32, device=model.device)
            lg = model.forward(tok.contiguous(), pos, batch, 1, pos + 1, model._slots(batch, pos))
    if model.peer is not None:
        model.peer.check()
    return logits, tokens


def measure_decode(model: Decoder, batch: int, *, prompt_len: int = 512, gen: int = 256, seed: int = 1) -> dict:
    """tok/s of ``gen`` greedy decode steps (CUDA-graph replays) after a
    ``prompt_len`` prefill, batch sequences; device time by CUDA events."""
    import torch

    g = torch.Generator(device=model.device).manual_seed(seed)
    prompt = torch.randint(0, model.cfg.vocab, (batch, prompt_len), device=model.device, generator=g)
    graph, tokens, pos = model.decode_graph(batch)
    for rep in range(2):  # warm-up pass, then the measured pass
        model.reset()
        with torch.no_grad():
            first = model.prefill(prompt)
        tokens.copy_(first)
        pos.fill_(prompt_len)
        torch.cuda.synchronize(model.device)
        steps = 8 if rep == 0 else gen
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize(model.device)
    ms = start.elapsed_time(end)
    return {"batch": batch, "prompt": prompt_len, "generated": gen, "ms_per_step": ms / gen,
            "tok_s": batch * gen / (ms * 1e-3), "last_tokens": tokens.tolist()}
