// Prefill GEMM for HiF8 W8A8 on the 5th-generation tensor cores (tcgen05).
//
//   y[m, n] = cast((acc[m, n] * cs[n]) * ts[m] + bias[n]),
//   acc = sum_k decode(a[m, k]) * decode(w[n, k])   (BF16 operands, FP32 in TMEM)
//
// Every finite HiF8 code is exactly a BF16, so decoding both operands to BF16
// and accumulating in FP32 is exact up to the summation order.
//
// Work split per CTA (one 128-channel x BN-token output tile, 10 warps):
//   * the activation is decoded once per call into a BF16 workspace
//     [M, K]; warp 0 streams its BN x 64 tiles with TMA (128-byte swizzle)
//     into a 4-stage shared-memory ring -- the MMA's B operand -- together
//     with the raw 128 x 64-byte HiF8 weight tile of the same stage (64-byte
//     swizzle, so the row reads below are bank-conflict free);
//   * warps 2..9 own one weight row per lane (128 rows, two warps per row
//     quarter, 32 bytes of each 64-byte stage each), decode it with the
//     lane-replicated shared-memory table and write the BF16 values straight
//     into tensor memory with tcgen05.st: the MMA's A operand lives in TMEM,
//     so the decoded weight never goes back to shared memory;
//   * warp 1 issues tcgen05.mma (M=128, N=BN, K=16) from one thread and
//     returns each stage with tcgen05.commit;
//   * warps 2..9 then read the FP32 accumulator with tcgen05.ld (each warp
//     half the columns of its 32-lane quarter), apply the channel scale,
//     token scale and bias, stage the tile in shared memory and write it with
//     one TMA tensor store.
// Every wait is bounded; a timed-out wait is counted in the error word of the
// workspace and the kernel runs to completion.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "linear.cuh"

namespace hif8 {

constexpr int kTcBM = 128;      // weight rows (output channels) per tile = TMEM lanes
constexpr int kTcBK = 64;       // K per stage: one 128-byte swizzle atom of BF16
constexpr int kTcStages = 4;
constexpr int kDecoderWarps = 8;
constexpr int kTcThreads = 32 * (2 + kDecoderWarps);  // TMA warp, MMA warp, decoder/epilogue warps
constexpr int kTcLut = 256 * 256;  // lane-replicated decode table (see gemv.cu)
constexpr uint64_t kWaitNs = 100ull * 1000 * 1000;  // 100 ms per pipeline wait

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(addr), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity.  A wait that outlives
// kWaitNs raises the CTA's abort flag, after which every later wait returns
// false at once, so a broken pipeline ends the kernel within milliseconds.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
  const uint32_t addr = smem_addr(bar);
  for (int i = 0; i < 64; ++i)
    if (mbar_try(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!*abort) {
    if (mbar_try(addr, parity)) return true;
    if (global_ns() - t0 > kWaitNs) *abort = 1;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// K-major, 128-byte swizzle UMMA shared-memory descriptor (8-row atoms of
// 128 bytes, atoms 1024 bytes apart).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *p) {
  const uint64_t addr = smem_addr(p);
  uint64_t d = (addr >> 4) & 0x3FFFull;   // start address
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused with swizzle)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset between 8-row atoms
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: BF16 A and B (both K-major), FP32 D.
template <int BN>
__device__ __forceinline__ constexpr uint32_t instr_desc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ uint32_t lut_pair(const uint8_t *lut, uint32_t word, uint32_t lane4, bool high) {
  const uint32_t e0 = *reinterpret_cast<const uint32_t *>(lut + __byte_perm(word, lane4, high ? 0x5524u : 0x5504u));
  const uint32_t e1 = *reinterpret_cast<const uint32_t *>(lut + __byte_perm(word, lane4, high ? 0x5534u : 0x5514u));
  return __byte_perm(e0, e1, 0x5410u);
}

struct TcParams {
  const uint8_t *w;
  const float *ts, *cs;
  const void *bias;
  void *out;
  int *err;
  int m, n, k, bias_dtype, ts_stride;
  int kb_per;  // K blocks per split (blockIdx.z): all of them without split-K
};

template <int OUT>
__device__ __forceinline__ uint32_t to_out_bits(float v) {
  if constexpr (OUT == HIF8_DTYPE_BF16) return f32_to_bf16_bits(v);
  else return f32_to_f16_bits(v);
}

template <int BN, int OUT>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_hif8_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                        const __grid_constant__ CUtensorMap ymap, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled operand stages
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kBBytes = BN * 128;
  constexpr int kWBytes = kTcBM * kTcBK;                    // 128 weight rows x 64 bytes
  uint8_t *b_stages = smem;                                  // [stages][BN][128 B], 128-byte swizzle
  uint8_t *w_stages = b_stages + kTcStages * kBBytes;       // [stages][128][64 B], 64-byte swizzle
  uint8_t *lut = w_stages + kTcStages * kWBytes;            // 64 KB
  uint64_t *bars = reinterpret_cast<uint64_t *>(lut + kTcLut);
  uint64_t *full_a = bars, *full_b = bars + kTcStages, *empty = bars + 2 * kTcStages;
  uint64_t *accum_full = bars + 3 * kTcStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum_full + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // token tiles vary fastest, so the CTAs sharing one weight tile run together
  // and the weight crosses HBM once while the BF16 activation stays in L2
  const int m0 = blockIdx.x * BN, n0 = blockIdx.y * kTcBM;
  constexpr uint32_t kTmemCols = BN + 4 * 32 <= 256 ? 256 : 512;
  // split-K: CTA z takes K blocks [kb0, kb0 + nkb) and stores its FP32
  // partial tile into slice z of a [splits][M][N] buffer
  const int kb0 = blockIdx.z * p.kb_per;
  const int nkb = min(p.k / kTcBK - kb0, p.kb_per);

  // ---- set-up: barriers, TMEM, decode table --------------------------------
  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full_a[s], kDecoderWarps);  // one arrival per decoding warp
      mbar_init(&full_b[s], 1);  // TMA transactions (activation + weight tile)
      mbar_init(&empty[s], 1);   // tcgen05.commit
    }
    mbar_init(accum_full, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // whole warp allocates: BN accumulator columns + 4 stages x 32 A columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // lane-replicated table: a warp loads 16 entries (one per lane) and
  // writes each as 32 consecutive words
  for (int b0 = warp * 16; b0 < 256; b0 += (kTcThreads / 32) * 16) {
    const uint32_t mine = g_decode_f32.v[b0 + (lane & 15)] >> 16;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      reinterpret_cast<uint32_t *>(lut)[(b0 + j) * 64 + lane] = __shfl_sync(0xFFFFFFFFu, mine, j);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t d_tmem = tmem;                  // columns [0, BN)
  const uint32_t a_tmem0 = tmem + (uint32_t)BN;  // stage s: columns BN + 32 s

  if (warp == 0) {
    // ---- TMA producer of the activation (B) and raw weight tiles -------------
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kTcStages;
        if (kb >= kTcStages && !mbar_wait(&empty[s], ((kb / kTcStages) - 1) & 1, abort)) atomicAdd(p.err, 1);
        mbar_expect_tx(&full_b[s], kBBytes + kWBytes);
        tma_load_2d(b_stages + s * kBBytes, &xmap, (kb0 + kb) * kTcBK, m0, &full_b[s]);
        tma_load_2d(w_stages + s * kWBytes, &wmap, (kb0 + kb) * kTcBK, n0, &full_b[s]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc_bf16<BN>();
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kTcStages;
        const uint32_t parity = (kb / kTcStages) & 1;
        bool ok = mbar_wait(&full_a[s], parity, abort);
        ok = mbar_wait(&full_b[s], parity, abort) && ok;
        if (!ok) atomicAdd(p.err, 1);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t bdesc = smem_desc_sw128(b_stages + s * kBBytes);
#pragma unroll
        for (int j = 0; j < kTcBK / 16; ++j)  // K = 16 per MMA: 32 bytes along the swizzled row
          mma_ts(d_tmem, a_tmem0 + s * 32 + j * 8, bdesc + (uint64_t)(j * 2), idesc, (kb | j) != 0);
        mma_commit(&empty[s]);
      }
      mma_commit(accum_full);
    }
  } else {
    // ---- weight decoders (warps 2..9), then the epilogue ---------------------
    // Warp w owns TMEM lane quarter w % 4 (the only lanes it may access) and
    // half h of every 64-byte stage: lane = one weight row, 32 bytes per stage.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int n = n0 + row;
    const uint32_t lane4 = (uint32_t)lane << 2;
    const uint32_t a_lane = (uint32_t)(quarter * 32) << 16;
    // this lane's 32 bytes of the stage: 16-byte chunks 2h and 2h+1 of row
    // `row`, placed by the 64-byte swizzle at chunk c ^ ((row >> 1) & 3)
    const int sw = (row >> 1) & 3;
    const int off0 = row * kTcBK + ((2 * half) ^ sw) * 16;
    const int off1 = row * kTcBK + ((2 * half + 1) ^ sw) * 16;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kTcStages;
      const uint32_t parity = (kb / kTcStages) & 1;
      // the weight tile of this stage has landed (which also means the MMAs
      // that read A stage s four stages ago have completed)
      if (!mbar_wait(&full_b[s], parity, abort)) atomicAdd(p.err, 1);
      if (kb >= kTcStages && !mbar_wait(&empty[s], parity ^ 1, abort)) atomicAdd(p.err, 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint8_t *ws = w_stages + s * kWBytes;
      const uint4 x0 = *reinterpret_cast<const uint4 *>(ws + off0);
      const uint4 x1 = *reinterpret_cast<const uint4 *>(ws + off1);
      const uint32_t words[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      uint32_t v[16];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[q * 2] = lut_pair(lut, words[q], lane4, false);
        v[q * 2 + 1] = lut_pair(lut, words[q], lane4, true);
      }
      tmem_st16(a_tmem0 + s * 32 + half * 16 + a_lane, v);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_a[s]);
    }

    // epilogue: lane = output channel n, columns = tokens; warp half h takes
    // columns [h * BN / 2, (h + 1) * BN / 2).  The tile is staged as
    // [BN tokens][128 channels] in the (now idle) activation ring and written
    // by one TMA tensor store: per-lane 2-byte stores to BN different output
    // rows cost more than the whole main loop's issue budget.
    const bool n_ok = n < p.n;
    const float cs = n_ok ? p.cs[n] : 0.f;
    float bias = 0.f;
    if (n_ok && p.bias) {
      const uint16_t h = static_cast<const uint16_t *>(p.bias)[n];
      bias = p.bias_dtype == HIF8_DTYPE_BF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
    }
    // token scales, fetched while the last MMAs run: lane l holds
    // ts[m0 + c0 + 32 c + l] of chunk c, broadcast by shuffles below
    constexpr int kChunks = BN / 64;  // 32-token chunks per warp half
    const int c0 = half * (BN / 2);
    float tsr[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int m = m0 + c0 + c * 32 + lane;
      tsr[c] = m < p.m ? p.ts[(int64_t)m * p.ts_stride] : 0.f;
    }
    if (!mbar_wait(accum_full, 0, abort)) atomicAdd(p.err, 1);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // [BN][128] output values; an FP32 tile (BN x 512 bytes) fills the
    // activation ring exactly (kTcStages x BN x 128 bytes)
    static_assert(kTcStages * kTcBK * 2 >= kTcBM * 4, "the FP32 output tile fits the activation ring");
    uint16_t *stage_out = reinterpret_cast<uint16_t *>(b_stages);
    float *stage_out32 = reinterpret_cast<float *>(b_stages);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      uint32_t acc[32];
      tmem_ld32(d_tmem + (uint32_t)(c0 + c * 32) + a_lane, acc);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const float ts = __shfl_sync(0xFFFFFFFFu, tsr[c], q);
        float val = __uint_as_float(acc[q]) * cs;
        val = val * ts;
        val += bias;
        if constexpr (OUT == HIF8_DTYPE_F32) stage_out32[(c0 + c * 32 + q) * kTcBM + row] = val;
        else stage_out[(c0 + c * 32 + q) * kTcBM + row] = (uint16_t)to_out_bits<OUT>(val);
      }
    }
    // make the staged tile visible to the TMA engine, then one thread stores it
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("bar.sync 1, %0;" ::"n"(kDecoderWarps * 32) : "memory");
    if (warp == 2 && lane == 0) {
      if (gridDim.z > 1)  // split-K partial: slice blockIdx.z of the [splits][M][N] buffer
        asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                     ::"l"(&ymap), "r"(n0), "r"(m0), "r"((int)blockIdx.z), "r"(smem_addr(stage_out))
                     : "memory");
      else
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                     ::"l"(&ymap), "r"(n0), "r"(m0), "r"(smem_addr(stage_out))
                     : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // smem read before the CTA exits
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------- CTA-pair variant ---
//
// The same pipeline on a pair of CTAs (a 2-CTA cluster on two SMs) issuing
// tcgen05.mma.cta_group::2 with M = 256: the pair computes 256 weight rows x
// 256 tokens.  Each CTA decodes its own 128 weight rows into its own tensor
// memory (the A operand of its half) and stages its own 128 of the 256 tokens
// of the BF16 activation (the B operand is split between the two CTAs'
// shared memory at the same offset); each CTA's tensor memory receives its
// 128 rows x 256 tokens of the accumulator.  Per CTA and K block this moves
// 8 KB of weights and 16 KB of activations from L2 for the same 128 x 256 x
// 64 MMA that the single-CTA kernel feeds with 8 + 32 KB.
//
// Barriers (every wait bounded as in the single-CTA kernel):
//   * w_full[s] (each CTA): its weight tile of stage s has landed (TMA);
//   * full_b[s] (leader CTA 0): both CTAs' activation halves have landed --
//     the leader's producer expects both halves' bytes, each CTA's TMA
//     (.cta_group::2) completes its bytes on the leader's barrier;
//   * full_a[s] (leader): all 16 decoding warps of both CTAs have stored
//     their rows of stage s into tensor memory (CTA 1's warps arrive
//     remotely);
//   * empty[s] (each CTA): the MMAs of stage s have completed -- the leader's
//     MMA thread commits to its own and to the peer's barrier;
//   * accum_full (each CTA): every MMA of the tile has completed.
// Both CTAs allocate tensor memory with cta_group::2 from the same warp, and
// a cluster barrier at the end keeps either CTA from exiting (or freeing its
// tensor memory) while the other may still touch its shared memory.
constexpr int kTc2Stages = 6;
constexpr int kTc2BN = 256;           // tokens per pair tile
constexpr int kTc2Half = kTc2BN / 2;  // tokens staged per CTA
constexpr int kTc2Rows = 2 * kTcBM;   // weight rows per pair tile
// Two sets of 8 decoding warps take alternate K blocks (set j the blocks kb
// with kb % 2 == j), so each warp's per-stage chain (table lookups, tensor
// memory store, its wait, the arrive) has two MMA steps of time; set 0 also
// runs the epilogue.
constexpr int kTc2DecSets = 2;
constexpr int kTc2Threads = 32 * (2 + kTc2DecSets * kDecoderWarps);

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared-memory location in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}

// Arrive on a barrier of either CTA of the pair (a shared::cluster address).
// Default (CTA-scope release) semantics, like the local arrivals: what the
// waiting side consumes is tensor memory, ordered by the tcgen05 fences and
// tcgen05.wait::st around the arrive, not shared-memory data.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// arrive on the barrier at a shared::cluster address once the pair's prior
// MMAs have completed
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}

// TMA load into this CTA's shared memory whose bytes complete on the
// leader's barrier (a shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int x, int y,
                                                 uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];"
      ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(leader_bar)
      : "memory");
}

__device__ __forceinline__ constexpr uint32_t instr_desc_bf16_pair() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTc2BN >> 3) << 17) | ((uint32_t)(kTc2Rows >> 4) << 24);
}

template <int OUT>
__global__ void __launch_bounds__(kTc2Threads, 1)
    gemm_hif8_tc_pair_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                             const __grid_constant__ CUtensorMap ymap, const TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kBBytes = kTc2Half * 128;  // this CTA's 128 tokens x 64 K of BF16
  constexpr int kWBytes = kTcBM * kTcBK;   // this CTA's 128 weight rows x 64 bytes
  uint8_t *b_stages = smem;                // [stages][128][128 B], 128-byte swizzle
  uint8_t *w_stages = b_stages + kTc2Stages * kBBytes;
  uint8_t *lut = w_stages + kTc2Stages * kWBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(lut + kTcLut);
  uint64_t *full_a = bars, *full_b = bars + kTc2Stages, *w_full = bars + 2 * kTc2Stages;
  uint64_t *empty = bars + 3 * kTc2Stages, *accum_full = bars + 4 * kTc2Stages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum_full + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the MMAs
  const int m0 = (int)(blockIdx.x >> 1) * kTc2BN;                 // the pair's first token
  const int n0 = (int)blockIdx.y * kTc2Rows + (int)rank * kTcBM;  // this CTA's first weight row
  const int kb0 = blockIdx.z * p.kb_per;
  const int nkb = min(p.k / kTcBK - kb0, p.kb_per);
  constexpr uint32_t kTmemCols = 512;  // 256 accumulator columns + 6 stages x 32 A columns

  if (tid == 0) {
    for (int s = 0; s < kTc2Stages; ++s) {
      mbar_init(&full_a[s], 2 * kDecoderWarps);  // the stage's decoding set in both CTAs (used on the leader)
      mbar_init(&full_b[s], 1);                  // the leader's expect_tx of both halves
      mbar_init(&w_full[s], 1);                  // this CTA's weight tile
      mbar_init(&empty[s], 1);                   // the leader's commit
    }
    mbar_init(accum_full, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // the same warp in both CTAs allocates the pair's columns
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  for (int b0 = warp * 16; b0 < 256; b0 += (kTc2Threads / 32) * 16) {
    const uint32_t mine = g_decode_f32.v[b0 + (lane & 15)] >> 16;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      reinterpret_cast<uint32_t *>(lut)[(b0 + j) * 64 + lane] = __shfl_sync(0xFFFFFFFFu, mine, j);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_barrier();  // both CTAs' barriers are initialised before any remote arrive or TMA
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t d_tmem = tmem;                      // columns [0, 256)
  const uint32_t a_tmem0 = tmem + (uint32_t)kTc2BN;  // stage s: columns 256 + 32 s

  if (warp == 0) {
    // ---- TMA producer: this CTA's weight tile and activation half ------------
    if (lane == 0) {
      const uint32_t leader_full_b0 = map_to_rank(&full_b[0], 0);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kTc2Stages;
        if (kb >= kTc2Stages && !mbar_wait(&empty[s], ((kb / kTc2Stages) - 1) & 1, abort))
          atomicAdd(p.err, 1);
        mbar_expect_tx(&w_full[s], kWBytes);
        tma_load_2d(w_stages + s * kWBytes, &wmap, (kb0 + kb) * kTcBK, n0, &w_full[s]);
        if (rank == 0) mbar_expect_tx(&full_b[s], 2 * kBBytes);
        tma_load_2d_pair(b_stages + s * kBBytes, &xmap, (kb0 + kb) * kTcBK, m0 + (int)rank * kTc2Half,
                         leader_full_b0 + (uint32_t)(s * sizeof(uint64_t)));
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (leader only) ---------------------------------------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = instr_desc_bf16_pair();
      const uint32_t own_empty0 = map_to_rank(&empty[0], 0), peer_empty0 = map_to_rank(&empty[0], 1);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kTc2Stages;
        const uint32_t parity = (kb / kTc2Stages) & 1;
        bool ok = mbar_wait(&full_a[s], parity, abort);
        ok = mbar_wait(&full_b[s], parity, abort) && ok;
        if (!ok) atomicAdd(p.err, 1);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t bdesc = smem_desc_sw128(b_stages + s * kBBytes);
#pragma unroll
        for (int j = 0; j < kTcBK / 16; ++j)
          mma_ts_pair(d_tmem, a_tmem0 + s * 32 + j * 8, bdesc + (uint64_t)(j * 2), idesc, (kb | j) != 0);
        mma_commit_pair(own_empty0 + (uint32_t)(s * sizeof(uint64_t)));
        mma_commit_pair(peer_empty0 + (uint32_t)(s * sizeof(uint64_t)));
      }
      mma_commit_pair(map_to_rank(accum_full, 0));
      mma_commit_pair(map_to_rank(accum_full, 1));
    }
  } else {
    // ---- weight decoders (warps 2..9 of each CTA), then the epilogue ---------
    const int quarter = warp & 3;
    const int half = ((warp - 2) >> 2) & 1;
    const int set = (warp - 2) / kDecoderWarps;  // K blocks kb % 2 == set
    const int row = quarter * 32 + lane;
    const int n = n0 + row;
    const uint32_t lane4 = (uint32_t)lane << 2;
    const uint32_t a_lane = (uint32_t)(quarter * 32) << 16;
    const int sw = (row >> 1) & 3;
    const int off0 = row * kTcBK + ((2 * half) ^ sw) * 16;
    const int off1 = row * kTcBK + ((2 * half + 1) ^ sw) * 16;
    const uint32_t leader_full_a0 = map_to_rank(&full_a[0], 0);
    static_assert(kTc2Stages % kTc2DecSets == 0, "each ring slot belongs to one decoding set");
    for (int kb = set; kb < nkb; kb += kTc2DecSets) {
      const int s = kb % kTc2Stages;
      const uint32_t parity = (kb / kTc2Stages) & 1;
      // this CTA's weight tile has landed; the MMAs that read A stage s one
      // ring ago have completed
      if (!mbar_wait(&w_full[s], parity, abort)) atomicAdd(p.err, 1);
      if (kb >= kTc2Stages && !mbar_wait(&empty[s], parity ^ 1, abort)) atomicAdd(p.err, 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint8_t *ws = w_stages + s * kWBytes;
      const uint4 x0 = *reinterpret_cast<const uint4 *>(ws + off0);
      const uint4 x1 = *reinterpret_cast<const uint4 *>(ws + off1);
      const uint32_t words[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      uint32_t v[16];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[q * 2] = lut_pair(lut, words[q], lane4, false);
        v[q * 2 + 1] = lut_pair(lut, words[q], lane4, true);
      }
      tmem_st16(a_tmem0 + s * 32 + half * 16 + a_lane, v);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(leader_full_a0 + (uint32_t)(s * sizeof(uint64_t)));
    }

    if (set == 0) {
    // epilogue (set 0): as in the single-CTA kernel, over this CTA's 128 rows
    // x the pair's 256 tokens, staged in the (idle) activation and weight rings
    const bool n_ok = n < p.n;
    const float cs = n_ok ? p.cs[n] : 0.f;
    float bias = 0.f;
    if (n_ok && p.bias) {
      const uint16_t h = static_cast<const uint16_t *>(p.bias)[n];
      bias = p.bias_dtype == HIF8_DTYPE_BF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
    }
    constexpr int kChunks = kTc2BN / 64;
    const int c0 = half * (kTc2BN / 2);
    float tsr[kChunks];
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int m = m0 + c0 + c * 32 + lane;
      tsr[c] = m < p.m ? p.ts[(int64_t)m * p.ts_stride] : 0.f;
    }
    if (!mbar_wait(accum_full, 0, abort)) atomicAdd(p.err, 1);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    static_assert(kTc2Stages * (kBBytes + kWBytes) >= kTc2BN * kTcBM * 4, "the FP32 output tile fits the rings");
    uint16_t *stage_out = reinterpret_cast<uint16_t *>(b_stages);
    float *stage_out32 = reinterpret_cast<float *>(b_stages);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      uint32_t acc[32];
      tmem_ld32(d_tmem + (uint32_t)(c0 + c * 32) + a_lane, acc);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const float ts = __shfl_sync(0xFFFFFFFFu, tsr[c], q);
        float val = __uint_as_float(acc[q]) * cs;
        val = val * ts;
        val += bias;
        if constexpr (OUT == HIF8_DTYPE_F32) stage_out32[(c0 + c * 32 + q) * kTcBM + row] = val;
        else stage_out[(c0 + c * 32 + q) * kTcBM + row] = (uint16_t)to_out_bits<OUT>(val);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("bar.sync 1, %0;" ::"n"(kDecoderWarps * 32) : "memory");
    if (warp == 2 && lane == 0 && n0 < p.n) {  // a pair's second row block may lie past N
      if (gridDim.z > 1)
        asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                     ::"l"(&ymap), "r"(n0), "r"(m0), "r"((int)blockIdx.z), "r"(smem_addr(stage_out))
                     : "memory");
      else
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                     ::"l"(&ymap), "r"(n0), "r"(m0), "r"(smem_addr(stage_out))
                     : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_barrier();  // neither CTA leaves while the pair's MMAs or arrivals may touch it
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Decode HiF8 activation bytes to unscaled BF16 (exact) for the TMA B operand.
__global__ void __launch_bounds__(256) decode_to_bf16(const uint8_t *__restrict__ a, uint16_t *__restrict__ out,
                                                      int64_t chunks) {
  __shared__ uint32_t tbl[256];  // decoded value as FP32 bits (BF16 payload in the high half)
  tbl[threadIdx.x] = g_decode_f32.v[threadIdx.x];
  __syncthreads();
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks; c += (int64_t)gridDim.x * blockDim.x) {
    const uint4 v = *reinterpret_cast<const uint4 *>(a + c * 16);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t r[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      r[2 * j] = __byte_perm(tbl[w[j] & 0xFF], tbl[(w[j] >> 8) & 0xFF], 0x7632u);
      r[2 * j + 1] = __byte_perm(tbl[(w[j] >> 16) & 0xFF], tbl[w[j] >> 24], 0x7632u);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out + c * 16);
    dst[0] = make_uint4(r[0], r[1], r[2], r[3]);
    dst[1] = make_uint4(r[4], r[5], r[6], r[7]);
  }
}

// Static quantisation of FP16/BF16 activations with the fixed scale *scale
// fused with the decode: the unscaled BF16 value of each element's static
// code, written straight into the GEMM's BF16 operand (bit-identical to
// hif8_static_quant followed by decode_to_bf16, without the byte round
// trip).  The fake-quant table gives each correctly rounded quotient's value
// (fake_quant16); a chunk with a huge or non-finite product, or a scale that
// needs it, takes the exact FP64 path.
template <int kDtype>
__global__ void __launch_bounds__(256) fake_quant_to_bf16(const uint16_t *__restrict__ x,
                                                          const float *__restrict__ scale,
                                                          uint16_t *__restrict__ out, int64_t chunks) {
  __shared__ __align__(16) uint16_t fq[4096];
  __shared__ __align__(16) uint8_t mag[4096];
  __shared__ uint32_t dec[256];
  for (int i = threadIdx.x; i < 4096 / 8; i += blockDim.x)
    reinterpret_cast<uint4 *>(fq)[i] = reinterpret_cast<const uint4 *>(g_fake_quant_bf16.v)[i];
  load_encode_mag_table(mag);
  dec[threadIdx.x] = g_decode_f32.v[threadIdx.x];
  __syncthreads();
  const float s = __ldg(scale);
  const float r = __frcp_rn(s);
  const double r64 = __drcp_rn((double)s);
  const uint32_t re = __float_as_uint(r) & 0x7F800000u;
  const bool exact_only = (re == 0u) | (re == 0x7F800000u) | !(s > 0.f) | !scale_edge_ok(s);
  const float s_half = 0.5f * s;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks; c += (int64_t)gridDim.x * blockDim.x) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4 *>(x) + 2 * c);
    const uint4 b = __ldcs(reinterpret_cast<const uint4 *>(x) + 2 * c + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t o[8];
    if (exact_only || !fake_quant16<kDtype>(w, s, r, s_half, fq, o)) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = (dec[static_code_exact(half_bits_to_f32<kDtype>(w[j] & 0xFFFFu), r64, mag)] >> 16) |
               (dec[static_code_exact(half_bits_to_f32<kDtype>(w[j] >> 16), r64, mag)] & 0xFFFF0000u);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(out) + 2 * c;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// Split-K epilogue: out[m, n] = sum over the splits in order of the FP32
// partials (each (acc * cs[n]) * ts[m] of its K range) + bias[n], rounded
// once to the output type.  Four outputs per thread.
template <int OUT>
__global__ void __launch_bounds__(256) splitk_reduce(const float *__restrict__ part, int splits, int64_t mn,
                                                     int n, const void *__restrict__ bias, int bias_dtype,
                                                     void *__restrict__ out) {
  for (int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) * 4; i < mn;
       i += (int64_t)gridDim.x * blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4 *>(part + i);
    for (int z = 1; z < splits; ++z) {
      const float4 w = *reinterpret_cast<const float4 *>(part + (int64_t)z * mn + i);
      v.x += w.x, v.y += w.y, v.z += w.z, v.w += w.w;
    }
    float r[4] = {v.x, v.y, v.z, v.w};
    if (bias) {
      const int c = (int)(i % n);  // n % 8 == 0: the four outputs share a row
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint16_t h = static_cast<const uint16_t *>(bias)[c + q];
        r[q] += bias_dtype == HIF8_DTYPE_BF16 ? bf16_bits_to_f32(h) : f16_bits_to_f32(h);
      }
    }
    if constexpr (OUT == HIF8_DTYPE_F32) {
      *reinterpret_cast<float4 *>(static_cast<float *>(out) + i) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
      const uint32_t lo = to_out_bits<OUT>(r[0]) | (to_out_bits<OUT>(r[1]) << 16);
      const uint32_t hi = to_out_bits<OUT>(r[2]) | (to_out_bits<OUT>(r[3]) << 16);
      *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(out) + i) = make_uint2(lo, hi);
    }
  }
}

// ------------------------------------------------------------------ host --

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

constexpr int64_t kTcMinM = 32;

bool hif8_gemm_tc_supported(int64_t m, int64_t n, int64_t k) {
  // n % 8: the output rows must be 16-byte strided for the TMA store
  return m >= kTcMinM && n >= 64 && n % 8 == 0 && k % kTcBK == 0 && k >= kTcBK && m < (1LL << 31) &&
         n <= 65535LL * kTcBM;
}

static size_t err_offset(int64_t m, int64_t k) { return ((size_t)m * k * 2 + 255) & ~size_t(255); }

// Tile width BN (tokens per CTA) and split-K count of a call, by the estimated
// time: waves of tiles over the SMs x the cost of a tile, whose weight decode
// dominates and grows with the tile's K blocks (measured on B200: 0.53-0.57
// us per 64-wide K block at BN 256, a little less at BN 128 / 64, about 3 us
// of set-up per tile), plus for split-K the FP32 partial round trip and the
// reduce launch.  Splitting K pays where the token x channel tiles alone
// leave SMs idle (configs[2] down, M = 512: 64 tiles for 148 SMs).
struct TcPlan {
  int bn, splits, kb_per;
  bool pair;  // the CTA-pair kernel (256 weight rows x 256 tokens per pair)
};

template <int OUT>
static const void *tc_pair_kernel_ptr() {
  return reinterpret_cast<const void *>(gemm_hif8_tc_pair_kernel<OUT>);
}

static constexpr size_t tc_pair_smem_bytes() {
  return 1024 + (size_t)kTc2Stages * (kTc2Half * 128 + kTcBM * kTcBK) + kTcLut + (4 * kTc2Stages + 1) * 8 + 16;
}

// Resident CTA pairs of the pair kernel on this device (cached per device).
static int tc_pair_slots() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    const void *k = tc_pair_kernel_ptr<HIF8_DTYPE_BF16>();
    v = -1;
    if (ensure_smem_limit(k, tc_pair_smem_bytes()) == HIF8_OK) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, 1, 1);
      cfg.blockDim = dim3(kTc2Threads, 1, 1);
      cfg.dynamicSmemBytes = tc_pair_smem_bytes();
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) == cudaSuccess && clusters > 0) v = clusters;
    }
    cudaGetLastError();
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v > 0 ? v : 0;
}

// The CTA-pair kernel runs only when HIF8_GEMM_PAIR=1 (measured slower than
// the single-CTA kernel on the configs[2] shapes); with it set, every call
// of at least 256 tokens takes the pair kernel.
static bool tc_pair_requested() {
  const char *v = std::getenv("HIF8_GEMM_PAIR");
  return v != nullptr && v[0] == '1';
}

static TcPlan tc_plan(int64_t m, int64_t n, int64_t k) {
  const int sms = num_sms();
  const int64_t nkb = k / kTcBK;
  const int bns[3] = {256, 128, 64};
  const double per_kb[3] = {0.55, 0.49, 0.46};
  TcPlan best{64, 1, (int)nkb, false};
  double best_t = -1.0;
  const int pair_slots = m >= kTc2BN && tc_pair_requested() ? tc_pair_slots() : 0;
  for (int i = 0; i < 4; ++i) {
    const bool pair = i == 3;  // candidate 3: the CTA pair, only where requested
    if (pair != (pair_slots > 0)) continue;
    const int bn = pair ? kTc2BN : bns[i];
    if (!pair && bn > 64 && m < bn / 2) continue;
    const int rows = pair ? kTc2Rows : kTcBM;
    const int slots = pair ? pair_slots : sms;
    const int stages = pair ? kTc2Stages : kTcStages;
    const double kb_cost = pair ? 0.55 : per_kb[i];
    const int64_t tiles = ((m + bn - 1) / bn) * ((n + rows - 1) / rows);
    for (int splits = 1; splits <= 4; ++splits) {
      const int64_t kb_per = (nkb + splits - 1) / splits;
      if (splits > 1 && (kb_per < 2 * stages || (splits - 1) * kb_per >= nkb)) break;
      const int64_t waves = (tiles * splits + slots - 1) / slots;
      double t = (double)waves * (3.0 + kb_cost * (double)kb_per);
      // FP32 partials written by the GEMM and read back by the reduce (~5 TB/s
      // achieved), one more launch (measured: configs[2] down, M = 4096, two
      // splits 446 us against 430 unsplit; M = 512 108 -> 76 us)
      if (splits > 1) t += (double)(2 * splits + 1) * (double)m * (double)n * 4.0 / 5.0e6 + 5.0;
      if (best_t < 0 || t < best_t) {
        best_t = t;
        best = TcPlan{bn, splits, (int)kb_per, pair};
      }
    }
  }
  return best;
}

static size_t part_offset(int64_t m, int64_t k) { return err_offset(m, k) + 256; }

size_t hif8_gemm_tc_workspace(int64_t m, int64_t n, int64_t k) {
  // BF16 activation copy + error word (+ FP32 split-K partials)
  const TcPlan plan = tc_plan(m, n, k);
  const size_t part = plan.splits > 1 ? (size_t)plan.splits * m * n * sizeof(float) : 0;
  return part_offset(m, k) + (part + 255) / 256 * 256;
}

template <int BN>
static constexpr size_t tc_smem_bytes() {
  return 1024 + (size_t)kTcStages * (BN * 128 + kTcBM * kTcBK) + kTcLut + (3 * kTcStages + 1) * 8 + 16;
}

template <int OUT>
static int launch_tc_pair(const CUtensorMap &xmap, const CUtensorMap &wmap, const CUtensorMap &ymap,
                          const TcParams &p, cudaStream_t stream, int splits) {
  const void *kernel = tc_pair_kernel_ptr<OUT>();
  const size_t smem = tc_pair_smem_bytes();
  const int st = ensure_smem_limit(kernel, smem);
  if (st != HIF8_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * ((p.m + kTc2BN - 1) / kTc2BN)), (unsigned)((p.n + kTc2Rows - 1) / kTc2Rows),
                     (unsigned)splits);
  cfg.blockDim = dim3(kTc2Threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, gemm_hif8_tc_pair_kernel<OUT>, xmap, wmap, ymap, p);
  if (err != cudaSuccess) {
    set_last_error(err);
    return HIF8_ERR_CUDA;
  }
  return check_launch();
}

template <int BN, int OUT>
static int launch_tc(const CUtensorMap &xmap, const CUtensorMap &wmap, const CUtensorMap &ymap, const TcParams &p,
                     cudaStream_t stream, int splits) {
  auto kernel = gemm_hif8_tc_kernel<BN, OUT>;
  const size_t smem = tc_smem_bytes<BN>();
  const int st = ensure_smem_limit(reinterpret_cast<const void *>(kernel), smem);
  if (st != HIF8_OK) return st;
  dim3 grid((unsigned)((p.m + BN - 1) / BN), (unsigned)((p.n + kTcBM - 1) / kTcBM), (unsigned)splits);
  kernel<<<grid, kTcThreads, smem, stream>>>(xmap, wmap, ymap, p);
  return check_launch();
}

int hif8_gemm_tc(const GemvArgs &args, int output_dtype, void *workspace, size_t workspace_bytes,
                 cudaStream_t stream, int a_dtype) {
  const int64_t m = args.m, n = args.n, k = args.k;
  if (workspace_bytes < hif8_gemm_tc_workspace(m, n, k)) return HIF8_ERR_WORKSPACE;
  auto encode = tensor_map_encoder();
  if (!encode) return HIF8_ERR_CUDA;
  uint16_t *xb = static_cast<uint16_t *>(workspace);
  int *err = reinterpret_cast<int *>(static_cast<uint8_t *>(workspace) + err_offset(m, k));
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), stream);
  if (e != cudaSuccess) {
    set_last_error(e);
    return HIF8_ERR_CUDA;
  }
  // 1. activation -> BF16 (exact), 16 elements per thread (k % 64 == 0):
  // the decode of HiF8 bytes, or the static quant + decode of FP16/BF16
  // input with the fixed scale args.ts[0]
  const int64_t chunks = m * k / 16;
  int64_t blocks = (chunks + 255) / 256;
  if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
  if (a_dtype == HIF8_DTYPE_BF16)
    fake_quant_to_bf16<HIF8_DTYPE_BF16><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const uint16_t *>(args.a), args.ts, xb, chunks);
  else if (a_dtype == HIF8_DTYPE_F16)
    fake_quant_to_bf16<HIF8_DTYPE_F16><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const uint16_t *>(args.a), args.ts, xb, chunks);
  else
    decode_to_bf16<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const uint8_t *>(args.a), xb, chunks);
  int status = check_launch();
  if (status != HIF8_OK) return status;

  // 2. the tcgen05 GEMM, BN (tokens per tile) and split-K by tc_plan
  const TcPlan plan = tc_plan(m, n, k);
  const int bn = plan.bn, splits = plan.splits;
  const cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap xmap, wmap, ymap;
  {  // BF16 activation [M, K]: (tokens per CTA) x 64 boxes, 128-byte swizzle (UMMA SW128 K-major)
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)(plan.pair ? kTc2Half : bn)};
    if (encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xb, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return HIF8_ERR_CUDA;
  }
  {  // HiF8 weight [N, K] bytes: 128 x 64 boxes, 64-byte swizzle (conflict-free row reads)
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)k};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)kTcBM};
    if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(args.w), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return HIF8_ERR_CUDA;
  }
  float *part = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + part_offset(m, k));
  const bool f32 = output_dtype == HIF8_DTYPE_F32 || splits > 1;
  if (splits > 1) {  // FP32 partials [splits][M][N]: 128-channel x BN-token x 1 boxes
    const cuuint64_t dims[3] = {(cuuint64_t)n, (cuuint64_t)m, (cuuint64_t)splits};
    const cuuint64_t strides[2] = {(cuuint64_t)n * 4, (cuuint64_t)m * n * 4};
    const cuuint32_t box[3] = {(cuuint32_t)kTcBM, (cuuint32_t)bn, 1};
    if (encode(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, part, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return HIF8_ERR_CUDA;
  } else {  // output [M, N] (BF16 / FP16 bits, or FP32 partials): 128-channel x BN-token boxes for the TMA store
    const cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)n * (f32 ? 4 : 2)};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBM, (cuuint32_t)bn};
    if (encode(&ymap, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, args.out, dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return HIF8_ERR_CUDA;
  }
  // split-K partials carry no bias: the reduce adds it once
  TcParams p{args.w, args.ts, args.cs, splits > 1 ? nullptr : args.bias, splits > 1 ? (void *)part : args.out, err,
             args.m, args.n, args.k, args.bias_dtype, args.ts_stride, plan.kb_per};
  const bool bf16 = output_dtype == HIF8_DTYPE_BF16;
  if (plan.pair) {
    if (f32) status = launch_tc_pair<HIF8_DTYPE_F32>(xmap, wmap, ymap, p, stream, splits);
    else if (bf16) status = launch_tc_pair<HIF8_DTYPE_BF16>(xmap, wmap, ymap, p, stream, splits);
    else status = launch_tc_pair<HIF8_DTYPE_F16>(xmap, wmap, ymap, p, stream, splits);
  } else if (f32) {
    if (bn == 256) status = launch_tc<256, HIF8_DTYPE_F32>(xmap, wmap, ymap, p, stream, splits);
    else if (bn == 128) status = launch_tc<128, HIF8_DTYPE_F32>(xmap, wmap, ymap, p, stream, splits);
    else status = launch_tc<64, HIF8_DTYPE_F32>(xmap, wmap, ymap, p, stream, splits);
  } else if (bn == 256) {
    status = bf16 ? launch_tc<256, HIF8_DTYPE_BF16>(xmap, wmap, ymap, p, stream, 1)
                  : launch_tc<256, HIF8_DTYPE_F16>(xmap, wmap, ymap, p, stream, 1);
  } else if (bn == 128) {
    status = bf16 ? launch_tc<128, HIF8_DTYPE_BF16>(xmap, wmap, ymap, p, stream, 1)
                  : launch_tc<128, HIF8_DTYPE_F16>(xmap, wmap, ymap, p, stream, 1);
  } else {
    status = bf16 ? launch_tc<64, HIF8_DTYPE_BF16>(xmap, wmap, ymap, p, stream, 1)
                  : launch_tc<64, HIF8_DTYPE_F16>(xmap, wmap, ymap, p, stream, 1);
  }
  if (status != HIF8_OK || splits == 1) return status;
  // 3. split-K: sum the partials in split order, add the bias, round once
  const int64_t mn = m * n;
  int64_t rblocks = (mn / 4 + 255) / 256;
  if (rblocks > (int64_t)num_sms() * 8) rblocks = (int64_t)num_sms() * 8;
  if (output_dtype == HIF8_DTYPE_F32)
    splitk_reduce<HIF8_DTYPE_F32><<<(unsigned)rblocks, 256, 0, stream>>>(part, splits, mn, (int)n, args.bias,
                                                                          args.bias_dtype, args.out);
  else if (bf16)
    splitk_reduce<HIF8_DTYPE_BF16><<<(unsigned)rblocks, 256, 0, stream>>>(part, splits, mn, (int)n, args.bias,
                                                                           args.bias_dtype, args.out);
  else
    splitk_reduce<HIF8_DTYPE_F16><<<(unsigned)rblocks, 256, 0, stream>>>(part, splits, mn, (int)n, args.bias,
                                                                          args.bias_dtype, args.out);
  return check_launch();
}

}  // namespace hif8
