// bf16 tcgen05 GEMM whose weight operand is dequantized in shared memory.
//
// Replaces the dequantize-then-matmul of quantized_ops::linear_mx /
// matmul_mx (src/voyager_compiler/ops/quantized.py:455-472, 522-648) for
// every weight format that is not MXFP8 x MXFP8: posit / int / NormalFloat /
// E2M1 / any codebook, with or without a block scale.  The reference reads
// each weight back as
//
//   w[n, k] = bf16( decode(code[n, k]) * scale[n, k / bs] )
//
// (decode: the codebook entry, or the code's own value) and multiplies in
// bf16 with float32 accumulation.  Here the codes stay packed in HBM as
// indices into a palette of at most 16 (4-bit, "LUT4") or 256 (8-bit,
// "LUT8") bf16 values; producer warps turn one 64-element K step of them
// into bf16 in registers -- palette lookup, the bf16 product with the block
// scale (mul.rn.bf16x2: the exact product rounded once, as the reference's
// bf16 multiply) -- and store it straight into the tensor cores' K-major
// SWIZZLE_128B operand layout.  The activations (bf16, already read back by
// the dequantize kernels when they are codes) come in by TMA.  A third mode
// takes a plain bf16 weight by TMA as well: the library's own bf16 GEMM.
//
//   out[b][m, n] = sum_k A[b][m, k] * W[b][n, k] (+ bias[n]),  float32 sums,
//   one bf16 rounding.
//
// Weight layout ("step-major", vq_dq_pack): for each 64-element K step the
// indices of all rows are contiguous, [wb][K/64][Npad / 128][128-row block]
// (Npad = N rounded up to 256), a block holding its rows' 32 | 64 bytes
// chunk-major -- 16-byte chunk c of row r at c * 2048 + r * 16, so the 32
// rows of a warp read consecutive 16-byte pieces -- and the scales likewise,
// [wb][K/64][Npad][4] bf16: the scale of each 16-element quarter of the step
// (any block size >= 16 maps onto quarters at pack time).  One CTA's 128
// rows of a step are then one contiguous bulk copy.
//
// Kernel: CTA pairs (cluster of 2, tcgen05.mma.cta_group::2.kind::f16, bf16
// inputs, float32 accumulator), 256 x 256 output tiles, persistent over the
// tiles.  Per CTA:
//   warp 0      per 64-element K step, once the stage is free, this CTA's
//               128 rows of A by TMA (and, TMA mode, its 128-row half of the
//               bf16 weight), counted on the even CTA's "full" barrier;
//   warp 1      (even CTA) TMEM owner and MMA issuer: 4 x M256 N256 K16 per
//               step into one of two accumulators (512 TMEM columns), so the
//               epilogue of a tile overlaps the next tile's MMAs;
//   LUT modes:
//   warp 2      the packed indices and scales of this CTA's 128 weight rows,
//               step by step, by bulk copy into "raw" slots (RSG per decoder
//               group, used by that group's steps in turn; a slot is
//               refilled once its decoders have read it), so the weight bytes
//               are on chip long before their stage frees up.  Each group
//               waits on its own slots in order, so no wait can mistake a
//               phase two ahead for the one before (mbarrier parity);
//   warps 3-18  weight decoders, four groups of 4 taking every fourth step:
//               each thread reads the step's indices and scales of one weight
//               row, hands the slot back, and once the stage is free writes
//               the row's 64 bf16 values into the stage's weight tile; the
//               warp then arrives on the even CTA's "full" barrier after a
//               proxy fence;
//   last 4 warps epilogue: one TMEM lane quarter each, 32 columns at a time,
//               + bias, bf16, row stores; the accumulator is handed back as
//               soon as its loads land.
// Every wait is bounded by %globaltimer and records an error code instead
// of trapping; each thread that issued asynchronous work waits for it
// before the TMEM is freed.  No TMA multicast.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "vq_numerics.cuh"
#include "vq_tc.cuh"

namespace vq {
namespace dq {

using namespace vq::tc;

constexpr int KSTEP = 64;                  // K elements per pipeline stage
constexpr int A_BYTES = 128 * 128;         // this CTA's 128 rows x 128 bytes
constexpr int B_BYTES = 128 * 128;         // this CTA's half of the weight tile
constexpr int TMEM_COLS = 512;             // two 256-column accumulators
constexpr int DQ_GROUPS = 4, DQ_WARPS = 4, EPI_WARPS = 4;  // DQ_WARPS per group
constexpr int DEC_WARP0 = 3;               // the first decoder warp (LUT modes)
constexpr int PAL8_BYTES = 256 * 32 * 4;   // LUT8 palette, one copy per bank
constexpr int SCALE_BYTES = 128 * 8;       // a step's scales of 128 rows
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int BAR_BYTES = 512;

enum { MODE_TMA = 0, MODE_LUT4 = 1, MODE_LUT8 = 2 };
enum { ERR_FULL = 11, ERR_EMPTY = 12, ERR_ACC = 13, ERR_DRAIN = 14 };

template <int MODE>
struct Cfg {
  static constexpr bool LUT = MODE != MODE_TMA;
  static constexpr int STEP_BYTES = MODE == MODE_LUT4 ? 32 : 64;  // indices per row and step
  static constexpr int RAW_BYTES = LUT ? 128 * STEP_BYTES + SCALE_BYTES : 0;  // one raw slot
  static constexpr int STAGES = MODE == MODE_LUT4 ? 5 : (MODE == MODE_LUT8 ? 4 : 6);
  static constexpr int RSG = MODE == MODE_LUT4 ? 3 : (MODE == MODE_LUT8 ? 1 : 0);  // per group
  static constexpr int RSLOTS = RSG * DQ_GROUPS;
  static constexpr int RAW0 = STAGES * STAGE_BYTES;           // the raw ring
  static constexpr int PAL0 = RAW0 + RSLOTS * RAW_BYTES;      // LUT8 palette
  static constexpr int BARS = PAL0 + (MODE == MODE_LUT8 ? PAL8_BYTES : 0);
  static constexpr int SMEM = BARS + BAR_BYTES;
  static constexpr int EPI_WARP0 = LUT ? DEC_WARP0 + DQ_GROUPS * DQ_WARPS : 2;
  static constexpr int THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
};
static_assert(Cfg<MODE_TMA>::SMEM + 1024 <= 227 * 1024, "TMA-mode shared memory");
static_assert(Cfg<MODE_LUT4>::SMEM + 1024 <= 227 * 1024, "LUT4 shared memory");
static_assert(Cfg<MODE_LUT8>::SMEM + 1024 <= 227 * 1024, "LUT8 shared memory");
static_assert(STAGE_BYTES % 1024 == 0 && Cfg<MODE_LUT4>::RAW_BYTES % 16 == 0 &&
                  Cfg<MODE_LUT8>::RAW_BYTES % 16 == 0,
              "stages 1024-byte aligned, raw slots 16-byte aligned");
static_assert((2 * Cfg<MODE_LUT4>::STAGES + 2 * Cfg<MODE_LUT4>::RSLOTS + 6) * 8 <= BAR_BYTES &&
                  (2 * Cfg<MODE_LUT8>::STAGES + 2 * Cfg<MODE_LUT8>::RSLOTS + 6) * 8 <= BAR_BYTES &&
                  (2 * Cfg<MODE_TMA>::STAGES + 6) * 8 <= BAR_BYTES,
              "barrier area");
// A decoder group waits on the "empty" barrier of every DQ_GROUPS-th step;
// with at least DQ_GROUPS stages the phase it waits for is never two ahead.
static_assert(Cfg<MODE_LUT4>::STAGES >= DQ_GROUPS && Cfg<MODE_LUT8>::STAGES >= DQ_GROUPS,
              "decoder empty waits need STAGES >= DQ_GROUPS");

// Raw slot and phase parity of step st: the group's j-th step uses its slot
// j % RSG.
template <int MODE>
__device__ __forceinline__ void raw_slot(int st, int& slot, uint32_t& parity) {
  constexpr int RSG = Cfg<MODE>::RSG;
  const int grp = st % DQ_GROUPS, j = st / DQ_GROUPS;
  slot = grp * RSG + j % RSG;
  parity = (uint32_t)(j / RSG) & 1u;
}

struct DqArgs {
  const uint8_t* wq;      // packed indices [wb][KS][Npad][STEP_BYTES]
  const uint16_t* ws4;    // bf16 quarter-step scales [wb][KS][Npad][4], or null
  const uint16_t* pal;    // bf16 palette [16] (LUT4) or [256] (LUT8)
  const uint16_t* bias;   // bf16 [N] or null
  uint16_t* out;          // bf16 [batch][M, ldo]
  int64_t ldo, out_bs;
  int M, N, K, KS, Npad;  // KS = ceil(K / 64), Npad = N rounded up to 256
  int MT2, NTN, ntiles;   // 256-row tiles per batch, 256-column tiles, all tiles
  int w_shared;           // one weight for every batch
  int* err;
  // split-K (one batch): unit u is K slice u % S of tile u / S, KSU steps
  // from step (u % S) * KSU; with S > 1 the epilogue stores float32 partial
  // sums into part [S][M][N] and k_dq_finalize adds them up
  int S, KSU, nunits;
  float* part;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(s));
  return r;
}
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t s) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(s));
  return r;
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void arrive_release_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool try_wait_acq_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (the barrier's arrivals release
// shared-memory writes of both CTAs).
__device__ __forceinline__ bool wait_cluster(uint32_t bar, uint32_t parity, int* err, int code) {
  if (try_wait_acq_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (try_wait_acq_cluster(bar, parity)) return true;
    if (globaltimer_ns() - t0 > WAIT_NS) break;
  }
  note_err(err, code);
  return false;
}

__device__ __forceinline__ uint32_t idesc_bf16(uint32_t M, uint32_t N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc,
                                              uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void tile_of(const DqArgs& g, int t, int& b, int& tm, int& tn) {
  const int per_b = g.MT2 * g.NTN;
  b = t / per_b;
  const int r = t - b * per_b;
  tm = r / g.NTN;
  tn = r - tm * g.NTN;
}
// Work unit u: its tile and its first K step (adjacent units are the K
// slices of one tile).
__device__ __forceinline__ void unit_of(const DqArgs& g, int u, int& b, int& tm, int& tn, int& k0) {
  const int t = u / g.S;
  k0 = (u - t * g.S) * g.KSU;
  tile_of(g, t, b, tm, tn);
}
// A walk over a pair's K steps in order: step st is K step k0 + (st - ti
// KSU) of unit pair_id + ti npairs, ti = st / KSU.  It keeps ti, the offset
// sr within the unit and the unit's tile, and moves on by a fixed stride
// with no division (KSU, S and the tile counts are runtime values); the
// tile is worked out again only when the walk enters another unit.
struct StepWalk {
  int ti, sr, b, tm, tn, k0;
  __device__ __forceinline__ StepWalk(const DqArgs& g, int pair_id, int npairs, int st) {
    ti = st / g.KSU;
    sr = st - ti * g.KSU;
    unit_of(g, pair_id + ti * npairs, b, tm, tn, k0);
  }
  __device__ __forceinline__ int ks() const { return k0 + sr; }
  __device__ __forceinline__ void advance(const DqArgs& g, int pair_id, int npairs, int stride) {
    sr += stride;
    if (sr >= g.KSU) {
      do {
        sr -= g.KSU;
        ++ti;
      } while (sr >= g.KSU);
      unit_of(g, pair_id + ti * npairs, b, tm, tn, k0);
    }
  }
};

// ---- the weight decode shared by the GEMM producers and vq_dq_decode ------
// A 16-entry palette as byte planes for prmt lookups: lo[i] holds the low
// bytes of entries 4i..4i+3, hi[i] the high bytes.
struct Pal4 {
  uint32_t lo[4], hi[4];
};
__device__ __forceinline__ Pal4 load_pal4(const uint16_t* pal) {
  const uint4 a = *reinterpret_cast<const uint4*>(pal);
  const uint4 b = *reinterpret_cast<const uint4*>(pal + 8);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  Pal4 p;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    p.lo[i] = prmt(w[2 * i], w[2 * i + 1], 0x6420);
    p.hi[i] = prmt(w[2 * i], w[2 * i + 1], 0x7531);
  }
  return p;
}
// Four 4-bit indices (the low 16 bits of x, element j in nibble j) -> two
// bf16x2 words (elements 0,1 and 2,3).
__device__ __forceinline__ void lut4_quad(const Pal4& p, uint32_t x, uint32_t& e01, uint32_t& e23) {
  const uint32_t s = x & 0x7777u;                      // entry within its group of 8
  const uint32_t s2 = 0x3210u | ((x >> 1) & 0x4444u);  // bit 3: the second group
  const uint32_t lo = prmt(prmt(p.lo[0], p.lo[1], s), prmt(p.lo[2], p.lo[3], s), s2);
  const uint32_t hi = prmt(prmt(p.hi[0], p.hi[1], s), prmt(p.hi[2], p.hi[3], s), s2);
  e01 = prmt(lo, hi, 0x5140);
  e23 = prmt(lo, hi, 0x7362);
}

// 32 consecutive elements of one row (k0 .. k0 + 31 of K) from their packed
// indices, times their block scales: 16 bf16x2 words.  raw: LUT4 words 0-3
// (8 nibbles each), LUT8 words 0-7 (4 bytes each).  pal32 (LUT8): the
// palette in shared memory, entry e of lane l at word e * 32 + l.
template <int MODE>
__device__ __forceinline__ void decode32(const uint32_t (&raw)[8], const Pal4& p4,
                                         const uint32_t* pal32, int lane, uint32_t s_lo,
                                         uint32_t s_hi, bool scaled, int valid,
                                         uint32_t (&o)[16]) {
  if (MODE == MODE_LUT4) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      lut4_quad(p4, raw[w], o[4 * w], o[4 * w + 1]);
      lut4_quad(p4, raw[w] >> 16, o[4 * w + 2], o[4 * w + 3]);
    }
  } else {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t x = raw[w];
      const uint32_t v0 = pal32[((x & 0xFFu) << 5) + lane];
      const uint32_t v1 = pal32[(((x >> 8) & 0xFFu) << 5) + lane];
      const uint32_t v2 = pal32[(((x >> 16) & 0xFFu) << 5) + lane];
      const uint32_t v3 = pal32[((x >> 24) << 5) + lane];
      o[2 * w] = prmt(v0, v1, 0x5410);
      o[2 * w + 1] = prmt(v2, v3, 0x5410);
    }
  }
  if (scaled) {
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = bmul2(o[i], s_lo);
#pragma unroll
    for (int i = 8; i < 16; ++i) o[i] = bmul2(o[i], s_hi);
  }
  if (valid < 32) {  // the K tail: zeros past the last column
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (2 * i >= valid) o[i] = 0;
      else if (2 * i + 1 >= valid) o[i] &= 0xFFFFu;
    }
  }
}

// Index of packed row n of weight batch wb, step ks (rows of 8 scale bytes;
// the indices of a 128-row block start at the block's first row times
// STEP_BYTES).
__device__ __forceinline__ int64_t wrow(const DqArgs& g, int wb, int ks, int n) {
  return ((int64_t)wb * g.KS + ks) * g.Npad + n;
}

// One thread's 32 elements (half h of a step of row r of a 128-row block):
// raw index words and the scales of its two 16-element quarters.  blk: the
// block's indices (chunk-major: chunk c of row r at c * 2048 + r * 16);
// scales_row: the row's 4 quarter scales, or null.
template <int MODE>
__device__ __forceinline__ void read32(const uint8_t* blk, int r, const uint16_t* scales_row, int h,
                                       uint32_t (&raw)[8], uint32_t& s_lo, uint32_t& s_hi) {
  const int c0 = MODE == MODE_LUT8 ? 2 * h : h;  // this half's first chunk
  const uint4 a = *reinterpret_cast<const uint4*>(blk + c0 * 2048 + r * 16);
  raw[0] = a.x, raw[1] = a.y, raw[2] = a.z, raw[3] = a.w;
  if (MODE == MODE_LUT8) {
    const uint4 b = *reinterpret_cast<const uint4*>(blk + (c0 + 1) * 2048 + r * 16);
    raw[4] = b.x, raw[5] = b.y, raw[6] = b.z, raw[7] = b.w;
  } else {
    raw[4] = raw[5] = raw[6] = raw[7] = 0;
  }
  s_lo = s_hi = 0;
  if (scales_row) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(scales_row + 2 * h);
    s_lo = (v & 0xFFFFu) | (v << 16);
    s_hi = (v >> 16) | (v & 0xFFFF0000u);
  }
}

// ---------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(Cfg<MODE>::THREADS, 1)
    k_gemm_dq(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_w,
              const __grid_constant__ DqArgs g) {
  using C = Cfg<MODE>;
  constexpr int S = C::STAGES, RS = C::RSLOTS, SB = C::STEP_BYTES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint32_t* pal32 = reinterpret_cast<uint32_t*>(smem + C::PAL0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BARS);
  // full[S], empty[S], acc_full[2], acc_empty[2], drain, TMEM slot,
  // raw_full[RS], raw_empty[RS]
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
  const uint32_t accf0 = smem_u32(bars + 2 * S), acce0 = smem_u32(bars + 2 * S + 2);
  const uint32_t drain = smem_u32(bars + 2 * S + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  const uint32_t rfull0 = smem_u32(bars + 2 * S + 6), rempty0 = rfull0 + 8 * RS;
  const uint32_t rank = cluster_ctarank();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int pair_id = blockIdx.x / 2, npairs = gridDim.x / 2;
  const int my_tiles = pair_id < g.nunits ? (g.nunits - 1 - pair_id) / npairs + 1 : 0;
  const int nsteps = my_tiles * g.KSU;  // this pair's K steps, in order

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      // TMA mode: the even CTA's expect_tx arrival; LUT modes: that and one
      // arrival per decoder warp of the step's group in both CTAs
      mbar_init(full0 + 8 * s, C::LUT ? 1 + 2 * DQ_WARPS : 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int i = 0; i < RS; ++i) {
      mbar_init(rfull0 + 8 * i, 1);
      mbar_init(rempty0 + 8 * i, DQ_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(accf0 + 8 * i, 1);
      mbar_init(acce0 + 8 * i, 2 * EPI_WARPS);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (MODE == MODE_LUT8) {
    // the palette, one copy per bank: entry e of lane l at word e * 32 + l
    for (int i = threadIdx.x; i < 256 * 32; i += C::THREADS) pal32[i] = g.pal[i >> 5];
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- A (and TMA-mode weight) producer, both CTAs ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
      const uint32_t s0 = smem_u32(smem);
      const uint32_t fb0 = mapa_shared(full0, 0);
      int stage = 0;
      uint32_t phase = 0;
      StepWalk wk(g, pair_id, npairs, 0);
      for (int st = 0; st < nsteps; ++st, wk.advance(g, pair_id, npairs, 1)) {
        const int b = wk.b, tm = wk.tm, tn = wk.tn, ks = wk.ks();
        if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, g.err, ERR_EMPTY)) break;
        const uint32_t sb = s0 + stage * STAGE_BYTES;
        if (rank == 0)
          mbar_expect_tx(full0 + 8 * stage, C::LUT ? 2 * A_BYTES : 2 * (A_BYTES + B_BYTES));
        tma_load_2d_pair(sb, &tma_a, ks * 128, b * g.M + tm * 256 + (int)rank * 128,
                         fb0 + 8 * stage);
        if (!C::LUT)
          tma_load_2d_pair(sb + A_BYTES, &tma_w, ks * 128,
                           (g.w_shared ? 0 : b * g.N) + tn * 256 + (int)rank * 128,
                           fb0 + 8 * stage);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      // both CTAs' tiles complete on the even CTA's barriers
      if (rank == 0)
        for (int s = 0; s < S; ++s)
          mbar_wait(full0 + 8 * s, s < stage ? phase : phase ^ 1, g.err, ERR_DRAIN);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0, accp = 0;  // bit b: parity of accumulator b
      bool ok = true;
      const uint32_t id = idesc_bf16(256, 256);
      const uint32_t s0 = smem_u32(smem);
      const uint64_t dA0 = sw128_desc(s0), dB0 = sw128_desc(s0 + A_BYTES);
      for (int it = 0; it < my_tiles && ok; ++it) {
        const int buf = it & 1;
        if (!mbar_wait(acce0 + 8 * buf, ((accp >> buf) & 1) ^ 1, g.err, ERR_ACC)) break;
        accp ^= 1u << buf;
        tc_fence_after();
        const uint32_t dacc = tmem + buf * 256;
        for (int ks = 0; ks < g.KSU; ++ks) {
          if (!wait_cluster(full0 + 8 * stage, phase, g.err, ERR_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t soff = stage * (STAGE_BYTES / 16);
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j)
            mma_bf16_pair(dacc, desc_at(dA0, soff + 2 * j), desc_at(dB0, soff + 2 * j), id,
                          (ks > 0 || j > 0) ? 1u : 0u);
          tc_commit_pair(empty0 + 8 * stage, 0x3);  // frees the stage in both CTAs
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(accf0 + 8 * buf, 0x3);
      }
      tc_commit_pair(drain, 0x1);
      mbar_wait(drain, 0, g.err, ERR_DRAIN);
    }
  } else if (C::LUT && warp == 2) {
    // ---------------- raw producer (LUT modes, both CTAs) ----------------
    if (lane == 0) {
      const uint32_t r0s = smem_u32(smem + C::RAW0);
      int issued = 0;
      StepWalk wk(g, pair_id, npairs, 0);
      for (int st = 0; st < nsteps; ++st, wk.advance(g, pair_id, npairs, 1)) {
        const int b = wk.b, tn = wk.tn, ks = wk.ks();
        int slot;
        uint32_t phase;
        raw_slot<MODE>(st, slot, phase);
        if (!mbar_wait(rempty0 + 8 * slot, phase ^ 1, g.err, ERR_EMPTY)) break;
        const int64_t r0 = wrow(g, g.w_shared ? 0 : b, ks, tn * 256 + (int)rank * 128);
        const uint32_t rb = rfull0 + 8 * slot, dst = r0s + slot * C::RAW_BYTES;
        mbar_expect_tx(rb, 128 * SB + (g.ws4 ? SCALE_BYTES : 0));
        bulk_load(dst, g.wq + r0 * SB, 128 * SB, rb);
        if (g.ws4) bulk_load(dst + 128 * SB, g.ws4 + r0 * 4, SCALE_BYTES, rb);
        issued = st + 1;
      }
      // the last RS steps issued hold each slot's latest phase
      for (int st = max(0, issued - RS); st < issued; ++st) {
        int slot;
        uint32_t phase;
        raw_slot<MODE>(st, slot, phase);
        mbar_wait(rfull0 + 8 * slot, phase, g.err, ERR_DRAIN);
      }
    }
  } else if (C::LUT && warp < C::EPI_WARP0) {
    // ---------------- weight decoders (LUT modes, both CTAs) ----------------
    const int grp = (warp - DEC_WARP0) / DQ_WARPS;
    const int rl = ((warp - DEC_WARP0) % DQ_WARPS) * 32 + lane;  // this thread's weight row
    const uint32_t full_even0 = mapa_shared(full0, 0);
    Pal4 p4;
    if (MODE == MODE_LUT4) p4 = load_pal4(g.pal);
    const bool scaled = g.ws4 != nullptr;
    StepWalk wk(g, pair_id, npairs, grp);
    for (int st = grp; st < nsteps; st += DQ_GROUPS, wk.advance(g, pair_id, npairs, DQ_GROUPS)) {
      const int stage = st % S;
      int slot;
      uint32_t rphase;
      raw_slot<MODE>(st, slot, rphase);
      const int tn = wk.tn, ks = wk.ks();
      // the step's raw bytes: into registers, then the slot goes back
      if (!mbar_wait_warp(rfull0 + 8 * slot, rphase, g.err, ERR_FULL)) break;
      const uint8_t* rawc = smem + C::RAW0 + slot * C::RAW_BYTES;
      const uint16_t* raws =
          scaled ? reinterpret_cast<const uint16_t*>(rawc + 128 * SB) + rl * 4 : nullptr;
      uint32_t raw[2][8], s_lo[2], s_hi[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) read32<MODE>(rawc, rl, raws, h, raw[h], s_lo[h], s_hi[h]);
      __syncwarp();
      if (lane == 0) mbar_arrive(rempty0 + 8 * slot);
      // the stage's weight tile is free once the MMAs of its last round are done
      if (!mbar_wait_warp(empty0 + 8 * stage, ((uint32_t)(st / S) & 1u) ^ 1u, g.err, ERR_EMPTY))
        break;
      const int n = tn * 256 + (int)rank * 128 + rl;
      uint8_t* bt = smem + stage * STAGE_BYTES + A_BYTES + rl * 128;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t o[16];
        const int valid = n < g.N ? min(32, g.K - (ks * KSTEP + h * 32)) : 0;
        decode32<MODE>(raw[h], p4, pal32, lane, s_lo[h], s_hi[h], scaled, max(valid, 0), o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = 4 * h + j;
          *reinterpret_cast<uint4*>(bt + ((c ^ (rl & 7)) << 4)) =
              make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        }
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) arrive_release_cluster(full_even0 + 8 * stage);
    }
  } else if (warp >= C::EPI_WARP0) {
    // ---------------- epilogue (last 4 warps, both CTAs) ----------------
    const int q = warp & 3;
    const uint32_t acce_even0 = mapa_shared(acce0, 0);
    uint32_t accp = 0;
    for (int it = 0; it < my_tiles; ++it) {
      const int buf = it & 1;
      int b, tm, tn, k0;
      unit_of(g, pair_id + it * npairs, b, tm, tn, k0);
      if (!mbar_wait_warp(accf0 + 8 * buf, (accp >> buf) & 1, g.err, ERR_ACC)) break;
      accp ^= 1u << buf;
      tc_fence_after();
      const int row = tm * 256 + (int)rank * 128 + q * 32 + lane;
      const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + buf * 256;
      uint16_t* orow = g.out + (int64_t)b * g.out_bs + (int64_t)row * g.ldo;
      const bool row_ok = row < g.M;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t r[32];
        tmem_ld32(tq + c * 32, r);
        tmem_ld_wait();
        if (c == 7) {
          // the accumulator goes back to the MMA warp before the last stores
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acce_even0 + 8 * buf);
        }
        const int col0 = tn * 256 + c * 32;
        if (!row_ok || col0 >= g.N) continue;
        if (g.S > 1) {  // this K slice's float32 sums, rows of part[k0 / KSU]
          float4* dst = reinterpret_cast<float4*>(
              g.part + ((int64_t)(k0 / g.KSU) * g.M + row) * g.N + col0);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (col0 + 4 * i < g.N)
              dst[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                   __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
          continue;
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float v0 = __uint_as_float(r[2 * i]), v1 = __uint_as_float(r[2 * i + 1]);
          if (g.bias) {
            v0 += bf2f(g.bias[min(col0 + 2 * i, g.N - 1)]);
            v1 += bf2f(g.bias[min(col0 + 2 * i + 1, g.N - 1)]);
          }
          __nv_bfloat162 bb = __floats2bfloat162_rn(v0, v1);
          pk[i] = *reinterpret_cast<uint32_t*>(&bb);
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + col0);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (col0 + 8 * i < g.N) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
    }
  }
  __syncthreads();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// Split-K: out[m, n] = bf16(sum over s of part[s][m][n], in s order, + bias[n]),
// 8 columns per thread (N % 8 == 0).
__global__ void k_dq_finalize(const float* part, int S, int M, int N, const uint16_t* bias,
                              uint16_t* out, int64_t ldo) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int n8 = N / 8;
  if (i >= (int64_t)M * n8) return;
  const int m = (int)(i / n8), n = (int)(i % n8) * 8;
  float v[8];
  for (int e = 0; e < 8; ++e) v[e] = 0.f;
  for (int sp = 0; sp < S; ++sp) {
    const float4* q = reinterpret_cast<const float4*>(part + ((int64_t)sp * M + m) * N + n);
    const float4 a = q[0], b = q[1];
    v[0] += a.x, v[1] += a.y, v[2] += a.z, v[3] += a.w;
    v[4] += b.x, v[5] += b.y, v[6] += b.z, v[7] += b.w;
  }
  uint32_t pk[4];
  for (int e = 0; e < 4; ++e) {
    float x0 = v[2 * e], x1 = v[2 * e + 1];
    if (bias) {
      x0 += bf2f(bias[n + 2 * e]);
      x1 += bf2f(bias[n + 2 * e + 1]);
    }
    __nv_bfloat162 bb = __floats2bfloat162_rn(x0, x1);
    pk[e] = *reinterpret_cast<uint32_t*>(&bb);
  }
  *reinterpret_cast<uint4*>(out + (int64_t)m * ldo + n) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// The weight decode on its own: out[row, k] bf16 over [rows, K] (row-major),
// the same values the GEMM's decoder warps write into shared memory.  Used
// for large M, where one decode per call to HBM costs less than the GEMM's
// decode per 256-row tile of the activations, and by the tests.  Thread i
// takes 32 elements (half h of K step ks) of row i % rows, so a warp reads
// 32 rows' consecutive 16-byte chunks of a step and writes 32 row segments of
// 64 bytes.
template <int MODE>
__global__ void k_dq_decode(const __grid_constant__ DqArgs g, int rows, uint16_t* out) {
  __shared__ uint32_t pal32[MODE == MODE_LUT8 ? 256 * 32 : 1];
  if (MODE == MODE_LUT8) {
    for (int j = threadIdx.x; j < 256 * 32; j += blockDim.x) pal32[j] = g.pal[j >> 5];
    __syncthreads();
  }
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (step, half, row)
  const int64_t total = (int64_t)rows * g.KS * 2;
  if (i >= total) return;
  const int64_t row = i % rows, sh = i / rows;
  const int h = (int)(sh & 1), ks = (int)(sh >> 1);
  Pal4 p4;
  if (MODE == MODE_LUT4) p4 = load_pal4(g.pal);
  uint32_t raw[8], sl, sh_, o[16];
  const int64_t r0 = wrow(g, 0, ks, (int)row);
  const int64_t blk0 = wrow(g, 0, ks, (int)(row & ~127ll));  // the row's 128-row block
  read32<MODE>(g.wq + blk0 * Cfg<MODE>::STEP_BYTES, (int)(row & 127), g.ws4 ? g.ws4 + r0 * 4 : nullptr,
               h, raw, sl, sh_);
  const int k0 = ks * KSTEP + h * 32;
  const int valid = min(32, g.K - k0);
  if (valid <= 0) return;
  decode32<MODE>(raw, p4, pal32, threadIdx.x & 31, sl, sh_, g.ws4 != nullptr, valid, o);
  uint16_t* dst = out + row * g.K + k0;
  if (valid == 32 && (g.K & 7) == 0) {  // 16-byte aligned: K % 8 == 0, k0 % 32 == 0
#pragma unroll
    for (int j = 0; j < 4; ++j)
      reinterpret_cast<uint4*>(dst)[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e)
      if (e < valid) dst[e] = (uint16_t)((o[e / 2] >> (16 * (e & 1))) & 0xFFFFu);
  }
}

// ---- packing: bf16 codes -> palette indices --------------------------------
struct PackDqArgs {
  const uint16_t* codes;  // bf16 [wb * N, K]
  const uint16_t* keys;   // sorted bit patterns of the palette [P] (value mode)
  uint8_t* out;           // [wb][KS][Npad][step_bytes]
  int wb, N, Npad, K, KS, P, step_bytes;
  int index_mode;         // 1: the code is the index itself (a float 0 .. P-1)
  const uint8_t* key_index;  // value mode: palette position of keys[i]
  int* missing;           // codes with no palette entry
};

// One thread: 8 consecutive elements of a row -> 8 indices (4 or 8 bytes)
// in the step-major layout; rows from N to Npad are zero.
__global__ void k_dq_pack(const __grid_constant__ PackDqArgs p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = p.KS * KSTEP / 8;
  if (i >= (int64_t)p.wb * p.Npad * per_row) return;
  const int64_t rp = i / per_row;  // packed row over all weight batches
  const int wbi = (int)(rp / p.Npad), n = (int)(rp % p.Npad);
  const int c0 = (int)(i % per_row) * 8;
  const int64_t r = (int64_t)wbi * p.N + n;  // source row
  uint32_t idx[8];
  int bad = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int c = c0 + e;
    uint32_t v = 0;
    if (c < p.K && n < p.N) {
      const uint16_t bits = p.codes[r * p.K + c];
      if (p.index_mode) {
        const float f = bf2f(bits);
        const int n = (int)f;
        if (!(f >= 0.f) || (float)n != f || n >= p.P) bad++;
        else v = (uint32_t)n;
      } else {
        int lo = 0, hi = p.P - 1, found = -1;
        while (lo <= hi) {
          const int mid = (lo + hi) >> 1;
          const uint16_t k = p.keys[mid];
          if (k == bits) {
            found = mid;
            break;
          }
          if (k < bits) lo = mid + 1;
          else hi = mid - 1;
        }
        if (found < 0) bad++;
        else v = p.key_index[found];
      }
    }
    idx[e] = v;
  }
  // the row's 128-row block of this step, chunk-major inside
  const int ks = c0 / KSTEP, within = c0 % KSTEP;
  const int byte = p.step_bytes == 32 ? within / 2 : within;  // offset in the row's step bytes
  uint8_t* dst = p.out + (((int64_t)wbi * p.KS + ks) * p.Npad + (n & ~127)) * p.step_bytes +
                 (byte / 16) * 2048 + (n & 127) * 16 + byte % 16;
  if (p.step_bytes == 32) {  // nibbles, element j of a byte pair in the low nibble
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) w |= (idx[e] & 0xFu) << (4 * e);
    *reinterpret_cast<uint32_t*>(dst) = w;
  } else {
    const uint32_t w0 = idx[0] | (idx[1] << 8) | (idx[2] << 16) | (idx[3] << 24);
    const uint32_t w1 = idx[4] | (idx[5] << 8) | (idx[6] << 16) | (idx[7] << 24);
    *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);
  }
  if (bad && p.missing) atomicAdd(p.missing, bad);
}

// Quarter-step scales: out[wb][KS][Npad][4] = the scale of elements
// ks * 64 + 16 j .. + 15 of row n (block size 2^bs_log2; one per row when
// nkb == 1), 0 for rows from N to Npad.
__global__ void k_dq_pack_scales(const uint16_t* scale, int wb, int N, int Npad, int KS, int nkb,
                                 int bs_log2, uint16_t* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)wb * KS * Npad * 4;
  if (i >= total) return;
  const int j = (int)(i & 3);
  const int64_t q = i >> 2;
  const int n = (int)(q % Npad);
  const int64_t t = q / Npad;
  const int ks = (int)(t % KS), wbi = (int)(t / KS);
  uint16_t v = 0;
  if (n < N) {
    const int kb = nkb == 1 ? 0 : min((ks * KSTEP + 16 * j) >> bs_log2, nkb - 1);
    v = scale[((int64_t)wbi * N + n) * nkb + kb];
  }
  out[i] = v;
}

// Which bf16 bit patterns occur: present[bits] = 1.  Each CTA gathers a
// 65,536-bit set in shared memory first (a weight holds few patterns, so
// direct stores would pile onto the same bytes), then writes out its bits.
__global__ void k_dq_patterns(const uint16_t* codes, int64_t n, uint8_t* present) {
  __shared__ uint32_t bits[2048];
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) bits[i] = 0;
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t b = codes[i];
    const uint32_t m = 1u << (b & 31);
    if (!(bits[b >> 5] & m)) atomicOr(&bits[b >> 5], m);
  }
  __syncthreads();
  for (int w = threadIdx.x; w < 2048; w += blockDim.x) {
    uint32_t v = bits[w];
    while (v) {
      const int j = __ffs(v) - 1;
      v &= v - 1;
      present[w * 32 + j] = 1;
    }
  }
}

// dst[b][c][r] = src[b][r][c] for bf16 [batch][rows, cols]: 32 x 32 tiles
// through shared memory (a padded row against bank conflicts).
__global__ void k_transpose_bf16(const uint16_t* src, int rows, int cols, uint16_t* dst) {
  __shared__ uint16_t t[32][33];
  const int64_t b = blockIdx.z;
  const uint16_t* s = src + b * rows * (int64_t)cols;
  uint16_t* d = dst + b * rows * (int64_t)cols;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[i][threadIdx.x] = s[(int64_t)r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) d[(int64_t)c * rows + r] = t[threadIdx.x][i];
  }
}

int sticky_dq(int* out, int clear, cudaStream_t st) { return sticky_read(out, clear, st); }

}  // namespace dq
namespace mx {
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_bytes,
              uint32_t box_rows);
int sm_count();
}  // namespace mx
}  // namespace vq

using namespace vq::dq;

namespace {

template <int MODE>
int launch_dq(const CUtensorMap& ma, const CUtensorMap& mw, const DqArgs& g, cudaStream_t st) {
  const int smem = Cfg<MODE>::SMEM + 1024;
  if (cudaFuncSetAttribute(k_gemm_dq<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return VQ_ERR_CUDA;
  const int pairs = (int)std::min<int64_t>(g.nunits, vq::mx::sm_count() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(Cfg<MODE>::THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k_gemm_dq<MODE>, ma, mw, g) != cudaSuccess) return VQ_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int log2_exact(int64_t v) {
  int l = 0;
  while ((1ll << l) < v) ++l;
  return (1ll << l) == v ? l : -1;
}

int64_t npad_of(int64_t N) { return (N + 255) / 256 * 256; }

// K splits for one GEMM with fewer output tiles than CTA pairs: the count
// that gives the fewest K steps on the busiest pair, a split GEMM paying in
// step units for the finalize launch (4) and for its float32 slices written
// and read back (about 4 MB a step: the GPU's HBM traffic in the ~0.6 us of
// one decode-bound step); slices of at least 8 steps that divide the K steps
// evenly; one batch only.
int splits_for(int64_t batch, int64_t M, int64_t N, int64_t K) {
  if (batch != 1) return 1;
  const int64_t KS = (K + KSTEP - 1) / KSTEP, tiles = (M + 255) / 256 * ((N + 255) / 256);
  const int64_t pairs = std::max(1, vq::mx::sm_count() / 2);
  if (tiles >= pairs) return 1;
  int best = 1;
  int64_t best_cost = (tiles + pairs - 1) / pairs * KS;
  for (int S = 2; S <= 64; ++S) {
    if (KS % S || KS / S < 8) continue;
    const int64_t traffic = (int64_t)(S + 1) * M * N * 8;
    const int64_t cost =
        (tiles * S + pairs - 1) / pairs * (KS / S) + 4 + (traffic + 3999999) / 4000000;
    if (cost < best_cost) {
      best = S;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace

extern "C" {

int32_t vq_gemm_dq_splits(int64_t batch, int64_t M, int64_t N, int64_t K) {
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) return 1;
  return splits_for(batch, M, N, K);
}

int vq_gemm_dq(const void* a, int64_t batch, int64_t M, int64_t K, int32_t mode, const void* w,
               int32_t w_shared, int64_t N, const void* w_scale4, const void* palette,
               const void* bias, void* out, int64_t ldo, int64_t out_batch_stride, int32_t* d_err,
               void* stream) {
  return vq_gemm_dq_ex(a, batch, M, K, mode, w, w_shared, N, w_scale4, palette, bias, out, ldo,
                       out_batch_stride, 1, nullptr, d_err, stream);
}

int vq_gemm_dq_ex(const void* a, int64_t batch, int64_t M, int64_t K, int32_t mode, const void* w,
                  int32_t w_shared, int64_t N, const void* w_scale4, const void* palette,
                  const void* bias, void* out, int64_t ldo, int64_t out_batch_stride,
                  int32_t splits, float* workspace, int32_t* d_err, void* stream) {
  if (!a || !w || !out || !d_err) return VQ_ERR_NULL;
  if (mode < MODE_TMA || mode > MODE_LUT8) return VQ_ERR_INVALID;
  if (mode != MODE_TMA && !palette) return VQ_ERR_NULL;
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) return VQ_ERR_INVALID;
  if (K % 8 || N % 8 || ldo < N || ldo % 8) return VQ_ERR_UNSUPPORTED;
  if (batch > 1 && out_batch_stride < M * ldo) return VQ_ERR_INVALID;
  if (out_batch_stride % 8) return VQ_ERR_ALIGNMENT;
  if (batch * M >= (1ll << 31) || batch * npad_of(N) * ((K + 63) / 64) >= (1ll << 31) ||
      K >= (1 << 24))
    return VQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(bias) & 1) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(w_scale4) & 15) || (reinterpret_cast<uintptr_t>(palette) & 15))
    return VQ_ERR_ALIGNMENT;
  DqArgs g = {};
  g.wq = (const uint8_t*)w;
  g.ws4 = mode == MODE_TMA ? nullptr : (const uint16_t*)w_scale4;
  g.pal = (const uint16_t*)palette;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.KS = (int)((K + KSTEP - 1) / KSTEP);
  g.Npad = (int)npad_of(N);
  g.bias = (const uint16_t*)bias;
  g.out = (uint16_t*)out;
  g.ldo = ldo;
  g.out_bs = out_batch_stride;
  g.MT2 = (int)((M + 255) / 256);
  g.NTN = (int)((N + 255) / 256);
  const int64_t ntiles = batch * g.MT2 * g.NTN;
  if (ntiles >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  g.ntiles = (int)ntiles;
  g.w_shared = w_shared ? 1 : 0;
  g.err = d_err;
  if (splits < 1 || g.KS % splits) return VQ_ERR_INVALID;
  if (splits > 1) {
    if (batch != 1) return VQ_ERR_UNSUPPORTED;
    if (!workspace) return VQ_ERR_NULL;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return VQ_ERR_ALIGNMENT;
    if ((int64_t)splits * M * N >= (1ll << 40)) return VQ_ERR_UNSUPPORTED;
  }
  g.S = splits;
  g.KSU = g.KS / splits;
  if (ntiles * splits >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  g.nunits = (int)(ntiles * splits);
  g.part = workspace;
  CUtensorMap ma, mw;
  if (!vq::mx::make_map(&ma, a, batch * M, K * 2, 128)) return VQ_ERR_CUDA;
  if (mode == MODE_TMA) {
    if (!vq::mx::make_map(&mw, w, (w_shared ? 1 : batch) * N, K * 2, 128)) return VQ_ERR_CUDA;
  } else {
    mw = ma;  // unused
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(d_err, 0, sizeof(int32_t), s) != cudaSuccess) return VQ_ERR_CUDA;
  const int rc = mode == MODE_TMA    ? launch_dq<MODE_TMA>(ma, mw, g, s)
                 : mode == MODE_LUT4 ? launch_dq<MODE_LUT4>(ma, mw, g, s)
                                     : launch_dq<MODE_LUT8>(ma, mw, g, s);
  if (rc != VQ_OK || splits == 1) return rc;
  const int64_t n = M * (N / 8);
  k_dq_finalize<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(workspace, splits, (int)M, (int)N,
                                                           (const uint16_t*)bias, (uint16_t*)out, ldo);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_dq_pack_sizes(int64_t wbatch, int64_t N, int64_t K, int32_t mode, int64_t* codes_bytes,
                     int64_t* scale_bytes) {
  if (!codes_bytes || !scale_bytes) return VQ_ERR_NULL;
  if (wbatch <= 0 || N <= 0 || K <= 0 || (mode != MODE_LUT4 && mode != MODE_LUT8))
    return VQ_ERR_INVALID;
  const int64_t rows = wbatch * ((K + KSTEP - 1) / KSTEP) * npad_of(N);
  *codes_bytes = rows * (mode == MODE_LUT4 ? 32 : 64);
  *scale_bytes = rows * 8;
  return VQ_OK;
}

int vq_dq_pack(const vq_tensor* codes, int64_t wbatch, int32_t mode, int32_t index_mode,
               const void* keys, const void* key_index, int32_t npal, void* out,
               int32_t* d_missing, void* stream) {
  if (!codes || !out) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || codes->ndim != 2) return VQ_ERR_UNSUPPORTED;
  if (mode != MODE_LUT4 && mode != MODE_LUT8) return VQ_ERR_INVALID;
  // index mode: npal palette entries; value mode: npal keys (their palette
  // positions, key_index, are below 16 / 256)
  if (npal <= 0 || npal > 65536) return VQ_ERR_INVALID;
  if (index_mode && npal > (mode == MODE_LUT4 ? 16 : 256)) return VQ_ERR_INVALID;
  if (!index_mode && (!keys || !key_index)) return VQ_ERR_NULL;
  const int64_t R = codes->shape[0], K = codes->shape[1];
  if (wbatch <= 0 || R <= 0 || R % wbatch || K <= 0 || K >= (1 << 24)) return VQ_ERR_INVALID;
  const int64_t N = R / wbatch, KS = (K + KSTEP - 1) / KSTEP;
  if (wbatch * KS * npad_of(N) >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(out) & 15) return VQ_ERR_ALIGNMENT;
  PackDqArgs p;
  p.codes = (const uint16_t*)codes->data;
  p.keys = (const uint16_t*)keys;
  p.key_index = (const uint8_t*)key_index;
  p.out = (uint8_t*)out;
  p.wb = (int)wbatch;
  p.N = (int)N;
  p.Npad = (int)npad_of(N);
  p.K = (int)K;
  p.KS = (int)KS;
  p.P = npal;
  p.step_bytes = mode == MODE_LUT4 ? 32 : 64;
  p.index_mode = index_mode;
  p.missing = d_missing;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (d_missing && cudaMemsetAsync(d_missing, 0, sizeof(int32_t), s) != cudaSuccess)
    return VQ_ERR_CUDA;
  const int64_t n = wbatch * p.Npad * (KS * KSTEP / 8);
  k_dq_pack<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_dq_pack_scales(const void* scale, int64_t wbatch, int64_t N, int64_t K, int64_t nkb,
                      int64_t block_size, void* out, void* stream) {
  if (!scale || !out) return VQ_ERR_NULL;
  if (wbatch <= 0 || N <= 0 || K <= 0 || K >= (1 << 24) || nkb <= 0) return VQ_ERR_INVALID;
  int l = 30;
  if (nkb > 1) {
    l = log2_exact(block_size);
    if (l < 4 || (K + block_size - 1) / block_size != nkb) return VQ_ERR_UNSUPPORTED;
  }
  const int64_t KS = (K + KSTEP - 1) / KSTEP, total = wbatch * KS * npad_of(N) * 4;
  if (total >= (1ll << 33) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(scale) & 1))
    return total >= (1ll << 33) ? VQ_ERR_UNSUPPORTED : VQ_ERR_ALIGNMENT;
  k_dq_pack_scales<<<(unsigned)((total + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      (const uint16_t*)scale, (int)wbatch, (int)N, (int)npad_of(N), (int)KS, (int)nkb, l,
      (uint16_t*)out);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_dq_patterns(const vq_tensor* codes, void* present, void* stream) {
  if (!codes || !present) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  int64_t n = 1;
  for (int i = 0; i < codes->ndim; ++i) n *= codes->shape[i];
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(present, 0, 65536, s) != cudaSuccess) return VQ_ERR_CUDA;
  if (n == 0) return VQ_OK;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  k_dq_patterns<<<grid, 256, 0, s>>>((const uint16_t*)codes->data, n, (uint8_t*)present);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_transpose_bf16(const void* src, int64_t batch, int64_t rows, int64_t cols, void* dst,
                      void* stream) {
  if (!src || !dst) return VQ_ERR_NULL;
  if (batch <= 0 || rows <= 0 || cols <= 0) return VQ_ERR_INVALID;
  if (rows >= (1 << 30) || cols >= (1 << 30) || batch >= 65536 || (rows + 31) / 32 >= 65536)
    return VQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(src) & 1) || (reinterpret_cast<uintptr_t>(dst) & 1))
    return VQ_ERR_ALIGNMENT;
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch);
  k_transpose_bf16<<<grid, dim3(32, 8), 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      (const uint16_t*)src, (int)rows, (int)cols, (uint16_t*)dst);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_dq_decode(const void* w, int64_t N, int64_t K, int32_t mode, const void* w_scale4,
                 const void* palette, void* out, void* stream) {
  if (!w || !out || !palette) return VQ_ERR_NULL;
  if (mode != MODE_LUT4 && mode != MODE_LUT8) return VQ_ERR_INVALID;
  if (N <= 0 || K <= 0 || K >= (1 << 24) || N >= (1ll << 30)) return VQ_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(w_scale4) & 15) ||
      (reinterpret_cast<uintptr_t>(palette) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return VQ_ERR_ALIGNMENT;
  DqArgs g = {};
  g.wq = (const uint8_t*)w;
  g.ws4 = (const uint16_t*)w_scale4;
  g.pal = (const uint16_t*)palette;
  g.N = (int)N;
  g.K = (int)K;
  g.KS = (int)((K + KSTEP - 1) / KSTEP);
  g.Npad = (int)npad_of(N);
  const int64_t n = N * g.KS * 2;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (mode == MODE_LUT4)
    k_dq_decode<MODE_LUT4><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, (int)N, (uint16_t*)out);
  else
    k_dq_decode<MODE_LUT8><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(g, (int)N, (uint16_t*)out);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
