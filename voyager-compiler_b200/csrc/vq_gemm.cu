// MXFP8 block-scaled GEMM on the 5th-generation tensor cores (tcgen05).
//
// Replaces the dequantize-then-matmul of quantized_ops::linear_mx /
// matmul_mx (src/voyager_compiler/ops/quantized.py:455-472, 522-648) when
// both operands are E4M3 codes with power-of-two block-32 scales along K:
//
//   out[m, n] = sum_k (A[m,k] * sA[m,k/32]) * (B[n,k] * sB[n,k/32]) (+ bias[n])
//
// Operands are first packed (vq_mx_pack): codes to E4M3 bytes, row-major
// [rows, Kp] with Kp = K rounded up to 128 (zero filled), and scales to UE8M0
// bytes in the tensor cores' scale-factor layout: for each 128-element K tile
// and each 128-row chunk a 512-byte atom, byte (r % 32) * 16 + (r / 32 % 4) * 4
// + j for row r and K block j (0..3) of the tile; atoms ordered
// [k_tile][row_chunk].
//
// Kernel: persistent, one CTA (11 warps) per SM.
//   warp 0  TMA producer: A tile 128x128 B, B tile 256x128 B (SWIZZLE_128B),
//           scale atoms by bulk copy, 4-stage mbarrier pipeline;
//   warp 10 scale-copy issuer: per K tile, once the stage lands, tcgen05.cp
//           of its scale atoms into the stage's own TMEM slot, committed to
//           the stage's sf_full barrier (issued apart from the MMAs, the
//           copies overlap them in the tensor pipe);
//   warp 1  TMEM owner and MMA issuer: per K tile, after sf_full, 4 x
//           tcgen05.mma.kind::mxf8f6f4.block_scale (M=128, N=256, K=32)
//           accumulating in TMEM (fp32, 256 columns);
//   warps 2-9 epilogue: tcgen05.ld of the accumulator (two warps per lane
//           quarter, 128 columns each), + bias, round to bf16; the
//           accumulator is released as soon as the loads land, so the MMA
//           warp waits only for the TMEM reads.
// Every wait is bounded; a wait that gives up sets *err and the kernel ends.
// No TMA multicast is used.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "vq_numerics.cuh"
#include "vq_tc.cuh"

namespace vq {
namespace mx {

constexpr int BM = 128, BN = 256, BK = 128;  // BK in fp8 bytes = elements
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;             // 16 KB
constexpr int B_BYTES = BN * BK;             // 32 KB
constexpr int SFA_BYTES = 512;               // one 128-row atom
constexpr int SFB_BYTES = 1024;              // two 128-row atoms
constexpr int TX_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;  // per stage
constexpr int STAGE_BYTES = (TX_BYTES + 1023) / 1024 * 1024;  // stages stay 1024-aligned
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0;    // 256 fp32 columns
// Scale factors: one 16-column slot per pipeline stage (A: 4 columns, B: 8),
// so the copies of the next K tile's scales write columns that the MMAs of
// the K tiles still in flight do not read.
constexpr int SF_COL = 256;
constexpr int SF_SLOT = 16;
constexpr int SFA_OFF = 0, SFB_OFF = 4;
constexpr int THREADS = 320;

enum { ERR_TIMEOUT_FULL = 1, ERR_TIMEOUT_EMPTY = 2, ERR_TIMEOUT_ACC = 3, ERR_TIMEOUT_DRAIN = 4 };

// Before a CTA frees its TMEM and exits, each thread that issued
// asynchronous work waits (bounded) for it: the TMA producer for the loads
// of the last round of stages it armed (a stage never armed reads as
// complete at parity 1), the MMA and scale-copy threads for every tcgen05
// operation they issued (a commit to a barrier of their own).  On the
// normal path all of these have completed already; after a wait that gave
// up they keep TMEM and shared memory alive until the work in flight lands.
template <int NSTAGES>
__device__ __forceinline__ void drain_loads(uint32_t full0, int stage, uint32_t phase, int* err) {
#pragma unroll 1
  for (int s = 0; s < NSTAGES; ++s)
    tc::mbar_wait(full0 + 8 * s, s < stage ? phase : phase ^ 1, err, ERR_TIMEOUT_DRAIN);
}

struct SmemLayout {
  // stages first (1024-byte aligned for SWIZZLE_128B), then barriers
  static constexpr int kStages = 0;
  static constexpr int kBars = STAGES * STAGE_BYTES;
  static constexpr int kTotal = kBars + 256;
};

using namespace vq::tc;

// Instruction descriptor of this kernel's MMA (M = 128, N = 256).
__device__ __forceinline__ uint32_t idesc_mxf8(uint32_t j) { return tc::idesc_mxf8(j, BM, BN); }

// Batched problems (matmul_mx over leading dims): batch b's A rows are
// the packed rows [b * MTb * 128, (b + 1) * MTb * 128) and its scale atoms
// the 128-row tiles b * MTb .. of each K tile; B likewise with b_step
// 128-row chunks per batch (0: one B shared by every batch).  Rows of a
// tile past the batch's M read the next batch's operands and are never
// stored.
struct GemmArgs {
  const uint8_t* sfa;  // [KT][MT][512]
  const uint8_t* sfb;  // [KT][NT128][512]
  const uint16_t* bias;  // bf16 [N] or null
  const uint16_t* residual;  // bf16 [M, ldr] added after the bf16 rounding, or null
  int64_t ldr;
  uint16_t* out;         // bf16 [batch][M, ldo] (may be the residual itself)
  int64_t ldo, out_bs;   // out_bs: elements between batches
  int out_mc;            // out is an NVLS multicast address: multimem stores
  int M, N, KT;          // M per batch; KT = Kp / 128
  int MT, NT128, NTILE_N, ntiles;  // MT, NT128: atom rows over all batches
  int MTb, MT2b, b_step;  // per batch: 128-row A tiles, 256-row tiles, B chunks
  int* err;
};

// Tile t -> (batch, row tile of `mtiles` per batch, 256-column tile).
__device__ __forceinline__ void tile_of(const GemmArgs& g, int t, int mtiles, int& b, int& tm,
                                        int& tn) {
  const int per_b = mtiles * g.NTILE_N;
  b = t / per_b;
  const int r = t - b * per_b;
  tm = r / g.NTILE_N;
  tn = r - tm * g.NTILE_N;
}

// One 128-row x 256-column accumulator tile of this CTA's TMEM -> out rows
// (bias, bf16, optional residual add, optional multicast stores).  Two warps
// per TMEM lane quarter (q), each on 128 columns (half); the accumulator is
// read into registers and released (release()) before any arithmetic.
template <typename Release>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& g, uint32_t tmem, int q, int half,
                                              int lane, int b, int row, int colh, Release release) {
  // all four TMEM loads, one wait, then the accumulator goes back to the
  // MMA warp before any arithmetic
  uint32_t raw[4][32];
  const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + ACC_COL + half * 128;
  tmem_ld32(taddr, raw[0]);
  tmem_ld32(taddr + 32, raw[1]);
  tmem_ld32(taddr + 64, raw[2]);
  tmem_ld32(taddr + 96, raw[3]);
  tmem_ld_wait();
  tc_fence_before();
  release();
  uint32_t packed[64];
#pragma unroll
  for (int c2 = 0; c2 < 2; ++c2) {
    const uint32_t* r0 = raw[2 * c2];
    const uint32_t* r1 = raw[2 * c2 + 1];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float v0 = __uint_as_float(r0[2 * i]), v1 = __uint_as_float(r0[2 * i + 1]);
      float w0 = __uint_as_float(r1[2 * i]), w1 = __uint_as_float(r1[2 * i + 1]);
      if (g.bias) {
        const int c = colh + c2 * 64 + 2 * i;
        v0 += bf2f(g.bias[min(c, g.N - 1)]);
        v1 += bf2f(g.bias[min(c + 1, g.N - 1)]);
        w0 += bf2f(g.bias[min(c + 32, g.N - 1)]);
        w1 += bf2f(g.bias[min(c + 33, g.N - 1)]);
      }
      __nv_bfloat162 b0 = __floats2bfloat162_rn(v0, v1), b1 = __floats2bfloat162_rn(w0, w1);
      packed[c2 * 32 + i] = *reinterpret_cast<uint32_t*>(&b0);
      packed[c2 * 32 + 16 + i] = *reinterpret_cast<uint32_t*>(&b1);
    }
  }
  if (row < g.M && colh < g.N) {
    uint16_t* orow = g.out + (int64_t)b * g.out_bs + (int64_t)row * g.ldo;
    if (g.residual) {
      // out = bf16(bf16(acc) + residual): the residual add that follows
      // the linear in the graph, one rounding per op
      const uint4* rrow = reinterpret_cast<const uint4*>(g.residual + (int64_t)row * g.ldr + colh);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (colh + 8 * i >= g.N) break;
        const uint4 rv = rrow[i];
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t pw = packed[4 * i + k];
          __nv_bfloat162 b = __floats2bfloat162_rn(
              __uint_as_float(pw << 16) + __uint_as_float(rw[k] << 16),
              __uint_as_float(pw & 0xFFFF0000u) + __uint_as_float(rw[k] & 0xFFFF0000u));
          packed[4 * i + k] = *reinterpret_cast<uint32_t*>(&b);
        }
      }
    }
    // N is a multiple of 8: whole 16-byte groups up to the last column
    uint4* dst = reinterpret_cast<uint4*>(orow + colh);
    if (g.out_mc) {
      // one store reaches every rank's copy of the output
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (colh + 8 * i < g.N)
          asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(
                           dst + i),
                       "f"(__uint_as_float(packed[4 * i])), "f"(__uint_as_float(packed[4 * i + 1])),
                       "f"(__uint_as_float(packed[4 * i + 2])),
                       "f"(__uint_as_float(packed[4 * i + 3]))
                       : "memory");
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (colh + 8 * i < g.N)
          dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
    }
  }
}

__global__ void __launch_bounds__(THREADS + 32, 1)
    k_gemm_mxf8(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ GemmArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // align the stage area to 1024 bytes (SWIZZLE_128B atoms)
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SmemLayout::kBars);
  // bars[0..S) full, [S..2S) empty, [2S] acc_full, [2S+1] acc_empty, [2S+2] tmem slot,
  // [2S+3..3S+3) sf_full (the stage's scale atoms are in TMEM), [3S+3] drain
  // of the MMA thread's tcgen05 operations, [3S+4] of the scale copies
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t acc_full = smem_u32(bars + 2 * STAGES), acc_empty = smem_u32(bars + 2 * STAGES + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2);
  const uint32_t sf_full0 = smem_u32(bars + 2 * STAGES + 3);
  const uint32_t drain_mma = smem_u32(bars + 3 * STAGES + 3), drain_sf = drain_mma + 8;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
      mbar_init(sf_full0 + 8 * s, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    mbar_init(drain_mma, 1);
    mbar_init(drain_sf, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < g.ntiles && ok; t += gridDim.x) {
        int b, tm, tn;
        tile_of(g, t, g.MTb, b, tm, tn);
        const int ga = b * g.MTb + tm, gb = b * g.b_step + 2 * tn;  // atom rows
        for (int kt = 0; kt < g.KT; ++kt) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, g.err, ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t sbase = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t fb = full0 + 8 * stage;
          mbar_expect_tx(fb, TX_BYTES);
          tma_load_2d(sbase, &tma_a, kt * BK, ga * BM, fb);
          tma_load_2d(sbase + A_BYTES, &tma_b, kt * BK, gb * 128, fb);
          bulk_load(sbase + A_BYTES + B_BYTES, g.sfa + ((size_t)kt * g.MT + ga) * 512, SFA_BYTES, fb);
          bulk_load(sbase + A_BYTES + B_BYTES + SFA_BYTES,
                    g.sfb + ((size_t)kt * g.NT128 + gb) * 512, SFB_BYTES, fb);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      drain_loads<STAGES>(full0, stage, phase, g.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      // the descriptors of stage 0; a stage's are these moved by its offset
      const uint32_t s0 = smem_u32(smem);
      const uint64_t dA0 = sw128_desc(s0), dB0 = sw128_desc(s0 + A_BYTES);
      for (int t = blockIdx.x; t < g.ntiles && ok; t += gridDim.x) {
        // the epilogue has drained the accumulator of the previous tile
        if (!mbar_wait(acc_empty, acc_phase ^ 1, g.err, ERR_TIMEOUT_ACC)) break;
        acc_phase ^= 1;
        tc_fence_after();
        for (int kt = 0; kt < g.KT; ++kt) {
          // the stage's operands landed and warp 10 copied its scales
          if (!mbar_wait(sf_full0 + 8 * stage, phase, g.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t soff = stage * (STAGE_BYTES / 16);
          const uint32_t sfc = tmem + SF_COL + stage * SF_SLOT;
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {
            const uint64_t da = desc_at(dA0, soff + 2 * j);
            const uint64_t db = desc_at(dB0, soff + 2 * j);
            const uint32_t accum = (kt > 0 || j > 0) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], "
                "p;\n\t}" ::"r"(tmem + ACC_COL),
                "l"(da), "l"(db), "r"(idesc_mxf8(j)), "r"(accum), "r"(sfc + SFA_OFF + (j << 30)),
                "r"(sfc + SFB_OFF + (j << 30)));
          }
          // frees the stage once these MMAs (and copies) have read it
          asm volatile(
              "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                  empty0 + 8 * stage)
              : "memory");
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        asm volatile(
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                acc_full)
            : "memory");
      }
      tc_commit(drain_mma);
      mbar_wait(drain_mma, 0, g.err, ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 10) {
    // ---------------- scale-copy issuer ----------------
    // Per stage: once its operands land, the scale atoms go into the stage's
    // TMEM slot and sf_full[stage] fires when the copies complete (from a
    // thread of their own they overlap the MMAs).  The slot was last read by
    // the MMAs of this stage's previous round, which completed before the
    // stage was refilled.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t dS0 = sf_desc(smem_u32(smem) + A_BYTES + B_BYTES);
      for (int t = blockIdx.x; t < g.ntiles && ok; t += gridDim.x) {
        for (int kt = 0; kt < g.KT; ++kt) {
          if (!mbar_wait(full0 + 8 * stage, phase, g.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t soff = stage * (STAGE_BYTES / 16);
          const uint32_t sfc = tmem + SF_COL + stage * SF_SLOT;
          asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfc + SFA_OFF),
                       "l"(desc_at(dS0, soff)));
          asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfc + SFB_OFF),
                       "l"(desc_at(dS0, soff + SFA_BYTES / 16)));
          asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfc + SFB_OFF + 4),
                       "l"(desc_at(dS0, soff + (SFA_BYTES + 512) / 16)));
          asm volatile(
              "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                  sf_full0 + 8 * stage)
              : "memory");
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      tc_commit(drain_sf);
      mbar_wait(drain_sf, 0, g.err, ERR_TIMEOUT_DRAIN);
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // Two warps per TMEM lane quarter, each on half of the 256 columns.  The
    // accumulator is read into registers (as bf16) and released before the
    // stores, so the next tile's MMAs overlap them.
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;       // columns half * 128 .. + 127
    const int row_in_tile = q * 32 + lane;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < g.ntiles; t += gridDim.x) {
      int b, tm, tn;
      tile_of(g, t, g.MTb, b, tm, tn);
      if (!mbar_wait_warp(acc_full, acc_phase, g.err, ERR_TIMEOUT_ACC)) break;
      acc_phase ^= 1;
      tc_fence_after();
      const int row = tm * BM + row_in_tile;
      const int colh = tn * BN + half * 128;
      epilogue_tile(g, tmem, q, half, lane, b, row, colh, [&] { mbar_arrive(acc_empty); });
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of 2 CTAs on two SMs computes a 256 x 256 tile
// with tcgen05.mma.cta_group::2 (M = 256: 128 rows in each CTA's TMEM).  Each
// CTA loads its own 128 rows of A and its own 128 rows (half) of B per K
// tile -- 33.5 KB per stage instead of 49.5 KB, so 6 stages fit -- plus the
// full B scale atoms (each CTA's TMEM needs all 256 columns' scales).  Both
// CTAs' TMA loads count on the even CTA's "full" barrier; the even CTA's
// single MMA thread issues the pair's MMAs (its warp 10 the pair's scale
// copies) and releases stages and accumulators in both CTAs with multicast
// commits; both epilogues release the accumulator on the even CTA's
// barrier.  No TMA multicast.
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK, P_B_BYTES = 128 * BK;  // this CTA's halves
constexpr int P_TX = P_A_BYTES + P_B_BYTES + SFA_BYTES + SFB_BYTES;  // per CTA and stage
constexpr int P_STAGE_BYTES = (P_TX + 1023) / 1024 * 1024;
constexpr int P_BARS = P_STAGES * P_STAGE_BYTES;
constexpr int P_SMEM = P_BARS + 256;
constexpr int P_THREADS = THREADS + 32;  // + warp 10: the scale-copy issuer
// barrier words: full, empty, sf_full per stage, acc_full, acc_empty, TMEM
// slot, two drains
static_assert((3 * P_STAGES + 5) * 8 <= P_SMEM - P_BARS, "pair barriers exceed their area");
static_assert((3 * STAGES + 5) * 8 <= SmemLayout::kTotal - SmemLayout::kBars,
              "barriers exceed their area");
static_assert(P_SMEM + 1024 <= (1 << 18) && SmemLayout::kTotal + 1024 <= (1 << 18),
              "descriptor offsets assume shared addresses below 2^18");
static_assert(SF_COL + STAGES * SF_SLOT <= TMEM_COLS && SF_COL + P_STAGES * SF_SLOT <= TMEM_COLS,
              "scale-factor slots exceed the TMEM allocation");

__global__ void __launch_bounds__(P_THREADS, 1)
    k_gemm_mxf8_pair(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_sfa,
                     const __grid_constant__ CUtensorMap tma_sfb, const __grid_constant__ GemmArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P_BARS);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + P_STAGES);
  const uint32_t acc_full = smem_u32(bars + 2 * P_STAGES), acc_empty = smem_u32(bars + 2 * P_STAGES + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * P_STAGES + 2);
  // per stage: the stage's scale atoms are in TMEM (even CTA); then the
  // drains of the MMA thread's and the scale copies' tcgen05 operations
  const uint32_t sf_full0 = smem_u32(bars + 2 * P_STAGES + 3);
  const uint32_t drain_mma = smem_u32(bars + 3 * P_STAGES + 3), drain_sf = drain_mma + 8;
  const uint32_t rank = cluster_ctarank();  // 0: issues the pair's MMAs
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int pair_id = blockIdx.x / 2, npairs = gridDim.x / 2;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
      mbar_init(sf_full0 + 8 * s, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 2 * 8);  // one arrival per epilogue warp of both CTAs
    mbar_init(drain_mma, 1);
    mbar_init(drain_sf, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tma_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t s0 = smem_u32(smem);
      const uint32_t fb0 = mapa_shared(full0, 0);  // the even CTA's barriers
      for (int t = pair_id; t < g.ntiles && ok; t += npairs) {
        int b, tm, tn;  // 256-row, 256-column tile of batch b
        tile_of(g, t, g.MT2b, b, tm, tn);
        const int ga = b * g.MTb + 2 * tm + (int)rank, gb = b * g.b_step + 2 * tn;
        const int ya = ga * 128, yb = (gb + (int)rank) * 128;
        // scale-atom rows of K tile kt: (kt * MT + ga) * 2 and
        // (kt * NT128 + gb) * 2, stepped by 2 MT / 2 NT128 per K tile
        int ysa = ga * 2, ysb = gb * 2;
        for (int kt = 0; kt < g.KT; ++kt) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, g.err, ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t sbase = s0 + stage * P_STAGE_BYTES;
          const uint32_t fb = fb0 + 8 * stage;
          if (rank == 0) mbar_expect_tx(full0 + 8 * stage, 2 * P_TX);
          tma_load_2d_pair(sbase, &tma_a, kt * BK, ya, fb);
          tma_load_2d_pair(sbase + P_A_BYTES, &tma_b, kt * BK, yb, fb);
          // scale atoms: this CTA's 128 A rows, both 128-row chunks of B
          tma_load_2d_pair(sbase + P_A_BYTES + P_B_BYTES, &tma_sfa, 0, ysa, fb);
          tma_load_2d_pair(sbase + P_A_BYTES + P_B_BYTES + SFA_BYTES, &tma_sfb, 0, ysb, fb);
          ysa += 2 * g.MT;
          ysb += 2 * g.NT128;
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // both CTAs' loads complete on the even CTA's barriers, so its wait
      // covers the pair (the cluster barrier below holds the odd CTA)
      if (rank == 0) drain_loads<P_STAGES>(full0, stage, phase, g.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t id0 = tc::idesc_mxf8(0, 256, 256), id1 = tc::idesc_mxf8(1, 256, 256),
                     id2 = tc::idesc_mxf8(2, 256, 256), id3 = tc::idesc_mxf8(3, 256, 256);
      const uint32_t ids[4] = {id0, id1, id2, id3};
      // the descriptors of stage 0; a stage's are these moved by its offset
      // (one add per operand instead of rebuilding each descriptor)
      const uint32_t s0 = smem_u32(smem);
      const uint64_t dA0 = sw128_desc(s0), dB0 = sw128_desc(s0 + P_A_BYTES);
      uint32_t soff = 0;                 // stage * P_STAGE_BYTES / 16
      uint32_t sfc = tmem + SF_COL;      // the stage's scale-factor slot
      for (int t = pair_id; t < g.ntiles && ok; t += npairs) {
        // both CTAs' epilogues have drained the accumulator of the last tile
        if (!mbar_wait(acc_empty, acc_phase ^ 1, g.err, ERR_TIMEOUT_ACC)) break;
        acc_phase ^= 1;
        tc_fence_after();
        for (int kt = 0; kt < g.KT; ++kt) {
          // the stage's operands landed and warp 10 copied its scales
          if (!mbar_wait(sf_full0 + 8 * stage, phase, g.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          mma_mxf8_pair(tmem + ACC_COL, desc_at(dA0, soff), desc_at(dB0, soff), ids[0],
                        kt > 0 ? 1u : 0u, sfc + SFA_OFF, sfc + SFB_OFF);
#pragma unroll
          for (uint32_t j = 1; j < 4; ++j)
            mma_mxf8_pair_acc(tmem + ACC_COL, desc_at(dA0, soff + 2 * j),
                              desc_at(dB0, soff + 2 * j), ids[j], sfc + SFA_OFF + (j << 30),
                              sfc + SFB_OFF + (j << 30));
          tc_commit_pair(empty0 + 8 * stage, 0x3);  // frees the stage in both CTAs
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
            soff = 0;
            sfc = tmem + SF_COL;
          } else {
            soff += P_STAGE_BYTES / 16;
            sfc += SF_SLOT;
          }
        }
        if (!ok) break;
        tc_commit_pair(acc_full, 0x3);
      }
      tc_commit_pair(drain_mma, 0x1);
      mbar_wait(drain_mma, 0, g.err, ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 10) {
    // ---------------- scale-copy issuer (even CTA) ----------------
    // Per stage: once its operands land, the pair's scale atoms go into the
    // stage's TMEM slot and sf_full[stage] fires when the copies complete.
    // The slot was last read by the MMAs of this stage's previous round,
    // which completed before the stage was refilled (its "full" phase).
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t dS0 = sf_desc(smem_u32(smem) + P_A_BYTES + P_B_BYTES);
      uint32_t soff = 0, sfc = tmem + SF_COL;
      for (int t = pair_id; t < g.ntiles && ok; t += npairs) {
        for (int kt = 0; kt < g.KT; ++kt) {
          if (!mbar_wait(full0 + 8 * stage, phase, g.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          cp_sf_pair_desc(sfc + SFA_OFF, desc_at(dS0, soff));
          cp_sf_pair_desc(sfc + SFB_OFF, desc_at(dS0, soff + SFA_BYTES / 16));
          cp_sf_pair_desc(sfc + SFB_OFF + 4, desc_at(dS0, soff + (SFA_BYTES + 512) / 16));
          tc_commit_pair(sf_full0 + 8 * stage, 0x1);  // the even CTA's barrier
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
            soff = 0;
            sfc = tmem + SF_COL;
          } else {
            soff += P_STAGE_BYTES / 16;
            sfc += SF_SLOT;
          }
        }
      }
      tc_commit_pair(drain_sf, 0x1);
      mbar_wait(drain_sf, 0, g.err, ERR_TIMEOUT_DRAIN);
    }
  } else {
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t acc_empty0 = mapa_shared(acc_empty, 0);
    uint32_t acc_phase = 0;
    for (int t = pair_id; t < g.ntiles; t += npairs) {
      int b, tm, tn;
      tile_of(g, t, g.MT2b, b, tm, tn);
      if (!mbar_wait_warp(acc_full, acc_phase, g.err, ERR_TIMEOUT_ACC)) break;
      acc_phase ^= 1;
      tc_fence_after();
      const int row = tm * 256 + (int)rank * 128 + row_in_tile;
      const int colh = tn * BN + half * 128;
      epilogue_tile(g, tmem, q, half, lane, b, row, colh, [&] {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty0);
      });
    }
  }
  __syncthreads();
  // neither CTA leaves (or frees TMEM) while the other may still touch its
  // barriers or its TMEM
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// NVFP4 x NVFP4 (E2M1 codes, UE4M3 scales per 16 along K) on
// tcgen05.mma.kind::mxf4nvf4.block_scale.scale_vec::4X: the single-CTA
// kernel above with K tiles of 256 elements (128 bytes of packed E2M1 per
// row), K = 64 per MMA, and four scale bytes per row per MMA -- so one
// 512-byte atom per MMA and 128-row chunk (row r's byte t, the scale of
// elements 16 t .. 16 t + 15 of the MMA's 64, at (r % 32) * 16 + (r / 32) * 4
// + t), four per chunk and K tile, and a 48-column TMEM scale slot per stage
// (A: 4 columns per MMA; B: 8).  code x scale is exact in the tensor core,
// as it is in bf16 for the reference's dequantize.
constexpr int F4_STAGES = 4;
constexpr int F4_SFA = 4 * 512, F4_SFB = 8 * 512;  // per K tile: A 128 rows, B 256 rows
constexpr int F4_TX = A_BYTES + B_BYTES + F4_SFA + F4_SFB;
constexpr int F4_STAGE = (F4_TX + 1023) / 1024 * 1024;
constexpr int F4_BARS = F4_STAGES * F4_STAGE;
constexpr int F4_SMEM = F4_BARS + 256;
constexpr int F4_SLOT = 48;  // TMEM columns of one stage's scales (A 16, B 32)
static_assert(SF_COL + F4_STAGES * F4_SLOT <= TMEM_COLS, "NVFP4 scale slots exceed TMEM");
static_assert(F4_SMEM + 1024 <= 227 * 1024, "NVFP4 shared memory");
static_assert((3 * F4_STAGES + 5) * 8 <= 256, "NVFP4 barriers");

// E2M1 x E2M1 (format code 1 in both), UE4M3 scales (bit 23 clear), K-major.
__device__ __forceinline__ uint32_t idesc_nvf4(uint32_t M, uint32_t N) {
  return (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

__global__ void __launch_bounds__(THREADS + 32, 1)
    k_gemm_nvf4(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ GemmArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + F4_BARS);
  constexpr int S = F4_STAGES;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
  const uint32_t acc_full = smem_u32(bars + 2 * S), acc_empty = smem_u32(bars + 2 * S + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 2);
  const uint32_t sf_full0 = smem_u32(bars + 2 * S + 3);
  const uint32_t drain_mma = smem_u32(bars + 3 * S + 3), drain_sf = drain_mma + 8;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
      mbar_init(sf_full0 + 8 * s, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    mbar_init(drain_mma, 1);
    mbar_init(drain_sf, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < g.ntiles && ok; t += gridDim.x) {
        int b, tm, tn;
        tile_of(g, t, g.MTb, b, tm, tn);
        const int ga = b * g.MTb + tm, gb = b * g.b_step + 2 * tn;
        for (int kt = 0; kt < g.KT; ++kt) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, g.err, ERR_TIMEOUT_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t sbase = smem_u32(smem + stage * F4_STAGE);
          const uint32_t fb = full0 + 8 * stage;
          mbar_expect_tx(fb, F4_TX);
          tma_load_2d(sbase, &tma_a, kt * BK, ga * BM, fb);
          tma_load_2d(sbase + A_BYTES, &tma_b, kt * BK, gb * 128, fb);
          // scale atoms: [kt][row chunk][4 MMAs][512]
          bulk_load(sbase + A_BYTES + B_BYTES, g.sfa + ((size_t)kt * g.MT + ga) * F4_SFA, F4_SFA,
                    fb);
          bulk_load(sbase + A_BYTES + B_BYTES + F4_SFA,
                    g.sfb + ((size_t)kt * g.NT128 + gb) * (F4_SFB / 2), F4_SFB, fb);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      drain_loads<S>(full0, stage, phase, g.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t s0 = smem_u32(smem);
      const uint64_t dA0 = sw128_desc(s0), dB0 = sw128_desc(s0 + A_BYTES);
      const uint32_t id = idesc_nvf4(BM, BN);
      for (int t = blockIdx.x; t < g.ntiles && ok; t += gridDim.x) {
        if (!mbar_wait(acc_empty, acc_phase ^ 1, g.err, ERR_TIMEOUT_ACC)) break;
        acc_phase ^= 1;
        tc_fence_after();
        for (int kt = 0; kt < g.KT; ++kt) {
          if (!mbar_wait(sf_full0 + 8 * stage, phase, g.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t soff = stage * (F4_STAGE / 16);
          const uint32_t sfc = tmem + SF_COL + stage * F4_SLOT;
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t accum = (kt > 0 || j > 0) ? 1u : 0u;
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, "
                "%3, [%5], [%6], p;\n\t}" ::"r"(tmem + ACC_COL),
                "l"(desc_at(dA0, soff + 2 * j)), "l"(desc_at(dB0, soff + 2 * j)), "r"(id),
                "r"(accum), "r"(sfc + 4 * j), "r"(sfc + 16 + 8 * j));
          }
          asm volatile(
              "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                  empty0 + 8 * stage)
              : "memory");
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        asm volatile(
            "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                acc_full)
            : "memory");
      }
      tc_commit(drain_mma);
      mbar_wait(drain_mma, 0, g.err, ERR_TIMEOUT_DRAIN);
    }
  } else if (warp == 10) {
    // ---------------- scale-copy issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t dS0 = sf_desc(smem_u32(smem) + A_BYTES + B_BYTES);
      for (int t = blockIdx.x; t < g.ntiles && ok; t += gridDim.x) {
        for (int kt = 0; kt < g.KT; ++kt) {
          if (!mbar_wait(full0 + 8 * stage, phase, g.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t soff = stage * (F4_STAGE / 16);
          const uint32_t sfc = tmem + SF_COL + stage * F4_SLOT;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // A: MMA j's atom; B: MMA j's atoms of both 128-row chunks
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfc + 4 * j),
                         "l"(desc_at(dS0, soff + (j * 512) / 16)));
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sfc + 16 + 8 * j),
                         "l"(desc_at(dS0, soff + (F4_SFA + j * 512) / 16)));
            asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(
                             sfc + 16 + 8 * j + 4),
                         "l"(desc_at(dS0, soff + (F4_SFA + 2048 + j * 512) / 16)));
          }
          asm volatile(
              "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                  sf_full0 + 8 * stage)
              : "memory");
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      tc_commit(drain_sf);
      mbar_wait(drain_sf, 0, g.err, ERR_TIMEOUT_DRAIN);
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < g.ntiles; t += gridDim.x) {
      int b, tm, tn;
      tile_of(g, t, g.MTb, b, tm, tn);
      if (!mbar_wait_warp(acc_full, acc_phase, g.err, ERR_TIMEOUT_ACC)) break;
      acc_phase ^= 1;
      tc_fence_after();
      const int row = tm * BM + row_in_tile;
      const int colh = tn * BN + half * 128;
      epilogue_tile(g, tmem, q, half, lane, b, row, colh, [&] { mbar_arrive(acc_empty); });
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// NVFP4 packing: bf16 E2M1 codes [R, K] -> nibbles [RT * 128][KT * 128 bytes]
// (element 2i in the low nibble); one thread per 32 codes (16 bytes out).
struct PackF4Args {
  const uint16_t* codes;  // bf16 [R, K]
  const uint16_t* scale;  // bf16 [R, K / 16]
  uint8_t* out;
  uint8_t* sf;            // [KT][RT][4][512]
  int R, K, KT, RT, nkb;
  int* inexact;
};

__global__ void k_pack_nvf4_codes(const __grid_constant__ PackF4Args p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = p.KT * 8;  // 16-byte pieces per packed row (256 elements per K tile)
  if (i >= (int64_t)p.RT * 128 * per_row) return;
  const int r = (int)(i / per_row), c0 = (int)(i % per_row) * 32;
  uint32_t w[4] = {0, 0, 0, 0};
  int bad = 0;
  if (r < p.R) {
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      const int c = c0 + k;
      float f0 = 0.f, f1 = 0.f;
      if (c < p.K) f0 = bf2f(p.codes[(int64_t)r * p.K + c]);
      if (c + 1 < p.K) f1 = bf2f(p.codes[(int64_t)r * p.K + c + 1]);
      uint32_t b;
      asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
          : "=r"(b)
          : "f"(f1), "f"(f0));
      uint32_t h2;
      asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
          : "=r"(h2)
          : "r"(b));
      const float g0 = __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFF)));
      const float g1 = __half2float(__ushort_as_half((unsigned short)(h2 >> 16)));
      bad += (__float_as_uint(g0) != __float_as_uint(f0) && !(g0 == 0.f && f0 == 0.f));
      bad += (__float_as_uint(g1) != __float_as_uint(f1) && !(g1 == 0.f && f1 == 0.f));
      w[k / 8] |= b << (8 * ((k / 2) & 3));
    }
  }
  *reinterpret_cast<uint4*>(p.out + (int64_t)r * (p.KT * 128) + c0 / 2) =
      make_uint4(w[0], w[1], w[2], w[3]);
  if (bad && p.inexact) atomicAdd(p.inexact, bad);
}

// One thread per (row, block of 16): the UE4M3 byte of its scale.
__global__ void k_pack_nvf4_scales(const __grid_constant__ PackF4Args p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int kb_all = p.KT * 16;
  if (i >= (int64_t)p.RT * 128 * kb_all) return;
  const int r = (int)(i / kb_all), kb = (int)(i % kb_all);
  uint32_t e = 0x38;  // 1.0 for padding rows / blocks
  int bad = 0;
  if (r < p.R && kb < p.nkb) {
    const float s = bf2f(p.scale[(int64_t)r * p.nkb + kb]);
    uint16_t pair;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pair) : "f"(0.0f), "f"(s));
    e = pair & 0xFFu;
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((uint16_t)e));
    const float back = __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFF)));
    // a positive E4M3 value (UE4M3 has no sign) that round-trips exactly
    bad = !(s > 0.0f) || __float_as_uint(back) != __float_as_uint(s);
  }
  const int kt = kb / 16, j = (kb % 16) / 4, t = kb % 4, rt = r / 128, rr = r % 128;
  p.sf[(((int64_t)kt * p.RT + rt) * 4 + j) * 512 + (rr % 32) * 16 + (rr / 32) * 4 + t] = (uint8_t)e;
  if (bad && p.inexact) atomicAdd(p.inexact, 1);
}

// ---------------------------------------------------------------------------
// Packing: bf16 E4M3 codes -> bytes, bf16 power-of-two scales -> UE8M0 atoms
// ---------------------------------------------------------------------------
struct PackArgs {
  const uint16_t* codes;  // bf16 [R, K] (or, batched, element strides below)
  const uint16_t* scale;  // bf16 [R, nkb]
  uint8_t* out;           // [R_pad, Kp]
  uint8_t* sf;            // [KT][RT][512]
  int R, K, Kp, nkb, RT, KT;
  int* inexact;           // count of codes / scales not representable (may be null)
  // batched / transposed sources: batch b's R rows are packed rows
  // [b * RTb * 128, ...); element (b, r, k) of the codes at b * cb + r * cr +
  // k * ck, scale (b, r, kb) at b * sb + r * sr + kb * sk; RT = batch * RTb
  int batch, RTb;
  int64_t cb, cr, ck, sb, sr, sk;
};

// One thread: 16 codes of a row (16 bytes out); rows of every batch
// (row-major K: batch b's source rows at b * cb, row stride cr).
__global__ void k_pack_codes(const __grid_constant__ PackArgs p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = p.Kp / 16;
  const int64_t total = (int64_t)p.RT * 128 * per_row;
  if (i >= total) return;
  const int64_t rg = i / per_row;  // packed row over all batches
  const int c0 = (int)(i % per_row) * 16;
  const int b = (int)(rg / (p.RTb * 128)), r = (int)(rg % (p.RTb * 128));
  uint32_t w[4] = {0, 0, 0, 0};
  int bad = 0;
  if (r < p.R) {
    const uint16_t* src = p.codes + (int64_t)b * p.cb + (int64_t)r * p.cr;
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
      const int c = c0 + k;
      float f0 = 0.f, f1 = 0.f;
      if (c < p.K) f0 = bf2f(src[c]);
      if (c + 1 < p.K) f1 = bf2f(src[c + 1]);
      uint16_t b;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b) : "f"(f1), "f"(f0));
      // exact round trip check
      uint32_t h2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(b));
      const float g0 = __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFF)));
      const float g1 = __half2float(__ushort_as_half((unsigned short)(h2 >> 16)));
      bad += (__float_as_uint(g0) != __float_as_uint(f0) && !(g0 == 0.f && f0 == 0.f));
      bad += (__float_as_uint(g1) != __float_as_uint(f1) && !(g1 == 0.f && f1 == 0.f));
      w[k / 4] |= (uint32_t)b << (16 * ((k / 2) & 1));
    }
  }
  *reinterpret_cast<uint4*>(p.out + rg * p.Kp + c0) = make_uint4(w[0], w[1], w[2], w[3]);
  if (bad && p.inexact) atomicAdd(p.inexact, bad);
}

// One thread per (row, K block of 32): the UE8M0 byte in its atom.
__global__ void k_pack_scales(const __grid_constant__ PackArgs p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int kb_all = p.KT * 4;
  const int64_t total = (int64_t)p.RT * 128 * kb_all;
  if (i >= total) return;
  const int r = (int)(i / kb_all), kb = (int)(i % kb_all);
  uint8_t e = 127;  // 1.0 for padding rows / blocks
  int bad = 0;
  if (r < p.R && kb < p.nkb) {
    const uint32_t s = p.scale[(int64_t)r * p.nkb + kb];
    const uint32_t ex = (s >> 7) & 0xFF;
    // a positive normal power of two; UE8M0 holds 2^-127 .. 2^127
    bad = (s & 0x807Fu) != 0 || ex == 0 || ex == 0xFF;
    e = (uint8_t)(ex == 0 ? 0 : (ex == 0xFF ? 0xFE : ex));
  }
  const int kt = kb / 4, j = kb % 4, rt = r / 128, rr = r % 128;
  p.sf[((int64_t)kt * p.RT + rt) * 512 + (rr % 32) * 16 + (rr / 32) * 4 + j] = e;
  if (bad && p.inexact) atomicAdd(p.inexact, 1);
}

// Batched, transposed codes ([batch, K, R]: rows contiguous): one thread per
// (packed row, 16 codes along K), packed rows fastest so a warp's loads of
// each K index are contiguous.
__global__ void k_pack_codes_t(const __grid_constant__ PackArgs p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int rows_b = p.RTb * 128, per_row = p.Kp / 16;
  const int64_t total = (int64_t)p.batch * rows_b * per_row;
  if (i >= total) return;
  const int64_t rb = i % ((int64_t)p.batch * rows_b);  // packed row over all batches
  const int c0 = (int)(i / ((int64_t)p.batch * rows_b)) * 16;
  const int b = (int)(rb / rows_b), r = (int)(rb % rows_b);
  uint32_t w[4] = {0, 0, 0, 0};
  int bad = 0;
  if (r < p.R) {
    const uint16_t* src = p.codes + (int64_t)b * p.cb + (int64_t)r * p.cr;
#pragma unroll
    for (int k = 0; k < 16; k += 2) {
      const int c = c0 + k;
      float f0 = 0.f, f1 = 0.f;
      if (c < p.K) f0 = bf2f(src[(int64_t)c * p.ck]);
      if (c + 1 < p.K) f1 = bf2f(src[(int64_t)(c + 1) * p.ck]);
      uint16_t e;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(e) : "f"(f1), "f"(f0));
      uint32_t h2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(e));
      const float g0 = __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFF)));
      const float g1 = __half2float(__ushort_as_half((unsigned short)(h2 >> 16)));
      bad += (__float_as_uint(g0) != __float_as_uint(f0) && !(g0 == 0.f && f0 == 0.f));
      bad += (__float_as_uint(g1) != __float_as_uint(f1) && !(g1 == 0.f && f1 == 0.f));
      w[k / 4] |= (uint32_t)e << (16 * ((k / 2) & 1));
    }
  }
  *reinterpret_cast<uint4*>(p.out + rb * p.Kp + c0) = make_uint4(w[0], w[1], w[2], w[3]);
  if (bad && p.inexact) atomicAdd(p.inexact, bad);
}

// Batched scales at any strides: one thread per (packed row, K block), rows
// fastest; the UE8M0 byte of its atom ([KT][batch * RTb][512]).
__global__ void k_pack_scales_b(const __grid_constant__ PackArgs p) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int rows_b = p.RTb * 128;
  const int64_t rows = (int64_t)p.batch * rows_b;
  const int kb_all = p.KT * 4;
  if (i >= rows * kb_all) return;
  const int64_t rb = i % rows;
  const int kb = (int)(i / rows);
  const int b = (int)(rb / rows_b), r = (int)(rb % rows_b);
  uint8_t e = 127;  // 1.0 for padding rows / blocks
  int bad = 0;
  if (r < p.R && kb < p.nkb) {
    const uint32_t s = p.scale[(int64_t)b * p.sb + (int64_t)r * p.sr + (int64_t)kb * p.sk];
    const uint32_t ex = (s >> 7) & 0xFF;
    bad = (s & 0x807Fu) != 0 || ex == 0 || ex == 0xFF;
    e = (uint8_t)(ex == 0 ? 0 : (ex == 0xFF ? 0xFE : ex));
  }
  const int kt = kb / 4, j = kb % 4;
  const int64_t rt = rb / 128;
  const int rr = (int)(rb % 128);
  p.sf[((int64_t)kt * p.RT + rt) * 512 + (rr % 32) * 16 + (rr / 32) * 4 + j] = e;
  if (bad && p.inexact) atomicAdd(p.inexact, 1);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_bytes,
              uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols_bytes, rows};
  cuuint64_t strides[1] = {cols_bytes};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_plain(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols_bytes,
                    uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols_bytes, rows};
  cuuint64_t strides[1] = {cols_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// The CTA-pair kernel is used unless VQ_GEMM_PAIR=0 is set in the environment.
bool pair_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("VQ_GEMM_PAIR");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// ---------------------------------------------------------------------------
// Scratch for vq_linear_mxf8_noalloc: a file-scope device array, one copy per
// GPU that loads the library, held until the process exits.  Layout: the
// kernel's error word (first 256 bytes), then the packed activation codes,
// then their scale atoms.  Every call reuses it, so calls that overlap on
// the GPU (different streams, or graph replays in flight together) race.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_noalloc_scratch[VQ_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch, looked up once per device with that
// device current (host code may not use the symbol itself as an address).
uint8_t* noalloc_scratch_ptr(int* status) {
  static std::mutex mu;
  static uint8_t* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = VQ_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      *status = VQ_ERR_CUDA;
      return nullptr;
    }
    ptrs[dev] = static_cast<uint8_t*>(p);
  }
  *status = VQ_OK;
  return ptrs[dev];
}

// Launch of either GEMM kernel for `batch` problems (batch 1: one linear).
int gemm_run(const void* a, const void* a_sf, const void* b, const void* b_sf, int64_t batch,
             int64_t MTb, int64_t M, int64_t N, int64_t K, int b_shared, const void* bias,
             const void* residual, int64_t ldr, void* out, int64_t ldo, int64_t out_bs,
             int32_t out_multicast, int32_t* d_err, void* stream) {
  if (batch > 1 && (residual || out_multicast)) return VQ_ERR_UNSUPPORTED;
  if (out_multicast && residual) return VQ_ERR_UNSUPPORTED;
  if (!a || !a_sf || !b || !b_sf || !out || !d_err) return VQ_ERR_NULL;
  if (residual && (ldr < N || ldr % 8 || (reinterpret_cast<uintptr_t>(residual) & 15)))
    return VQ_ERR_UNSUPPORTED;
  if (M <= 0 || N <= 0 || K <= 0) return VQ_ERR_INVALID;
  if (N % 8 != 0 || ldo < N || ldo % 8 != 0) return VQ_ERR_UNSUPPORTED;
  if (M > (1 << 30) || N > (1 << 30)) return VQ_ERR_UNSUPPORTED;
  if (MTb * 128 < M || batch * MTb >= (1 << 24)) return VQ_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(a) & 15) ||
      (reinterpret_cast<uintptr_t>(b) & 15) || (reinterpret_cast<uintptr_t>(a_sf) & 15) ||
      (reinterpret_cast<uintptr_t>(b_sf) & 15))
    return VQ_ERR_ALIGNMENT;
  const int64_t KT = (K + 127) / 128, Kp = KT * 128;
  const int64_t MT = batch * MTb;  // 128-row A tiles over all batches
  // B is packed over 128-row chunks; a 256-wide tile reads two chunks, so
  // the packed B must hold an even number of chunks per batch (the caller pads).
  const int64_t NTILE_N = (N + BN - 1) / BN;
  const int64_t NT128 = (b_shared ? 1 : batch) * NTILE_N * 2;
  if (NT128 >= (1 << 24) || (int64_t)NTILE_N * MT >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  CUtensorMap ma, mb;
  if (!make_map(&ma, a, MT * 128, Kp, BM) || !make_map(&mb, b, NT128 * 128, Kp, BN))
    return VQ_ERR_CUDA;
  GemmArgs g;
  g.sfa = (const uint8_t*)a_sf;
  g.sfb = (const uint8_t*)b_sf;
  g.bias = (const uint16_t*)bias;
  g.residual = (const uint16_t*)residual;
  g.ldr = ldr;
  g.out = (uint16_t*)out;
  g.ldo = ldo;
  g.out_bs = out_bs;
  g.out_mc = out_multicast ? 1 : 0;
  g.M = (int)M;
  g.N = (int)N;
  g.KT = (int)KT;
  g.MT = (int)MT;
  g.NT128 = (int)NT128;
  g.NTILE_N = (int)NTILE_N;
  g.MTb = (int)MTb;
  g.MT2b = (int)((M + 255) / 256);
  g.b_step = b_shared ? 0 : (int)(NTILE_N * 2);
  g.ntiles = (int)(batch * MTb * NTILE_N);
  g.err = d_err;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(d_err, 0, sizeof(int32_t), st) != cudaSuccess) return VQ_ERR_CUDA;
  if (M >= 256 && pair_enabled()) {
    // CTA pairs: 256 x 256 tiles, B loaded in 128-row halves; scale atoms
    // through plain (unswizzled) maps of 256-byte rows
    CUtensorMap mbh, msa, msb;
    if (!make_map(&mbh, b, NT128 * 128, Kp, 128) ||
        !make_map_plain(&msa, a_sf, (uint64_t)KT * MT * 2, 256, 256, 2) ||
        !make_map_plain(&msb, b_sf, (uint64_t)KT * NT128 * 2, 256, 256, 4))
      return VQ_ERR_CUDA;
    GemmArgs gp = g;
    gp.ntiles = (int)(batch * g.MT2b * NTILE_N);
    const int smem = P_SMEM + 1024;
    if (cudaFuncSetAttribute(k_gemm_mxf8_pair, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return VQ_ERR_CUDA;
    const int pairs = (int)std::min<int64_t>(gp.ntiles, sm_count() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(P_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_gemm_mxf8_pair, ma, mbh, msa, msb, gp) != cudaSuccess)
      return VQ_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
  }
  const int smem = SmemLayout::kTotal + 1024;
  if (cudaFuncSetAttribute(k_gemm_mxf8, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return VQ_ERR_CUDA;
  const int grid = (int)std::min<int64_t>(g.ntiles, sm_count());
  k_gemm_mxf8<<<grid, THREADS + 32, smem, st>>>(ma, mb, g);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}


}  // namespace mx
namespace attn {
int sticky_attn(int* out, int clear, cudaStream_t st);
}
namespace tp {
int sticky_tp(int* out, int clear, cudaStream_t st);
}
namespace dq {
int sticky_dq(int* out, int clear, cudaStream_t st);
}
namespace w4 {
int sticky_w4(int* out, int clear, cudaStream_t st);
}
}  // namespace vq

using namespace vq::mx;

extern "C" {

int vq_mx_pack_sizes(int64_t rows, int64_t k, int32_t row_multiple, int64_t* codes_bytes,
                     int64_t* sf_bytes, int64_t* ld_bytes) {
  if (rows < 0 || k <= 0 || !codes_bytes || !sf_bytes || !ld_bytes) return VQ_ERR_INVALID;
  if (row_multiple != 128 && row_multiple != 256) return VQ_ERR_INVALID;
  const int64_t RT = (rows + row_multiple - 1) / row_multiple * (row_multiple / 128);
  const int64_t KT = (k + 127) / 128;
  *ld_bytes = KT * 128;
  *codes_bytes = RT * 128 * KT * 128;
  *sf_bytes = KT * RT * 512;
  return VQ_OK;
}

int vq_mx_pack(const vq_tensor* codes, const vq_tensor* scale, int64_t block_size,
               int32_t row_multiple, void* packed_codes, void* packed_sf, int32_t* d_inexact,
               void* stream) {
  if (!codes || !scale || !packed_codes || !packed_sf) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || scale->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (block_size != 32) return VQ_ERR_UNSUPPORTED;
  if (codes->ndim != 2 || scale->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t R = codes->shape[0], K = codes->shape[1];
  if (scale->shape[0] != R || scale->shape[1] != (K + 31) / 32) return VQ_ERR_SHAPE;
  if (R <= 0 || K <= 0) return VQ_ERR_INVALID;
  if (row_multiple != 128 && row_multiple != 256) return VQ_ERR_INVALID;
  if (R >= (1ll << 31) / 4 || K >= (1 << 24)) return VQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(packed_codes) & 15) || (reinterpret_cast<uintptr_t>(packed_sf) & 15))
    return VQ_ERR_ALIGNMENT;
  PackArgs p;
  p.codes = (const uint16_t*)codes->data;
  p.scale = (const uint16_t*)scale->data;
  p.out = (uint8_t*)packed_codes;
  p.sf = (uint8_t*)packed_sf;
  p.R = (int)R;
  p.K = (int)K;
  p.RT = (int)((R + row_multiple - 1) / row_multiple * (row_multiple / 128));
  p.KT = (int)((K + 127) / 128);
  p.Kp = p.KT * 128;
  p.nkb = (int)((K + 31) / 32);
  p.inexact = d_inexact;
  p.batch = 1;
  p.RTb = p.RT;
  p.cb = 0, p.cr = K, p.ck = 1, p.sb = 0, p.sr = p.nkb, p.sk = 1;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_inexact && cudaMemsetAsync(d_inexact, 0, sizeof(int32_t), st) != cudaSuccess)
    return VQ_ERR_CUDA;
  const int64_t n1 = (int64_t)p.RT * 128 * (p.Kp / 16);
  k_pack_codes<<<(unsigned)((n1 + 255) / 256), 256, 0, st>>>(p);
  const int64_t n2 = (int64_t)p.RT * 128 * p.KT * 4;
  k_pack_scales<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_mx_pack_batched(const vq_tensor* codes, const vq_tensor* scale, int64_t block_size,
                       int32_t row_multiple, int32_t k_axis, void* packed_codes, void* packed_sf,
                       int32_t* d_inexact, void* stream) {
  if (!codes || !scale || !packed_codes || !packed_sf) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || scale->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (block_size != 32) return VQ_ERR_UNSUPPORTED;
  if (codes->ndim != 3 || scale->ndim != 3) return VQ_ERR_SHAPE;
  if (k_axis != 1 && k_axis != 2) return VQ_ERR_INVALID;
  if (row_multiple != 128 && row_multiple != 256) return VQ_ERR_INVALID;
  const int64_t B = codes->shape[0];
  const int64_t R = k_axis == 2 ? codes->shape[1] : codes->shape[2];
  const int64_t K = k_axis == 2 ? codes->shape[2] : codes->shape[1];
  const int64_t nkb = (K + 31) / 32;
  if (scale->shape[0] != B) return VQ_ERR_SHAPE;
  if (k_axis == 2 && (scale->shape[1] != R || scale->shape[2] != nkb)) return VQ_ERR_SHAPE;
  if (k_axis == 1 && (scale->shape[1] != nkb || scale->shape[2] != R)) return VQ_ERR_SHAPE;
  if (B <= 0 || R <= 0 || K <= 0) return VQ_ERR_INVALID;
  const int64_t RTb = (R + row_multiple - 1) / row_multiple * (row_multiple / 128);
  if (B * RTb * 128 >= (1ll << 31) / 4 || K >= (1 << 24)) return VQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(packed_codes) & 15) || (reinterpret_cast<uintptr_t>(packed_sf) & 15))
    return VQ_ERR_ALIGNMENT;
  PackArgs p;
  p.codes = (const uint16_t*)codes->data;
  p.scale = (const uint16_t*)scale->data;
  p.out = (uint8_t*)packed_codes;
  p.sf = (uint8_t*)packed_sf;
  p.R = (int)R;
  p.K = (int)K;
  p.KT = (int)((K + 127) / 128);
  p.Kp = p.KT * 128;
  p.nkb = (int)nkb;
  p.batch = (int)B;
  p.RTb = (int)RTb;
  p.RT = (int)(B * RTb);
  p.inexact = d_inexact;
  p.cb = R * K;
  p.sb = R * nkb;
  if (k_axis == 2) {
    p.cr = K, p.ck = 1, p.sr = nkb, p.sk = 1;
  } else {
    p.cr = 1, p.ck = R, p.sr = 1, p.sk = R;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_inexact && cudaMemsetAsync(d_inexact, 0, sizeof(int32_t), st) != cudaSuccess)
    return VQ_ERR_CUDA;
  if (k_axis == 2) {
    const int64_t n1 = B * RTb * 128 * (p.Kp / 16);
    k_pack_codes<<<(unsigned)((n1 + 255) / 256), 256, 0, st>>>(p);
  } else {
    const int64_t n1 = B * RTb * 128 * (p.Kp / 16);
    k_pack_codes_t<<<(unsigned)((n1 + 255) / 256), 256, 0, st>>>(p);
  }
  const int64_t n2 = B * RTb * 128 * p.KT * 4;
  k_pack_scales_b<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_gemm_mxf8(const void* a, const void* a_sf, const void* b, const void* b_sf, int64_t M,
                 int64_t N, int64_t K, const void* bias, void* out, int64_t ldo, int32_t* d_err,
                 void* stream) {
  return vq_gemm_mxf8_ex(a, a_sf, b, b_sf, M, N, K, bias, nullptr, 0, out, ldo, 0, d_err,
                         stream);
}

int vq_gemm_mxf8_ex(const void* a, const void* a_sf, const void* b, const void* b_sf, int64_t M,
                    int64_t N, int64_t K, const void* bias, const void* residual, int64_t ldr,
                    void* out, int64_t ldo, int32_t out_multicast, int32_t* d_err,
                    void* stream) {
  return gemm_run(a, a_sf, b, b_sf, 1, (M + 127) / 128, M, N, K, 0, bias, residual, ldr, out, ldo,
                  0, out_multicast, d_err, stream);
}

int vq_gemm_mxf8_batched(const void* a, const void* a_sf, const void* b, const void* b_sf,
                         int64_t batch, int64_t a_rows_per_batch, int64_t M, int64_t N, int64_t K,
                         int32_t b_shared, const void* bias, void* out, int64_t ldo,
                         int64_t out_batch_stride, int32_t* d_err, void* stream) {
  if (batch <= 0 || a_rows_per_batch <= 0 || a_rows_per_batch % 128) return VQ_ERR_INVALID;
  if (a_rows_per_batch < M || out_batch_stride < 0) return VQ_ERR_INVALID;
  if (batch > 1 && out_batch_stride < M * ldo) return VQ_ERR_INVALID;
  if (out_batch_stride % 8) return VQ_ERR_ALIGNMENT;
  return gemm_run(a, a_sf, b, b_sf, batch, a_rows_per_batch / 128, M, N, K, b_shared ? 1 : 0, bias,
                  nullptr, 0, out, ldo, out_batch_stride, 0, d_err, stream);
}

int vq_nvf4_pack_sizes(int64_t rows, int64_t k, int32_t row_multiple, int64_t* codes_bytes,
                       int64_t* sf_bytes) {
  if (rows <= 0 || k <= 0 || !codes_bytes || !sf_bytes) return VQ_ERR_INVALID;
  if (row_multiple != 128 && row_multiple != 256) return VQ_ERR_INVALID;
  const int64_t RT = (rows + row_multiple - 1) / row_multiple * (row_multiple / 128);
  const int64_t KT = (k + 255) / 256;
  *codes_bytes = RT * 128 * KT * 128;
  *sf_bytes = KT * RT * 4 * 512;
  return VQ_OK;
}

int vq_nvf4_pack(const vq_tensor* codes, const vq_tensor* scale, int32_t row_multiple,
                 void* packed_codes, void* packed_sf, int32_t* d_inexact, void* stream) {
  if (!codes || !scale || !packed_codes || !packed_sf) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || scale->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (codes->ndim != 2 || scale->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t R = codes->shape[0], K = codes->shape[1];
  if (R <= 0 || K <= 0) return VQ_ERR_INVALID;
  if (scale->shape[0] != R || scale->shape[1] != (K + 15) / 16) return VQ_ERR_SHAPE;
  if (row_multiple != 128 && row_multiple != 256) return VQ_ERR_INVALID;
  if (R >= (1ll << 31) / 4 || K >= (1 << 24)) return VQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(packed_codes) & 15) || (reinterpret_cast<uintptr_t>(packed_sf) & 15))
    return VQ_ERR_ALIGNMENT;
  PackF4Args p;
  p.codes = (const uint16_t*)codes->data;
  p.scale = (const uint16_t*)scale->data;
  p.out = (uint8_t*)packed_codes;
  p.sf = (uint8_t*)packed_sf;
  p.R = (int)R;
  p.K = (int)K;
  p.KT = (int)((K + 255) / 256);
  p.RT = (int)((R + row_multiple - 1) / row_multiple * (row_multiple / 128));
  p.nkb = (int)((K + 15) / 16);
  p.inexact = d_inexact;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_inexact && cudaMemsetAsync(d_inexact, 0, sizeof(int32_t), st) != cudaSuccess)
    return VQ_ERR_CUDA;
  const int64_t n1 = (int64_t)p.RT * 128 * p.KT * 8;
  k_pack_nvf4_codes<<<(unsigned)((n1 + 255) / 256), 256, 0, st>>>(p);
  const int64_t n2 = (int64_t)p.RT * 128 * p.KT * 16;
  k_pack_nvf4_scales<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_gemm_nvf4(const void* a, const void* a_sf, const void* b, const void* b_sf, int64_t M,
                 int64_t N, int64_t K, const void* bias, void* out, int64_t ldo, int32_t* d_err,
                 void* stream) {
  if (!a || !a_sf || !b || !b_sf || !out || !d_err) return VQ_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0) return VQ_ERR_INVALID;
  if (N % 8 != 0 || ldo < N || ldo % 8 != 0) return VQ_ERR_UNSUPPORTED;
  if (M > (1 << 30) || N > (1 << 30) || K >= (1 << 24)) return VQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(a) & 15) ||
      (reinterpret_cast<uintptr_t>(b) & 15) || (reinterpret_cast<uintptr_t>(a_sf) & 15) ||
      (reinterpret_cast<uintptr_t>(b_sf) & 15) || (reinterpret_cast<uintptr_t>(bias) & 1))
    return VQ_ERR_ALIGNMENT;
  const int64_t KT = (K + 255) / 256, Kb = KT * 128;  // packed bytes per row
  const int64_t MT = (M + 127) / 128, NTILE_N = (N + BN - 1) / BN;
  if (NTILE_N * MT >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  CUtensorMap ma, mb;
  if (!make_map(&ma, a, MT * 128, Kb, BM) || !make_map(&mb, b, NTILE_N * 2 * 128, Kb, BN))
    return VQ_ERR_CUDA;
  GemmArgs g = {};
  g.sfa = (const uint8_t*)a_sf;
  g.sfb = (const uint8_t*)b_sf;
  g.bias = (const uint16_t*)bias;
  g.out = (uint16_t*)out;
  g.ldo = ldo;
  g.M = (int)M;
  g.N = (int)N;
  g.KT = (int)KT;
  g.MT = (int)MT;
  g.NT128 = (int)(NTILE_N * 2);
  g.NTILE_N = (int)NTILE_N;
  g.MTb = (int)MT;
  g.MT2b = (int)((M + 255) / 256);
  g.b_step = 0;
  g.ntiles = (int)(MT * NTILE_N);
  g.err = d_err;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(d_err, 0, sizeof(int32_t), st) != cudaSuccess) return VQ_ERR_CUDA;
  const int smem = F4_SMEM + 1024;
  if (cudaFuncSetAttribute(k_gemm_nvf4, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return VQ_ERR_CUDA;
  const int grid = (int)std::min<int64_t>(g.ntiles, sm_count());
  k_gemm_nvf4<<<grid, THREADS + 32, smem, st>>>(ma, mb, g);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_linear_mxf8_noalloc(const vq_tensor* a_codes, const vq_tensor* a_scale,
                           const void* w_packed, const void* w_sf_packed, int64_t N,
                           const void* bias, void* out, int64_t ldo, void* stream) {
  if (!a_codes || !a_scale || !w_packed || !w_sf_packed || !out) return VQ_ERR_NULL;
  if (a_codes->dtype != VQ_BF16 || a_scale->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (a_codes->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t M = a_codes->shape[0], K = a_codes->shape[1];
  if (M <= 0 || K <= 0 || N <= 0) return VQ_ERR_INVALID;
  // everything the GEMM would reject is rejected here, before the packing
  // overwrites the shared scratch
  if (N % 8 != 0 || ldo < N || ldo % 8 != 0 || M > (1 << 30) || N > (1 << 30))
    return VQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(w_packed) & 15) ||
      (reinterpret_cast<uintptr_t>(w_sf_packed) & 15) || (reinterpret_cast<uintptr_t>(bias) & 1))
    return VQ_ERR_ALIGNMENT;
  int64_t cb = 0, sb = 0, ld = 0;
  int st = vq_mx_pack_sizes(M, K, 128, &cb, &sb, &ld);
  if (st) return st;
  // error word, packed codes, scale atoms; each region 256-byte aligned
  const int64_t codes_off = 256, sf_off = codes_off + (cb + 255) / 256 * 256;
  if (sf_off + sb > (int64_t)VQ_NOALLOC_SCRATCH_BYTES) return VQ_ERR_TOO_LARGE;
  uint8_t* base = noalloc_scratch_ptr(&st);
  if (!base) return st;
  int32_t* err = reinterpret_cast<int32_t*>(base);
  if ((st = vq_mx_pack(a_codes, a_scale, 32, 128, base + codes_off, base + sf_off, nullptr,
                       stream)))
    return st;
  return vq_gemm_mxf8(base + codes_off, base + sf_off, w_packed, w_sf_packed, M, N, K, bias, out,
                      ldo, err, stream);
}

int vq_linear_mxf8_noalloc_status(int32_t* code, void* stream) {
  if (!code) return VQ_ERR_NULL;
  int st = VQ_OK;
  uint8_t* base = noalloc_scratch_ptr(&st);
  if (!base) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, base, sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return VQ_ERR_CUDA;
  *code = v;
  return VQ_OK;
}

int vq_device_errors(int32_t* code, int32_t clear, void* stream) {
  if (!code) return VQ_ERR_NULL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v[5] = {0, 0, 0, 0, 0};
  if (vq::tc::sticky_read(&v[0], clear, s) || vq::dq::sticky_dq(&v[1], clear, s) ||
      vq::tp::sticky_tp(&v[2], clear, s) || vq::attn::sticky_attn(&v[3], clear, s) ||
      vq::w4::sticky_w4(&v[4], clear, s))
    return VQ_ERR_CUDA;
  // the first nonzero word: MXFP8 GEMM 1-4, bf16 GEMM 11-14, W4A8 21-23,
  // tensor-parallel barrier 100 + rank, attention 200 + its code
  *code = v[0] ? v[0] : (v[1] ? v[1] : (v[4] ? v[4] : (v[2] ? v[2] : (v[3] ? 200 + v[3] : 0))));
  return VQ_OK;
}

}  // extern "C"
