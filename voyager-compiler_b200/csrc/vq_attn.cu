// Fused MXFP8 attention on the tcgen05 tensor cores: quantized_ops::sdpa_mx
// (src/voyager_compiler/ops/quantized.py:651-784) for E4M3 query / key /
// value codes with power-of-two block-32 scales along their contraction axes
// and probabilities quantized to MXFP8 along the keys:
//
//   scores = bf16(bf16(Q . K^T) * scale)        (masked: -inf past the diagonal)
//   probs  = bf16(softmax(scores))               (float32 statistics)
//   (sP, cP) = quantize_mx(probs, E4M3, [-1], 32, quant_max, pow2 scales)
//   out    = bf16((cP * sP) . V)
//
// which is also the eager graph matmul_mx -> * scale -> + causal mask ->
// softmax -> quantize_mx -> matmul_mx of a converted LLaMA attention.
//
// Operands come packed (the layout vq_mx_pack / vq_quantize_mx_packed write):
//   Q   E4M3 bytes [B*H*Sq, 128], scale atoms [B*H*Sq/128][512]
//   K   E4M3 bytes [B*Hkv*Skv, 128], atoms [B*Hkv*Skv/128][512]
//   V^T E4M3 bytes [B*Hkv*128, Skv] (head_dim rows, keys contiguous),
//       atoms [Skv/128][B*Hkv][512]
// head_dim = 128; Sq and Skv multiples of 128.
//
// One work item = one (batch*head, 128-query tile), heaviest first under a
// causal mask; persistent CTAs (one per SM) take items round-robin.  Two
// passes over the key tiles of an item:
//   pass 1  S = Q K^T per key tile into TMEM; the softmax warps take the row
//           max and the running sum of exp (float32, online rescaling);
//   pass 2  S again; the softmax warps write P = bf16(exp(s - m) / l) as
//           E4M3 codes + UE8M0 block scales into shared memory in the MMA's
//           operand layout, and the MMA warp accumulates O += P . V in TMEM.
// Since P is final after pass 1, O needs no rescaling.
//
// Warps: 0 TMA producer (Q double-buffered, K / V^T tiles through a 6-slot
// ring), 1 TMEM owner + single-thread MMA issuer, 2-17 softmax (four warps
// per TMEM lane quarter, each on 32 of the 128 columns: one block of 32
// probabilities per thread and tile).  Every wait is bounded
// and sets *err when it gives up; no TMA multicast.
//
// exp is evaluated as ex2.approx.ftz(s * log2 e - m * log2 e); a block of 32
// probabilities whose largest value is below 2^-108 is given code 0 (the
// flush-to-zero exp and the subnormal block scales live there): its share
// of an output row is below 2^-90 of the row's largest probability, which
// is at least 1 / keys.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "vq_numerics.cuh"
#include "vq_tc.cuh"

namespace vq {
namespace attn {

using namespace vq::tc;

constexpr int TILE_BYTES = 128 * 128;  // one E4M3 tile (128 rows x 128 bytes)
constexpr int SF_BYTES = 512;          // one UE8M0 scale atom (128 rows x 4 blocks)
constexpr int SLOT = 17408;            // tile + atom, 1024-aligned
constexpr int RING = 6;
constexpr int SM_WARPS = 16;           // softmax warps
constexpr int NG = SM_WARPS / 4;       // column groups of 32 per TMEM lane quarter
constexpr int SMT = 32 * SM_WARPS;     // softmax threads
constexpr int THREADS = 64 + SMT;

constexpr int OFF_Q = 0;                         // 2 slots
constexpr int OFF_RING = 2 * SLOT;               // RING slots
constexpr int OFF_P = (2 + RING) * SLOT;         // 2 slots
constexpr int OFF_BAR = (4 + RING) * SLOT;
constexpr int OFF_STATS = OFF_BAR + 256;         // float2 [2 items][NG groups][128 rows]
constexpr int SMEM_TOTAL = OFF_STATS + 2 * NG * 128 * 8;

// barrier indices
constexpr int B_RFULL = 0, B_REMPTY = RING, B_QFULL = 2 * RING, B_QEMPTY = B_QFULL + 2,
              B_SFULL = B_QEMPTY + 2, B_SEMPTY = B_SFULL + 2, B_PFULL = B_SEMPTY + 2,
              B_PEMPTY = B_PFULL + 2, B_OFULL = B_PEMPTY + 2, B_OEMPTY = B_OFULL + 1,
              B_STATS = B_OEMPTY + 1, B_DRAIN = B_STATS + 2, NBARS = B_DRAIN + 1;
static_assert(NBARS * 8 + 8 <= 256, "barrier area");

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0;    // two 128-column score buffers
constexpr uint32_t COL_O = 256;  // 128 columns
constexpr uint32_t COL_SFQ = 384, COL_SFK = 388, COL_SFP = 392, COL_SFV = 396;

enum { ERR_RING_FULL = 1, ERR_RING_EMPTY, ERR_Q, ERR_S, ERR_P, ERR_O, ERR_STATS };

struct AttnArgs {
  const uint8_t* q_sf;
  const uint8_t* k_sf;
  const uint8_t* v_sf;
  uint16_t* out;             // bf16, element strides below; head_dim contiguous
  int64_t os_b, os_h, os_s;
  int B, H, HKV, SQ, SKV;
  int QT, KVT, n_items;
  float scale;
  int fl2q;
  int causal;
  int* err;
};

__device__ __forceinline__ void item_coords(const AttnArgs& a, int t, int& bh, int& qt, int& nkv) {
  const int BH = a.B * a.H;
  const int r = t / BH;
  bh = t % BH;
  qt = a.causal ? a.QT - 1 - r : r;  // heaviest first
  nkv = a.causal ? min(qt + 1, a.KVT) : a.KVT;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t bf2_rn(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}
// 2^x, one MUFU op; results below 2^-126 flush to zero
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float L2E = 1.4426950408889634f;

// 32 score columns of one row -> 16 packed bf16 pairs of
// bf16(bf16(acc) * scale), -inf where the key lies past the query.
__device__ __forceinline__ void scores_bf16(const uint32_t (&v)[32], float scale, int key0,
                                            int q_idx, bool diag, uint32_t (&tb)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t s2 = bf2_rn(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
    uint32_t t2 = bf2_rn(bf_lo(s2) * scale, bf_hi(s2) * scale);
    if (diag) {
      if (key0 + 2 * i > q_idx) t2 = (t2 & 0xFFFF0000u) | 0xFF80u;
      if (key0 + 2 * i + 1 > q_idx) t2 = (t2 & 0x0000FFFFu) | 0xFF800000u;
    }
    tb[i] = t2;
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    k_attn_mxf8(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_v, const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  float2* stats = reinterpret_cast<float2*>(smem + OFF_STATS);
  const uint32_t sbase = smem_u32(smem);
  auto bar = [&](int i) { return smem_u32(bars + i); };

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < RING; ++i) {
      mbar_init(bar(B_RFULL + i), 1);
      mbar_init(bar(B_REMPTY + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(B_QFULL + i), 1);
      mbar_init(bar(B_QEMPTY + i), 1);
      mbar_init(bar(B_SFULL + i), 1);
      mbar_init(bar(B_SEMPTY + i), SMT);
      mbar_init(bar(B_PFULL + i), SMT);
      mbar_init(bar(B_PEMPTY + i), 1);
      mbar_init(bar(B_STATS + i), SMT);
    }
    mbar_init(bar(B_OFULL), 1);
    mbar_init(bar(B_OEMPTY), SMT);
    mbar_init(bar(B_DRAIN), 1);
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
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_v)) : "memory");
      int st = 0, qb = 0;
      uint32_t ph = 0, qph = 0;
      bool ok = true;
      auto slot_wait = [&]() -> uint32_t {
        if (!mbar_wait(bar(B_REMPTY + st), ph ^ 1, a.err, ERR_RING_EMPTY)) return 0;
        return sbase + OFF_RING + st * SLOT;
      };
      auto advance = [&]() {
        if (++st == RING) {
          st = 0;
          ph ^= 1;
        }
      };
      for (int t = blockIdx.x; t < a.n_items && ok; t += gridDim.x) {
        int bh, qt, nkv;
        item_coords(a, t, bh, qt, nkv);
        const int bhkv = (bh / a.H) * a.HKV + (bh % a.H) / (a.H / a.HKV);
        if (!mbar_wait(bar(B_QEMPTY + qb), qph ^ 1, a.err, ERR_Q)) break;
        const uint32_t sq = sbase + OFF_Q + qb * SLOT;
        const int qrow = bh * a.SQ + qt * 128;
        mbar_expect_tx(bar(B_QFULL + qb), TILE_BYTES + SF_BYTES);
        tma_load_2d(sq, &map_q, 0, qrow, bar(B_QFULL + qb));
        bulk_load(sq + TILE_BYTES, a.q_sf + (size_t)(qrow / 128) * 512, SF_BYTES, bar(B_QFULL + qb));
        if (++qb == 2) {
          qb = 0;
          qph ^= 1;
        }
        auto load_k = [&](int kt) -> bool {
          const uint32_t s = slot_wait();
          if (!s) return false;
          const int krow = bhkv * a.SKV + kt * 128;
          mbar_expect_tx(bar(B_RFULL + st), TILE_BYTES + SF_BYTES);
          tma_load_2d(s, &map_k, 0, krow, bar(B_RFULL + st));
          bulk_load(s + TILE_BYTES, a.k_sf + (size_t)(krow / 128) * 512, SF_BYTES, bar(B_RFULL + st));
          advance();
          return true;
        };
        auto load_v = [&](int kt) -> bool {
          const uint32_t s = slot_wait();
          if (!s) return false;
          mbar_expect_tx(bar(B_RFULL + st), TILE_BYTES + SF_BYTES);
          tma_load_2d(s, &map_v, kt * 128, bhkv * 128, bar(B_RFULL + st));
          bulk_load(s + TILE_BYTES, a.v_sf + ((size_t)kt * (a.B * a.HKV) + bhkv) * 512, SF_BYTES,
                    bar(B_RFULL + st));
          advance();
          return true;
        };
        for (int kt = 0; kt < nkv && ok; ++kt) ok = load_k(kt);
        if (ok) ok = load_k(0);
        for (int kt = 0; kt < nkv && ok; ++kt) {
          if (kt + 1 < nkv) ok = load_k(kt + 1);
          if (ok) ok = load_v(kt);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int st = 0, sb = 0, pb = 0, qb = 0;
      uint32_t ph = 0, sph = 0, pph = 0, qph = 0, oph = 0;
      bool ok = true;
      const uint32_t idesc0 = idesc_mxf8(0, 128, 128), idesc1 = idesc_mxf8(1, 128, 128),
                     idesc2 = idesc_mxf8(2, 128, 128), idesc3 = idesc_mxf8(3, 128, 128);
      const uint32_t idescs[4] = {idesc0, idesc1, idesc2, idesc3};
      for (int t = blockIdx.x; t < a.n_items && ok; t += gridDim.x) {
        int bh, qt, nkv;
        item_coords(a, t, bh, qt, nkv);
        if (!mbar_wait(bar(B_QFULL + qb), qph, a.err, ERR_Q)) break;
        tc_fence_after();
        const uint32_t sq = sbase + OFF_Q + qb * SLOT;
        cp_sf(tmem + COL_SFQ, sq + TILE_BYTES);
        // S[sb] = Q . K^T of the next ring slot
        auto issue_s = [&]() -> bool {
          if (!mbar_wait(bar(B_RFULL + st), ph, a.err, ERR_RING_FULL)) return false;
          if (!mbar_wait(bar(B_SEMPTY + sb), sph ^ 1, a.err, ERR_S)) return false;
          tc_fence_after();
          const uint32_t sk = sbase + OFF_RING + st * SLOT;
          cp_sf(tmem + COL_SFK, sk + TILE_BYTES);
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j)
            mma_mxf8(tmem + COL_S + sb * 128, sw128_desc(sq + j * 32), sw128_desc(sk + j * 32),
                     idescs[j], j > 0, tmem + COL_SFQ + (j << 30), tmem + COL_SFK + (j << 30));
          tc_commit(bar(B_REMPTY + st));
          tc_commit(bar(B_SFULL + sb));
          if (++st == RING) {
            st = 0;
            ph ^= 1;
          }
          if (++sb == 2) {
            sb = 0;
            sph ^= 1;
          }
          return true;
        };
        for (int kt = 0; kt < nkv && ok; ++kt) ok = issue_s();
        if (ok) ok = issue_s();
        for (int kt = 0; kt < nkv && ok; ++kt) {
          if (kt + 1 < nkv && !(ok = issue_s())) break;
          // O += P . V for key tile kt
          if (!mbar_wait(bar(B_RFULL + st), ph, a.err, ERR_RING_FULL) ||
              !mbar_wait(bar(B_PFULL + pb), pph, a.err, ERR_P) ||
              (kt == 0 && !mbar_wait(bar(B_OEMPTY), oph ^ 1, a.err, ERR_O))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sp = sbase + OFF_P + pb * SLOT;
          const uint32_t sv = sbase + OFF_RING + st * SLOT;
          cp_sf(tmem + COL_SFP, sp + TILE_BYTES);
          cp_sf(tmem + COL_SFV, sv + TILE_BYTES);
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j)
            mma_mxf8(tmem + COL_O, sw128_desc(sp + j * 32), sw128_desc(sv + j * 32), idescs[j],
                     (kt > 0 || j > 0) ? 1u : 0u, tmem + COL_SFP + (j << 30),
                     tmem + COL_SFV + (j << 30));
          tc_commit(bar(B_REMPTY + st));
          tc_commit(bar(B_PEMPTY + pb));
          if (++st == RING) {
            st = 0;
            ph ^= 1;
          }
          if (++pb == 2) {
            pb = 0;
            pph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(bar(B_QEMPTY + qb));
        tc_commit(bar(B_OFULL));
        oph ^= 1;
        if (++qb == 2) {
          qb = 0;
          qph ^= 1;
        }
      }
      // every MMA issued has completed before the TMEM is released
      tc_commit(bar(B_DRAIN));
      mbar_wait(bar(B_DRAIN), 0, a.err, ERR_O);
    }
  } else {
    // ---------------- softmax + P quantization + O epilogue ----------------
    const int wq = warp & 3;           // TMEM lane quarter
    const int grp = (warp - 2) >> 2;   // column group: columns grp * 32 .. + 31
    const int r = wq * 32 + lane;      // row in the tile
    const int cb = grp * 32;
    const uint32_t tq = tmem + ((uint32_t)(wq * 32) << 16);
    int sb = 0, pb = 0, it = 0;
    uint32_t sph = 0, pph = 0, oph = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < a.n_items && ok; t += gridDim.x, ++it) {
      int bh, qt, nkv;
      item_coords(a, t, bh, qt, nkv);
      const int q_idx = qt * 128 + r;
      auto load_s = [&](uint32_t (&v)[32]) -> bool {
        if (!mbar_wait_warp(bar(B_SFULL + sb), sph, a.err, ERR_S)) return false;
        tc_fence_after();
        tmem_ld32(tq + COL_S + sb * 128 + cb, v);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar(B_SEMPTY + sb));
        if (++sb == 2) {
          sb = 0;
          sph ^= 1;
        }
        return true;
      };
      // ---- pass 1: row max and sum of exp over this thread's 32 columns ----
      float m = -INFINITY, l = 0.f;
      for (int kt = 0; kt < nkv; ++kt) {
        uint32_t v[32], tb[16];
        if (!(ok = load_s(v))) break;
        scores_bf16(v, a.scale, kt * 128 + cb, q_idx, a.causal && kt == qt, tb);
        __nv_bfloat162 mx2 = *reinterpret_cast<__nv_bfloat162*>(&tb[0]);
#pragma unroll
        for (int i = 1; i < 16; ++i) mx2 = __hmax2(mx2, *reinterpret_cast<__nv_bfloat162*>(&tb[i]));
        const float mn = fmaxf(m, fmaxf(__low2float(mx2), __high2float(mx2)));
        if (mn == -INFINITY) continue;  // every key of this group is masked for this row
        const float nml = -mn * L2E;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          s0 += ex2(fmaf(bf_lo(tb[i]), L2E, nml));
          s1 += ex2(fmaf(bf_hi(tb[i]), L2E, nml));
        }
        l = l * ex2((m - mn) * L2E) + (s0 + s1);
        m = mn;
      }
      if (!ok) break;
      // ---- combine the column groups of each row (same order everywhere) ----
      float2* slot = stats + (it & 1) * (NG * 128);
      slot[grp * 128 + r] = make_float2(m, l);
      mbar_arrive(bar(B_STATS + (it & 1)));
      if (!(ok = mbar_wait_warp(bar(B_STATS + (it & 1)), (it >> 1) & 1, a.err, ERR_STATS))) break;
      float2 st[NG];
#pragma unroll
      for (int g = 0; g < NG; ++g) st[g] = slot[g * 128 + r];
      float M = st[0].x;
#pragma unroll
      for (int g = 1; g < NG; ++g) M = fmaxf(M, st[g].x);
      float L = 0.f;
#pragma unroll
      for (int g = 0; g < NG; ++g)
        L += st[g].x == -INFINITY ? 0.f : st[g].y * ex2((st[g].x - M) * L2E);
      const float rinv = __frcp_rn(L);
      const float nml = -M * L2E;
      // ---- pass 2: P = bf16(exp(s - M) / L) as MXFP8 into shared memory ----
      for (int kt = 0; kt < nkv; ++kt) {
        uint32_t v[32], tb[16];
        if (!(ok = load_s(v))) break;
        scores_bf16(v, a.scale, kt * 128 + cb, q_idx, a.causal && kt == qt, tb);
        uint32_t p2[16];
        uint32_t am = 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float e0 = ex2(fmaf(bf_lo(tb[i]), L2E, nml));
          const float e1 = ex2(fmaf(bf_hi(tb[i]), L2E, nml));
          p2[i] = bf2_rn(e0 * rinv, e1 * rinv);
          am = __vmaxu2(am, p2[i]);
        }
        const uint32_t amax = max(am & 0xFFFFu, am >> 16);
        const uint32_t sbits = pow2_scale_bf16(amax, a.fl2q);
        const uint32_t ue = (sbits >> 7) & 0xFFu;
        uint32_t c[8];
        if ((amax >> 7) < 19u) {  // block max below 2^-108: codes 0
#pragma unroll
          for (int i = 0; i < 8; ++i) c[i] = 0;
        } else {
          // 1 / scale = 2^(127 - ue), exact
          const float inv = __uint_as_float((254u - min(ue, 253u)) << 23);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            uint16_t b0, b1;
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;"
                : "=h"(b0)
                : "f"(bf_hi(p2[2 * i]) * inv), "f"(bf_lo(p2[2 * i]) * inv));
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;"
                : "=h"(b1)
                : "f"(bf_hi(p2[2 * i + 1]) * inv), "f"(bf_lo(p2[2 * i + 1]) * inv));
            c[i] = (uint32_t)b0 | ((uint32_t)b1 << 16);
          }
        }
        if (!(ok = mbar_wait_warp(bar(B_PEMPTY + pb), pph ^ 1, a.err, ERR_P))) break;
        uint8_t* sp = smem + OFF_P + pb * SLOT;
        // 32 codes = logical 16-byte chunks 2 grp, 2 grp + 1 of row r (SWIZZLE_128B)
        const int ch = 2 * grp;
        *reinterpret_cast<uint4*>(sp + r * 128 + ((ch ^ (r & 7)) * 16)) =
            make_uint4(c[0], c[1], c[2], c[3]);
        *reinterpret_cast<uint4*>(sp + r * 128 + (((ch + 1) ^ (r & 7)) * 16)) =
            make_uint4(c[4], c[5], c[6], c[7]);
        // scale byte j = grp of row r in the atom
        sp[TILE_BYTES + (r % 32) * 16 + (r / 32) * 4 + grp] = (uint8_t)ue;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(bar(B_PFULL + pb));
        if (++pb == 2) {
          pb = 0;
          pph ^= 1;
        }
      }
      if (!ok) break;
      // ---- O epilogue: this thread's 32 of the 128 head dims ----
      if (!(ok = mbar_wait_warp(bar(B_OFULL), oph, a.err, ERR_O))) break;
      oph ^= 1;
      tc_fence_after();
      uint32_t o0[32];
      tmem_ld32(tq + COL_O + cb, o0);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(bar(B_OEMPTY));
      const int b = bh / a.H, h = bh % a.H;
      uint16_t* orow = a.out + b * a.os_b + h * a.os_h + (int64_t)q_idx * a.os_s + cb;
      uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        dst[i] = make_uint4(bf2_rn(__uint_as_float(o0[8 * i]), __uint_as_float(o0[8 * i + 1])),
                            bf2_rn(__uint_as_float(o0[8 * i + 2]), __uint_as_float(o0[8 * i + 3])),
                            bf2_rn(__uint_as_float(o0[8 * i + 4]), __uint_as_float(o0[8 * i + 5])),
                            bf2_rn(__uint_as_float(o0[8 * i + 6]), __uint_as_float(o0[8 * i + 7])));
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// This file's sticky wait-timeout word (vq_device_errors).
int sticky_attn(int* out, int clear, cudaStream_t st) { return vq::tc::sticky_read(out, clear, st); }

}  // namespace attn
}  // namespace vq

using namespace vq::attn;

extern "C" {

int vq_attn_mxf8(const void* q, const void* q_sf, const void* k, const void* k_sf, const void* vt,
                 const void* vt_sf, int64_t batch, int64_t heads, int64_t kv_heads, int64_t sq,
                 int64_t skv, int64_t head_dim, float scale, int32_t causal,
                 int32_t floor_log2_qmax, void* out, int64_t out_stride_b, int64_t out_stride_h,
                 int64_t out_stride_s, int32_t* d_err, void* stream) {
  if (!q || !q_sf || !k || !k_sf || !vt || !vt_sf || !out || !d_err) return VQ_ERR_NULL;
  if (batch <= 0 || heads <= 0 || kv_heads <= 0 || sq <= 0 || skv <= 0) return VQ_ERR_INVALID;
  if (head_dim != 128 || sq % 128 || skv % 128 || heads % kv_heads) return VQ_ERR_UNSUPPORTED;
  if (batch * heads * sq >= (1ll << 31) || batch * kv_heads * skv >= (1ll << 31) ||
      skv >= (1 << 24))
    return VQ_ERR_UNSUPPORTED;
  if (out_stride_s < 128 || out_stride_b < 0 || out_stride_h < 0 || out_stride_b % 8 ||
      out_stride_h % 8 || out_stride_s % 8)
    return VQ_ERR_UNSUPPORTED;
  const void* ptrs[7] = {q, q_sf, k, k_sf, vt, vt_sf, out};
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return VQ_ERR_ALIGNMENT;
  CUtensorMap mq, mk, mv;
  if (!vq::mx::make_map(&mq, q, (uint64_t)(batch * heads * sq), 128, 128) ||
      !vq::mx::make_map(&mk, k, (uint64_t)(batch * kv_heads * skv), 128, 128) ||
      !vq::mx::make_map(&mv, vt, (uint64_t)(batch * kv_heads * 128), (uint64_t)skv, 128))
    return VQ_ERR_CUDA;
  AttnArgs g;
  g.q_sf = (const uint8_t*)q_sf;
  g.k_sf = (const uint8_t*)k_sf;
  g.v_sf = (const uint8_t*)vt_sf;
  g.out = (uint16_t*)out;
  g.os_b = out_stride_b;
  g.os_h = out_stride_h;
  g.os_s = out_stride_s;
  g.B = (int)batch;
  g.H = (int)heads;
  g.HKV = (int)kv_heads;
  g.SQ = (int)sq;
  g.SKV = (int)skv;
  g.QT = (int)(sq / 128);
  g.KVT = (int)(skv / 128);
  g.n_items = (int)(batch * heads * g.QT);
  g.scale = scale;
  g.fl2q = floor_log2_qmax;
  g.causal = causal ? 1 : 0;
  g.err = d_err;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int smem = SMEM_TOTAL + 1024;
  if (cudaFuncSetAttribute(k_attn_mxf8, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return VQ_ERR_CUDA;
  if (cudaMemsetAsync(d_err, 0, sizeof(int32_t), st) != cudaSuccess) return VQ_ERR_CUDA;
  const int grid = std::min(g.n_items, vq::mx::sm_count());
  k_attn_mxf8<<<grid, THREADS, smem, st>>>(mq, mk, mv, g);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
