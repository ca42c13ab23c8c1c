// Quantize / dequantize / microscaling kernels for sm_100a and their C ABI.
//
// Three kernels cover the reference's quantized_ops numerics
// (src/voyager_compiler/ops/quantized.py):
//
//   k_qmx_last   quantize_mx / calculate_mx_qparam with blocks along the last
//                dim: one pass over HBM, 16-byte loads, the block amax reduced
//                with warp shuffles, scale and codes written in the same pass.
//   k_qparam     calculate_mx_qparam for blocks along any one or two axes
//                (one thread per block).
//   k_elem       quantize / dequantize with any broadcast or expand()ed
//                scale / zero point (16-byte loads when the inner dim allows).
//
// Element rounding is a vq_rounder (vq_numerics.cuh): analytic for
// minifloat and integer tables, a shared-memory copy of the 65,536-entry bf16
// table otherwise.  Every launch validates its arguments on the host first,
// returns a status and never traps on the device.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <initializer_list>
#include <mutex>

#include "vq_numerics.cuh"
#include "vq_hw.cuh"

namespace vq {

__host__ __device__ __noinline__ float div_slow(float x, float s) { return fdiv_rn(x, s); }

// Any rounder, dispatched at run time, out of line (scale rounding once per
// block, qmaps of dequantize): keeps the switch out of the hot loops' code.
__device__ __noinline__ uint32_t round_any_dev(const vq_rounder& r, uint32_t b,
                                               const uint16_t* tbl) {
  return round_any(r, b, tbl);
}

// Block scale by division (see div_scale) with the scale rounder's kind known
// at compile time: SK 0 = none, 1 = minifloat (inline), 2 = any (out of line).
template <int SK>
__device__ __forceinline__ float div_scale_k(float amax, float qmax, bool is_bf16,
                                             const vq_rounder& sq, const uint16_t* sq_table) {
  // a power-of-two quant_max (1.0 for NormalFloat) divides by one exact multiply
  const float iq = pow2_inverse(qmax);
  float s = iq != 0.0f ? fmul_rn(amax, iq) : fdiv_rn(amax, qmax);
  if (is_bf16) s = round_bf(s);
  if (SK == 1) s = bf2f(round_minifloat(sq, f2bf(s)));
  if (SK == 2) s = bf2f(round_any_dev(sq, f2bf(s), sq_table));
  return (s > 0.0f) ? s : 1.0f;
}

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
constexpr int kTableBytes = 65536 * 2;
constexpr int kTable8Bytes = 65536 + 512;  // byte codes + bf16 palette
// shared memory a TABLE rounder's kernels stage
inline int table_smem(const vq_rounder& r) { return r.table8 ? kTable8Bytes : kTableBytes; }

// Launch shape of a kernel that stages a table in shared memory: of the CTA
// sizes `cands`, the one that keeps the most threads resident under the
// shared-memory and register limits, and the resident CTAs per SM at that
// size.  Found once per (device, kernel, shared-memory size): the host cost
// of a launch must stay well below the kernel's tens of microseconds.
template <typename Kern>
int table_launch_shape(Kern kern, int smem, std::initializer_list<int> cands, int* threads,
                       int* per_sm) {
  struct Entry {
    const void* fn;
    int dev, smem, threads, per_sm;
  };
  static std::mutex mu;
  static Entry cache[256];
  static int n = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return VQ_ERR_CUDA;
  const void* fn = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev && cache[i].smem == smem) {
      *threads = cache[i].threads;
      *per_sm = cache[i].per_sm;
      return VQ_OK;
    }
  // the kernel's dynamic shared-memory limit only ever grows: a launch of
  // this kernel with a larger size found in the cache earlier must still fit
  int limit = smem;
  for (int i = 0; i < n; ++i)
    if (cache[i].fn == fn && cache[i].dev == dev) limit = std::max(limit, cache[i].smem);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, limit) != cudaSuccess)
    return VQ_ERR_CUDA;
  int best = 0, best_t = *cands.begin(), best_per = 1;
  for (int t : cands) {
    int p = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&p, kern, t, smem);
    if (p * t > best) best = p * t, best_t = t, best_per = std::max(p, 1);
  }
  *threads = best_t;
  *per_sm = best_per;
  if (n < 256) cache[n++] = {fn, dev, smem, best_t, best_per};
  return VQ_OK;
}

// CTAs of `threads` threads of a kernel without dynamic shared memory that
// fit on an SM at once (at most 8), found once per device and kernel: a
// grid-stride launch of exactly that many per SM runs as one wave, where 8
// per SM of a kernel that holds more than 32 registers a thread would leave a
// partial second wave.
template <typename Kern>
int resident_ctas(Kern kern, int threads) {
  int t = threads, per_sm = 8;
  if (table_launch_shape(kern, 0, {threads}, &t, &per_sm) != VQ_OK) return 8;
  return std::max(1, std::min(per_sm, 8));
}

// Division by a run-time invariant (Granlund-Montgomery, round-up variant):
// q = (umulhi(n, m) + n) >> s, exact for every 32-bit n.
struct FastDiv {
  uint32_t d, m, s;
  static FastDiv make(uint32_t d) {
    FastDiv f;
    f.d = d;
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    f.s = l;
    f.m = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
    return f;
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    uint32_t hi = __umulhi(n, m);
    return (uint32_t)(((uint64_t)hi + n) >> s);
  }
};

__device__ __forceinline__ float ld_f(const void* p, int64_t i, bool bf) {
  if (bf) return bf2f(((const uint16_t*)p)[i]);
  return ((const float*)p)[i];
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Element rounder specialised at compile time.  TABLE reads the shared-memory
// copy of the bf16 table.
template <int K>
__device__ __forceinline__ uint32_t round_elem(const vq_rounder& r, uint32_t b,
                                               const uint16_t* stab) {
  if (K == VQ_R_IDENTITY) return b & 0xFFFFu;
  if (K == VQ_R_MINIFLOAT) return round_minifloat(r, b);
  if (K == VQ_R_INT) return round_int(r, b);
  if (r.table8) {
    const uint8_t* codes = reinterpret_cast<const uint8_t*>(stab);
    return reinterpret_cast<const uint16_t*>(codes + 65536)[codes[b & 0xFFFFu]];
  }
  return stab[b & 0xFFFFu];
}

// bf16 pattern of a float32 (nearest-even).  The analytic rounders map every
// NaN pattern alike, so they take the hardware conversion; a table needs the
// exact pattern the reference indexes with (0xFFFF for NaN).
template <int K>
__device__ __forceinline__ uint32_t to_bf16_index(float q) {
  if (K == VQ_R_TABLE) return f2bf(q);
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(q));
}

// Copy the 128 KB table into shared memory (TABLE kind only).
template <int K>
__device__ __forceinline__ void stage_table(const vq_rounder& r, uint16_t* stab) {
  if (K != VQ_R_TABLE) return;
  uint4* dst = reinterpret_cast<uint4*>(stab);
  if (r.table8) {
    const uint4* codes = reinterpret_cast<const uint4*>(r.table8);
    const uint4* pal = reinterpret_cast<const uint4*>(r.palette);
    for (int i = threadIdx.x; i < 65536 / 16; i += blockDim.x) dst[i] = __ldg(codes + i);
    for (int i = threadIdx.x; i < 512 / 16; i += blockDim.x) dst[65536 / 16 + i] = __ldg(pal + i);
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(r.table);
    for (int i = threadIdx.x; i < kTableBytes / 16; i += blockDim.x) dst[i] = __ldg(src + i);
  }
  __syncthreads();
}

template <int K>
__device__ __forceinline__ uint32_t round_pair(const vq_rounder& r, uint32_t idx2,
                                               const uint16_t* stab) {
  if (K >= K_HW_E4M3) return hw_pair<K>(idx2, r.nan_bits);
  return round_elem<K>(r, idx2 & 0xFFFFu, stab) | (round_elem<K>(r, idx2 >> 16, stab) << 16);
}

__global__ void k_check_hw(const __grid_constant__ vq_rounder r, int32_t* mism) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;  // pair 0..32767
  if (i >= 32768) return;
  const uint32_t idx2 = (2 * i) | ((2 * i + 1) << 16);
  uint32_t o;
  if (r.hw == VQ_HW_E4M3) o = hw_pair<K_HW_E4M3>(idx2, r.nan_bits);
  else if (r.hw == VQ_HW_E5M2) o = hw_pair<K_HW_E5M2>(idx2, r.nan_bits);
  else o = hw_pair<K_HW_E2M1>(idx2, r.nan_bits);
  const int bad = ((o & 0xFFFFu) != r.table[2 * i]) + ((o >> 16) != r.table[2 * i + 1]);
  if (bad) atomicAdd(mism, bad);
}

// bf16x2 of two floats, round-to-nearest-even (hardware; NaN -> 0x7FFF)
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// ---------------------------------------------------------------------------
// k_qmx_last: fused block scale + quantize, blocks along the last dim
// ---------------------------------------------------------------------------
struct QmxArgs {
  const void* in;
  void* codes;      // may be null (calculate_mx_qparam only)
  void* scale;
  uint32_t ngroups; // rows * nb
  uint32_t C;       // row length (elements)
  uint32_t bs;      // block size (elements)
  FastDiv nb;       // blocks per row
  float quant_max;
  int32_t pow2;
  int32_t fl2q;
  int32_t has_sq;
  const uint16_t* sq_table;  // device table for a TABLE-kind scale rounder
  vq_rounder qr;             // element rounder
  vq_rounder sq;             // scale rounder
  // optional MXFP8 GEMM operand written in the same pass (E4M3 codes with
  // power-of-two block-32 scales): E4M3 bytes [rows, C] and UE8M0 scale
  // atoms [C/128][ceil(rows/128)][512] (see vq_gemm.cu)
  uint8_t* packed;
  uint8_t* packed_sf;
  int32_t packed_rt;
  // quantize_mx_outlier: elements with mask_lo1 <= |x| bits <= +inf bits are
  // outliers and quantized as +0 (filter_outlier's inliers), when mask_on
  int32_t mask_on;
  uint32_t mask_lo1;
  // k_qmx_nvfp4: fl(1 / quant_max) when quant_max has at most 4 significant
  // bits (then bf16(amax * rq) == bf16(amax / quant_max) for a normal
  // quotient), else 0
  float rq;
};

// One block of bs = TPB * VPT * VEC elements per TPB threads; lane l holds
// vectors l, l + TPB, ... so each warp load instruction is contiguous within
// a block.  UNROLL blocks per thread are loaded before any is processed.
template <typename TIn, int K, int SK, int TPB, int VPT, int UNROLL>
__global__ void __launch_bounds__(1024) k_qmx_last(const __grid_constant__ QmxArgs a) {
  extern __shared__ __align__(16) uint16_t smem[];
  stage_table<K>(a.qr, smem);
  constexpr bool BF = sizeof(TIn) == 2;
  constexpr int VEC = 16 / sizeof(TIn);
  constexpr uint32_t GPW = 32 / TPB;  // blocks per warp
  const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t lane = tid % TPB;
  // the loop bound is warp-uniform so every lane reaches the shuffles
  const uint32_t warp_first = (tid / 32) * GPW;
  const uint32_t my_off = (tid % 32) / TPB;
  const uint32_t gstride = (gridDim.x * blockDim.x) / TPB;

  for (uint32_t wb = warp_first; wb < a.ngroups; wb += gstride * UNROLL) {
    uint4 v[UNROLL][VPT];
    uint64_t base[UNROLL];
    uint32_t cb[UNROLL];
    bool live[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const uint32_t g = wb + my_off + u * gstride;
      const uint32_t r = a.nb.div(g);
      const uint32_t blk = g - r * a.nb.d;
      cb[u] = blk * a.bs;
      base[u] = (uint64_t)r * a.C + cb[u];
      live[u] = g < a.ngroups;
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const uint32_t col = blk * a.bs + (j * TPB + lane) * VEC;
        v[u][j] = make_uint4(0, 0, 0, 0);
        if (live[u] && col < a.C)
          v[u][j] = __ldcs(reinterpret_cast<const uint4*>(
              reinterpret_cast<const TIn*>(a.in) + base[u] + (j * TPB + lane) * VEC));
      }
    }
    if (UNROLL == 1) {
      // one block per thread keeps the registers (and so the resident
      // threads) up; the next iteration's block is fetched into L2 meanwhile
      const uint32_t g = wb + my_off + gstride;
      if (g < a.ngroups) {
        const uint32_t r = a.nb.div(g);
        const uint32_t col = (g - r * a.nb.d) * a.bs + lane * (VPT * VEC);  // the block's lines
        if (col < a.C)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const TIn*>(a.in) +
                                                       (uint64_t)r * a.C + col));
      }
    }
    if (a.mask_on) {
#pragma unroll
      for (int u = 0; u < UNROLL; ++u)
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          uint32_t* q = reinterpret_cast<uint32_t*>(&v[u][j]);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (BF) {
              const uint32_t ab = q[k] & 0x7FFF7FFFu;
              q[k] &= ~(__vcmpgeu2(ab, a.mask_lo1 * 0x10001u) & __vcmpleu2(ab, 0x7F807F80u));
            } else {
              const uint32_t ab = q[k] & 0x7FFFFFFFu;
              if (ab >= a.mask_lo1 && ab <= 0x7F800000u) q[k] = 0;
            }
          }
        }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      // block amax on the magnitude bits: non-negative IEEE patterns order
      // like integers and every NaN sorts above +inf, so this max propagates
      // NaN exactly like torch.amax.
      uint32_t m = 0, mn = 0xFFFFu;  // mn: this lane's smallest bf16 magnitude
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        if (BF) {
          const uint32_t a0 = v[u][j].x & 0x7FFF7FFFu, a1 = v[u][j].y & 0x7FFF7FFFu,
                         a2 = v[u][j].z & 0x7FFF7FFFu, a3 = v[u][j].w & 0x7FFF7FFFu;
          const uint32_t w = __vmaxu2(__vmaxu2(a0, a1), __vmaxu2(a2, a3));
          m = max(m, max(w & 0xFFFFu, w >> 16));
          if (K == K_HW_E4M3 && SK == 0) {
            // columns past C hold zeros and send the lane down the exact path
            const uint32_t z = __vminu2(__vminu2(a0, a1), __vminu2(a2, a3));
            mn = min(mn, min(z & 0xFFFFu, z >> 16));
          }
        } else {
          m = max(m, max(max(v[u][j].x & 0x7FFFFFFFu, v[u][j].y & 0x7FFFFFFFu),
                         max(v[u][j].z & 0x7FFFFFFFu, v[u][j].w & 0x7FFFFFFFu)));
        }
      }
      const uint32_t lane_max = m;
#pragma unroll
      for (int o = TPB / 2; o >= 1; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o, TPB));
      // block scale
      float s;
      uint32_t sbits;
      if (a.pow2) {
        sbits = BF ? pow2_scale_bf16(m, a.fl2q) : pow2_scale_f32(m, a.fl2q);
        s = BF ? bf2f(sbits) : u2f(sbits);
      } else {
        float amax = BF ? bf2f(m) : u2f(m);
        s = div_scale_k<SK>(amax, a.quant_max, BF, a.sq, a.sq_table);
        sbits = BF ? f2bf(s) : f2u(s);
      }
      const uint32_t g = wb + my_off + u * gstride;
      if (live[u] && lane == 0) {
        if (BF) reinterpret_cast<uint16_t*>(a.scale)[g] = (uint16_t)sbits;
        else reinterpret_cast<uint32_t*>(a.scale)[g] = sbits;
        if (K == K_HW_E4M3 && BF && a.packed_sf) {
          // UE8M0 = the bf16 exponent field; a subnormal scale (block amax
          // below 2^-118) is stored as 2^-127
          const uint32_t row = (uint32_t)(base[u] / a.C), col = cb[u];
          const uint32_t kt = col / 128, j = (col / 32) % 4, rt = row / 128, rr = row % 128;
          a.packed_sf[((size_t)kt * a.packed_rt + rt) * 512 + (rr % 32) * 16 + (rr / 32) * 4 + j] =
              (uint8_t)((sbits >> 7) & 0xFF);
        }
      }
      if (a.codes == nullptr || !live[u]) continue;
      const Divisor dv = make_divisor(s);
      // float32 input: a NaN-free block with a normal reciprocal takes the
      // hardware bf16 rounding and the FMA-pipe tie test below
      const bool fastq = !BF && dv.fast && m <= 0x7F800000u;
      // bf16 input, E4M3 hardware rounder, power-of-two scale: the quotients
      // are the exact products x * (1 / s), and where none is -0 or NaN the
      // codes and bytes come from one conversion per pair
      const bool e4m3_plain = BF && K == K_HW_E4M3 && SK == 0 && a.pow2 && dv.fast &&
                              plain_quotients((sbits >> 7) & 0xFFu, dv.r, mn, lane_max);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const uint32_t off = (j * TPB + lane) * VEC;
        if (cb[u] + off >= a.C) continue;
        uint32_t w[4] = {v[u][j].x, v[u][j].y, v[u][j].z, v[u][j].w};
        if (BF && K == K_HW_E4M3 && e4m3_plain) {
          // one saturating conversion per pair gives both the code and its
          // GEMM byte (plain_quotients rules out hw_pair's special cases)
          uint32_t b16[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            b16[k] = e4m3_pair(bf16x2_rn(bf2f(w[k] & 0xFFFFu) * dv.r, bf2f(w[k] >> 16) * dv.r),
                               w[k]);
          if (a.packed)
            *reinterpret_cast<uint2*>(a.packed + base[u] + off) =
                make_uint2(b16[0] | (b16[1] << 16), b16[2] | (b16[3] << 16));
        } else if (BF) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float q0 = div_to_bf16_domain(bf2f(w[k] & 0xFFFFu), dv);
            const float q1 = div_to_bf16_domain(bf2f(w[k] >> 16), dv);
            w[k] = round_pair<K>(a.qr, pair_index<K>(q0, q1), smem);
          }
          if (K == K_HW_E4M3 && a.packed) {
            // the codes are E4M3 values: their bytes for the GEMM
            uint32_t pb[2];
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
              uint16_t b0, b1;
              const float c0 = __uint_as_float(w[k] << 16), c1 = __uint_as_float(w[k] & 0xFFFF0000u);
              const float c2 = __uint_as_float(w[k + 1] << 16),
                          c3 = __uint_as_float(w[k + 1] & 0xFFFF0000u);
              asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b0) : "f"(c1), "f"(c0));
              asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b1) : "f"(c3), "f"(c2));
              pb[k / 2] = (uint32_t)b0 | ((uint32_t)b1 << 16);
            }
            *reinterpret_cast<uint2*>(a.packed + base[u] + off) = make_uint2(pb[0], pb[1]);
          }
        } else {
          bool exact = true;
          if (fastq) {
            // quotients x * fl(1/s); the bf16 rounding of q - d and q + d
            // agrees (d = |q| 2^-21 + 2^-146, computed on the FMA pipe) unless
            // fl(x / s), which lies within 1.5 * 2^-23 |q| (3 subnormal ulps
            // below 2^-126) of q, could round to another bf16.  No NaN here
            // (finite r, NaN-free block), so the hardware rounding gives the
            // index the table takes.
            float q[4];
            uint32_t tie = 0, c[2];
#pragma unroll
            for (int k = 0; k < 4; ++k) q[k] = __fmul_rn(u2f(w[k]), dv.r);
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
              const float d0 = __fmaf_rn(fabsf(q[k]), 0x1p-21f, 0x1p-146f);
              const float d1 = __fmaf_rn(fabsf(q[k + 1]), 0x1p-21f, 0x1p-146f);
              tie |= bf16x2_rn(__fsub_rn(q[k], d0), __fsub_rn(q[k + 1], d1)) ^
                     bf16x2_rn(__fadd_rn(q[k], d0), __fadd_rn(q[k + 1], d1));
              c[k / 2] = round_pair<K>(a.qr, bf16x2_rn(q[k], q[k + 1]), smem);
            }
            if (!tie) {
              w[0] = c[0] << 16, w[1] = c[0] & 0xFFFF0000u;
              w[2] = c[1] << 16, w[3] = c[1] & 0xFFFF0000u;
              exact = false;
            }
          }
          if (exact) {
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
              const float q0 = div_to_bf16_domain(u2f(w[k]), dv);
              const float q1 = div_to_bf16_domain(u2f(w[k + 1]), dv);
              const uint32_t c2 = round_pair<K>(a.qr, pair_index<K>(q0, q1), smem);
              w[k] = c2 << 16;
              w[k + 1] = c2 & 0xFFFF0000u;
            }
          }
        }
        __stcs(reinterpret_cast<uint4*>(reinterpret_cast<TIn*>(a.codes) + base[u] + off),
               make_uint4(w[0], w[1], w[2], w[3]));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// k_qmx_nvfp4: quantize_mx for NVFP4 (the C1 configuration) -- bf16 input,
// E2M1 element table and E4M3 scale table both reproduced by the hardware
// conversions (verified), blocks of 16 along rows whose length is a multiple
// of 16 (so block g starts at element 16 g).  One thread per block.
//
// Per block: amax (and min) on magnitude bits; a block holding a NaN or a
// scale whose reciprocal is not a normal float takes the generic path (IEEE
// division, hw_pair); otherwise the quotients are x * fl(1/s), rounded to
// bf16 in pairs, converted to E2M1 pairs and back through a 256-entry table
// of the E2M1 values as bf16 (the -0 code stays -0).  When every quotient of
// the block is a normal float its bf16 is that of x / s with no test (the
// exact quotient of a bf16 by an E4M3 value is never near a bf16 rounding
// midpoint, see below); blocks with zeros or tiny values test the low 16 bits
// for a near-tie and turn a -0 index into +0, as the table has it.
// ---------------------------------------------------------------------------
// bf16 bits of an E2M1 code (4 bits: sign, 2 exponent bits with bias 1, 1
// mantissa bit): 0, 0.5, 1, 1.5, 2, 3, 4, 6 and their negatives (-0 too)
__device__ __forceinline__ uint32_t e2m1_bf16(uint32_t nib) {
  const uint32_t e = (nib >> 1) & 3u, f = nib & 1u;
  const uint32_t mag = e == 0 ? (f ? 0x3F00u : 0u) : (((e + 126u) << 7) | (f << 6));
  return mag | ((nib & 8u) << 12);
}

__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// E4M3 rounding (round-half-even, saturating) of a non-negative float, as
// bf16 bits: the value quantize's E4M3 table gives for it (verified
// hardware rounder).  A NaN gives a NaN (the caller's "not > 0" then takes
// the scale 1).
__device__ __forceinline__ uint32_t e4m3_bf16(float v) {
  uint32_t h;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %1;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(h) : "f"(v));
  return __float_as_uint(__half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)))) >> 16;
}

// bf16 bits of the positive E4M3 code b (b < 0x7F: 4 exponent bits with bias
// 7, 3 mantissa bits; subnormals below 2^-6)
__device__ __forceinline__ uint32_t e4m3_code_bf16(uint32_t b) {
  const uint32_t e = b >> 3, m = b & 7u;
  if (e == 0) return m ? __float_as_uint((float)m * 0x1p-9f) >> 16 : 0u;
  return ((e + 120u) << 7) | (m << 4);
}

template <bool MASK>
__global__ void __launch_bounds__(256) k_qmx_nvfp4(const __grid_constant__ QmxArgs a) {
  __shared__ uint32_t lut[256];
  // the positive E4M3 scale values by code: bf16 bits, and the IEEE
  // reciprocal of each (1 for the zero code: such a block takes the scale 1)
  __shared__ uint32_t sval[128];
  __shared__ float srcp[128];
  if (threadIdx.x < 256) lut[threadIdx.x] = e2m1_bf16(threadIdx.x) | (e2m1_bf16(threadIdx.x >> 4) << 16);
  if (threadIdx.x < 128) {
    const uint32_t v = threadIdx.x == 0x7Fu ? 0u : e4m3_code_bf16(threadIdx.x);  // NaN: scale 1
    sval[threadIdx.x] = v;
    srcp[threadIdx.x] = v ? fdiv_rn(1.0f, __uint_as_float(v << 16)) : 1.0f;
  }
  __syncthreads();
  const uint32_t nthr = gridDim.x * blockDim.x;
  for (uint32_t g0 = blockIdx.x * blockDim.x + threadIdx.x; g0 < a.ngroups; g0 += 2 * nthr) {
    uint32_t w[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t g = g0 + u * nthr;
      if (g < a.ngroups) {
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.in) +
                                                          (uint64_t)g * 16);
        const uint4 q0 = __ldcs(src), q1 = __ldcs(src + 1);
        w[u][0] = q0.x, w[u][1] = q0.y, w[u][2] = q0.z, w[u][3] = q0.w;
        w[u][4] = q1.x, w[u][5] = q1.y, w[u][6] = q1.z, w[u][7] = q1.w;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t g = g0 + u * nthr;
      if (g >= a.ngroups) continue;
      // block max / min of |x| as bf16x2 (NaN-propagating max: a NaN
      // magnitude sorts above +inf in the bits, so amax > 0x7F80 finds it)
      __nv_bfloat162 mx2 = __floats2bfloat162_rn(0.0f, 0.0f);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t ab = w[u][k] & 0x7FFF7FFFu;
        mx2 = __hmax2_nan(mx2, *reinterpret_cast<const __nv_bfloat162*>(&ab));
      }
      uint32_t mx = *reinterpret_cast<uint32_t*>(&mx2);
      uint32_t amax = max(mx & 0xFFFFu, mx >> 16);
      if (MASK && amax >= a.mask_lo1) {
        // quantize_mx_outlier: this block holds outliers, quantized as +0
        mx = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ab = w[u][k] & 0x7FFF7FFFu;
          w[u][k] &= ~(__vcmpgeu2(ab, a.mask_lo1 * 0x10001u) & __vcmpleu2(ab, 0x7F807F80u));
          mx = __vmaxu2(mx, w[u][k] & 0x7FFF7FFFu);
        }
        amax = max(mx & 0xFFFFu, mx >> 16);
      }
      __nv_bfloat162 mn2 = __floats2bfloat162_rn(__int_as_float(0x7F800000), __int_as_float(0x7F800000));
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t ab = w[u][k] & 0x7FFF7FFFu;
        mn2 = __hmin2(mn2, *reinterpret_cast<const __nv_bfloat162*>(&ab));
      }
      const float amin = fminf(__low2float(mn2), __high2float(mn2));  // a NaN is ignored
      // scale = e4m3(bf16(amax / quant_max)), 1 where not > 0; the
      // quotient by the reciprocal where that is exact in bf16 (rq != 0
      // and a normal quotient), else the IEEE division
      const float af = bf2f(amax);
      float sq = __fmul_rn(af, a.rq);
      if (!(sq >= 0x1p-126f) || isinf(sq)) sq = fdiv_rn(af, a.quant_max);
      const float s0 = round_bf(sq);
      uint32_t code;  // the saturating E4M3 rounding of s0 (0x7F: NaN)
      asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %1;\n\tcvt.u32.u16 %0, t;\n\t}"
          : "=r"(code) : "f"(s0));
      code &= 0x7Fu;
      const uint32_t svb = sval[code];
      const float s = svb ? __uint_as_float(svb << 16) : 1.0f;
      reinterpret_cast<uint16_t*>(a.scale)[g] = (uint16_t)f2bf(s);
      bool slow = amax > 0x7F80u || code == 0x7Fu;
      uint32_t out[8];
      if (!slow) {
        const float r = srcp[code];
        if (__fmul_rn(amin, r) >= 0x1p-126f) {
          // every quotient is a normal float (no zero index).  Then
          // bf16(x * fl(1/s)) == bf16(x / s): x / s = M_x / M_s * 2^E with
          // M_x < 256 (bf16) and M_s < 16 (E4M3) is never a bf16 rounding
          // midpoint and lies at least 2^-8 / 15 of its binade away from
          // one, while both float32 results are within 2^-23 of it (checked
          // on the host for every bf16 x and E4M3 s:
          // tests/test_nvfp4_quotients.py)
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float q0 = __fmul_rn(__uint_as_float(w[u][k] << 16), r);
            const float q1 = __fmul_rn(__uint_as_float(w[u][k] & 0xFFFF0000u), r);
            const uint32_t idx = bf16x2_rn(q0, q1);
            out[k] = lut[e2m1x2(__uint_as_float(idx << 16), __uint_as_float(idx & 0xFFFF0000u))];
          }
        } else {
          uint32_t tie = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float q0 = __fmul_rn(__uint_as_float(w[u][k] << 16), r);
            const float q1 = __fmul_rn(__uint_as_float(w[u][k] & 0xFFFF0000u), r);
            tie |= __vcmpleu2(__vsub2(__byte_perm(__float_as_uint(q0), __float_as_uint(q1), 0x5410),
                                      0x7FFC7FFCu),
                              0x00080008u);
            const uint32_t idx = bf16x2_rn(q0, q1);
            uint32_t o = lut[e2m1x2(__uint_as_float(idx << 16), __uint_as_float(idx & 0xFFFF0000u))];
            // a -0 index gives +0
            o &= ~(__vcmpeq2(idx & 0x7FFF7FFFu, 0u) & 0x80008000u);
            out[k] = o;
          }
          slow = tie != 0;
        }
      }
      if (slow) {
        // generic: IEEE quotients, the verified hardware pair rounder
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float q0 = div_slow(__uint_as_float(w[u][k] << 16), s);
          const float q1 = div_slow(__uint_as_float(w[u][k] & 0xFFFF0000u), s);
          out[k] = hw_pair<K_HW_E2M1>(f2bf(q0) | (f2bf(q1) << 16), a.qr.nan_bits);
        }
      }
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.codes) + (uint64_t)g * 16);
      __stcs(dst, make_uint4(out[0], out[1], out[2], out[3]));
      __stcs(dst + 1, make_uint4(out[4], out[5], out[6], out[7]));
    }
  }
}

// ---------------------------------------------------------------------------
// k_qparam: calculate_mx_qparam over one or two blocked axes (generic)
// ---------------------------------------------------------------------------
struct QparamArgs {
  const void* in;
  void* scale;
  int32_t is_bf16;
  int32_t ndim;
  int64_t nscale;
  int64_t sshape[VQ_MAX_DIMS];   // scale (blocked) shape
  int64_t ishape[VQ_MAX_DIMS];   // input shape
  int64_t istride[VQ_MAX_DIMS];  // input strides (elements)
  int32_t blocked[VQ_MAX_DIMS];  // 1 if the dim is blocked
  int64_t bs;
  float quant_max;
  int32_t pow2;
  int32_t fl2q;
  int32_t has_sq;
  const uint16_t* sq_table;
  vq_rounder sq;
};

__global__ void __launch_bounds__(256) k_qparam(const __grid_constant__ QparamArgs a) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.nscale) return;
  // coordinates of this block and the element range it covers
  int64_t rem = i, base = 0;
  int64_t ext[2] = {1, 1}, str[2] = {0, 0};
  int nb = 0;
  for (int d = a.ndim - 1; d >= 0; --d) {
    int64_t c = rem % a.sshape[d];
    rem /= a.sshape[d];
    if (a.blocked[d]) {
      int64_t lo = c * a.bs;
      int64_t e = a.ishape[d] - lo;
      if (e > a.bs) e = a.bs;
      base += lo * a.istride[d];
      if (nb < 2) {
        ext[nb] = e;
        str[nb] = a.istride[d];
      }
      ++nb;
    } else {
      base += c * a.istride[d];
    }
  }
  uint32_t m = 0;
  for (int64_t p = 0; p < ext[0]; ++p) {
    for (int64_t q = 0; q < ext[1]; ++q) {
      int64_t off = base + p * str[0] + q * str[1];
      uint32_t bits = a.is_bf16 ? (uint32_t)((const uint16_t*)a.in)[off] & 0x7FFFu
                                : ((const uint32_t*)a.in)[off] & 0x7FFFFFFFu;
      m = max(m, bits);
    }
  }
  uint32_t sbits;
  if (a.pow2) {
    sbits = a.is_bf16 ? pow2_scale_bf16(m, a.fl2q) : pow2_scale_f32(m, a.fl2q);
  } else {
    float amax = a.is_bf16 ? bf2f(m) : u2f(m);
    float s = div_scale(amax, a.quant_max, a.is_bf16, a.has_sq ? &a.sq : nullptr, a.sq_table);
    sbits = a.is_bf16 ? f2bf(s) : f2u(s);
  }
  if (a.is_bf16) ((uint16_t*)a.scale)[i] = (uint16_t)sbits;
  else ((uint32_t*)a.scale)[i] = sbits;
}

// ---------------------------------------------------------------------------
// k_affine_qparam: quantize_affine's per-block scale and zero point
// (quantized.py:884-948): min / max of each zero-padded block, then
//   scale = where(s > 0, s, 1) with s = (max - min) / (qmax - qmin),
//   optionally through scale_qmap (and where() again),
//   zero_point = -min / scale + qmin, optionally through scale_qmap,
// every binary op rounded to the input dtype.
// ---------------------------------------------------------------------------
struct AffineArgs {
  QparamArgs q;  // shapes, blocked dims, scale rounder
  void* zp;
  float qmin, qmax;
};

__device__ __forceinline__ float nan_min(float a, float b) {
  return (is_nan_f(a) || is_nan_f(b)) ? u2f(0x7FC00000u) : fminf(a, b);
}
__device__ __forceinline__ float nan_max(float a, float b) {
  return (is_nan_f(a) || is_nan_f(b)) ? u2f(0x7FC00000u) : fmaxf(a, b);
}

__global__ void __launch_bounds__(256) k_affine_qparam(const __grid_constant__ AffineArgs aa) {
  const QparamArgs& a = aa.q;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.nscale) return;
  int64_t rem = i, base = 0, ext = 1, str = 0;
  bool padded = false;
  for (int d = a.ndim - 1; d >= 0; --d) {
    int64_t c = rem % a.sshape[d];
    rem /= a.sshape[d];
    if (a.blocked[d]) {
      int64_t lo = c * a.bs;
      int64_t e = a.ishape[d] - lo;
      // _reshape_to_blocks pads the ragged tail with zeros
      if (e < a.bs && a.ishape[d] >= a.bs) padded = true;
      if (a.ishape[d] % a.bs != 0 && a.ishape[d] < a.bs) padded = true;
      if (e > a.bs) e = a.bs;
      base += lo * a.istride[d];
      ext = e;
      str = a.istride[d];
    } else {
      base += c * a.istride[d];
    }
  }
  const bool bf = a.is_bf16;
  float lo = padded ? 0.0f : INFINITY, hi = padded ? 0.0f : -INFINITY;
  for (int64_t p = 0; p < ext; ++p) {
    float v = ld_f(a.in, base + p * str, bf);
    lo = nan_min(lo, v);
    hi = nan_max(hi, v);
  }
  auto rnd = [bf](float v) { return bf ? round_bf(v) : v; };
  float s = rnd(fdiv_rn(rnd(fsub_rn(hi, lo)), fsub_rn(aa.qmax, aa.qmin)));
  s = (s > 0.0f) ? s : 1.0f;
  const vq_rounder* sq = a.has_sq ? &a.sq : nullptr;
  if (sq) {
    s = bf2f(round_any_dev(*sq, f2bf(s), a.sq_table));
    s = (s > 0.0f) ? s : 1.0f;
  }
  float z = rnd(fadd_rn(rnd(fdiv_rn(-lo, s)), aa.qmin));
  if (sq) z = bf2f(round_any_dev(*sq, f2bf(z), a.sq_table));
  if (bf) {
    ((uint16_t*)a.scale)[i] = (uint16_t)f2bf(s);
    ((uint16_t*)aa.zp)[i] = (uint16_t)f2bf(z);
  } else {
    ((float*)a.scale)[i] = s;
    ((float*)aa.zp)[i] = z;
  }
}

// ---------------------------------------------------------------------------
// k_elem2d: quantize / dequantize on a [R, C] view (the common layouts)
// ---------------------------------------------------------------------------
// The operand offset is (row / div_r) * str_r + (col / div_c) * str_c, with
// the layout known at compile time:
//   SL_SCALAR  one value (per-tensor scale),
//   SL_ROW     constant along a row (per-channel scale, [R, 1]),
//   SL_2D      anything else on the 2-D view (block scales along C, ...).
// Quantize divides by a cached Divisor (one reciprocal per distinct scale);
// the zero point, when present, is read per element through its own map.
enum { SL_SCALAR = 0, SL_ROW = 1, SL_2D = 2 };

struct Map2D {
  const void* ptr;
  int32_t is_bf16;
  int32_t uniform_vec;
  FastDiv div_r, div_c;
  int64_t str_r, str_c;
};

struct Elem2DArgs {
  const void* in;
  void* out;
  uint32_t nvec;
  FastDiv C;
  Map2D scale, zp;
  int32_t has_zp;
  int32_t r1_bf16, r2_bf16;
  int32_t exact_div;  // x / s feeds an fp32 add: needs the IEEE quotient
  int32_t has_inq, has_outq;
  const uint16_t* inq_table;
  const uint16_t* outq_table;
  vq_rounder inq, outq;
  vq_rounder qr;
};

__device__ __forceinline__ int64_t map_off(const Map2D& m, uint32_t row, uint32_t col) {
  return (int64_t)m.div_r.div(row) * m.str_r + (int64_t)m.div_c.div(col) * m.str_c;
}

// Quantize one vector's quotients (x / s, rounded to bf16 when the index is
// taken) into codes, in pairs.
template <typename TIn, int K, int VEC>
__device__ __forceinline__ void quant_vec(const Elem2DArgs& a, const TIn* xin, const float* s,
                                          const float* z, bool zp, uint32_t* codes,
                                          const uint16_t* stab) {
  constexpr bool IN_BF = sizeof(TIn) == 2;
  float t[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const float x = IN_BF ? bf2f(*reinterpret_cast<const uint16_t*>(&xin[j]))
                          : *reinterpret_cast<const float*>(&xin[j]);
    if (!zp) {
      t[j] = div_slow(x, s[j]);
    } else if (a.exact_div) {  // r1 float32: the add needs the IEEE quotient
      float q = fdiv_rn(x, s[j]);
      q = fadd_rn(q, z[j]);
      t[j] = a.r2_bf16 ? round_bf(q) : q;
    } else {  // r1 bf16: round the quotient, add, round per r2
      float q = fadd_rn(round_bf(fdiv_rn(x, s[j])), z[j]);
      t[j] = a.r2_bf16 ? round_bf(q) : q;
    }
  }
  if (VEC == 1) {
    codes[0] = round_elem<K < K_HW_E4M3 ? K : VQ_R_MINIFLOAT>(a.qr, f2bf(t[0]), stab);
    return;
  }
#pragma unroll
  for (int j = 0; j < VEC; j += 2) {
    const uint32_t c2 = round_pair<K>(a.qr, pair_index<K>(t[j], t[j + 1]), stab);
    codes[j] = c2 & 0xFFFFu;
    codes[j + 1] = c2 >> 16;
  }
}

// Same for a uniform scale with a Divisor (reciprocal multiply, exact).
template <typename TIn, int K, int VEC>
__device__ __forceinline__ void quant_vec_fast(const Elem2DArgs& a, const TIn* xin,
                                               const Divisor& dv, uint32_t* codes,
                                               const uint16_t* stab) {
  constexpr bool IN_BF = sizeof(TIn) == 2;
  float t[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const float x = IN_BF ? bf2f(*reinterpret_cast<const uint16_t*>(&xin[j]))
                          : *reinterpret_cast<const float*>(&xin[j]);
    t[j] = div_to_bf16_domain(x, dv);
  }
  if (VEC == 1) {
    codes[0] = round_elem<K < K_HW_E4M3 ? K : VQ_R_MINIFLOAT>(a.qr, f2bf(t[0]), stab);
    return;
  }
#pragma unroll
  for (int j = 0; j < VEC; j += 2) {
    const uint32_t c2 = round_pair<K>(a.qr, pair_index<K>(t[j], t[j + 1]), stab);
    codes[j] = c2 & 0xFFFFu;
    codes[j + 1] = c2 >> 16;
  }
}

template <typename TIn, typename TOut, bool DEQ, int K, int VEC, int SL, bool QM, int UNROLL>
__global__ void __launch_bounds__(1024) k_elem2d(const __grid_constant__ Elem2DArgs a) {
  extern __shared__ __align__(16) uint16_t smem[];
  if (!DEQ) stage_table<K>(a.qr, smem);
  constexpr bool IN_BF = sizeof(TIn) == 2;
  constexpr bool OUT_BF = sizeof(TOut) == 2;
  constexpr int IN_B = VEC * sizeof(TIn), OUT_B = VEC * sizeof(TOut);
  const uint32_t stride = gridDim.x * blockDim.x;
  const bool zp = a.has_zp;
  int64_t cached = -1;
  float s = 1.f;
  Divisor dv = make_divisor(1.f);
  if (SL == SL_SCALAR) {
    s = ld_f(a.scale.ptr, 0, a.scale.is_bf16);
    if (!DEQ) dv = make_divisor(s);
  }
  for (uint32_t v0 = blockIdx.x * blockDim.x + threadIdx.x; v0 < a.nvec; v0 += stride * UNROLL) {
    TIn xin[UNROLL][VEC];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const uint32_t v = v0 + u * stride;
      if (v >= a.nvec) continue;
      const TIn* src = reinterpret_cast<const TIn*>(a.in) + (uint64_t)v * VEC;
      if (IN_B == 16) {
        *reinterpret_cast<uint4*>(xin[u]) = __ldcs(reinterpret_cast<const uint4*>(src));
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) xin[u][j] = src[j];
      }
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const uint32_t v = v0 + u * stride;
      if (v >= a.nvec) continue;
      const uint32_t e = v * VEC;
      uint32_t row = 0, col = 0;
      if (SL != SL_SCALAR || zp) {
        row = a.C.div(e);
        col = e - row * a.C.d;
      }
      const bool uni = SL != SL_2D || a.scale.uniform_vec;
      if (SL != SL_SCALAR && uni) {
        const int64_t off = map_off(a.scale, row, col);
        if (off != cached) {
          cached = off;
          s = ld_f(a.scale.ptr, off, a.scale.is_bf16);
          if (!DEQ) dv = make_divisor(s);
        }
      }
      uint32_t ob[VEC];
      float of[VEC];
      if (!DEQ && uni && !zp) {
        // the hot path: one scale per vector, reciprocal multiply
        quant_vec_fast<TIn, K, VEC>(a, xin[u], dv, ob, smem);
#pragma unroll
        for (int j = 0; j < VEC; ++j) of[j] = bf2f(ob[j]);
      } else {
        float sv[VEC], zv[VEC];
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          sv[j] = uni ? s : ld_f(a.scale.ptr, map_off(a.scale, row, col + j), a.scale.is_bf16);
          zv[j] = zp ? ld_f(a.zp.ptr, map_off(a.zp, row, col + j), a.zp.is_bf16) : 0.f;
        }
        if (!DEQ) {
          quant_vec<TIn, K, VEC>(a, xin[u], sv, zv, zp, ob, smem);
#pragma unroll
          for (int j = 0; j < VEC; ++j) of[j] = bf2f(ob[j]);
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const uint32_t xb = IN_BF ? (uint32_t)(*reinterpret_cast<const uint16_t*>(&xin[u][j])) : 0u;
            float w = IN_BF ? bf2f(xb) : *reinterpret_cast<const float*>(&xin[u][j]);
            if (QM && a.has_inq)
              w = bf2f(round_any_dev(a.inq, IN_BF ? xb : f2bf(w), a.inq_table));
            if (zp) {
              w = fsub_rn(w, zv[j]);
              if (a.r1_bf16) w = round_bf(w);
            }
            w = fmul_rn(w, sv[j]);
            if (a.r2_bf16) w = round_bf(w);
            if (QM && a.has_outq) w = bf2f(round_any_dev(a.outq, f2bf(w), a.outq_table));
            of[j] = w;
            ob[j] = f2bf(w);
          }
        }
      }
      TOut res[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        if (OUT_BF) *reinterpret_cast<uint16_t*>(&res[j]) = (uint16_t)ob[j];
        else *reinterpret_cast<float*>(&res[j]) = of[j];
      }
      TOut* dst = reinterpret_cast<TOut*>(a.out) + (uint64_t)v * VEC;
      if (OUT_B == 16) {
        __stcs(reinterpret_cast<uint4*>(dst), *reinterpret_cast<uint4*>(res));
      } else if (OUT_B == 32) {
        __stcs(reinterpret_cast<uint4*>(dst), reinterpret_cast<uint4*>(res)[0]);
        __stcs(reinterpret_cast<uint4*>(dst) + 1, reinterpret_cast<uint4*>(res)[1]);
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) dst[j] = res[j];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// k_rows: quantize / dequantize row by row (the hot layouts)
// ---------------------------------------------------------------------------
// A persistent grid walks the rows of the [R, C] view; the CTA's threads
// stride over one row's vectors.  The scale is per tensor (SL_SCALAR), per
// row (SL_ROW) or per block of 2^shift columns along the row (SL_2D with
// str_c = 1 and a power-of-two block), so an element's scale needs no
// division: row offset + (col >> shift).  Quantize divides by the row's (or
// block's) Divisor: one reciprocal per distinct scale per thread.
struct RowsArgs {
  const void* in;
  void* out;
  const void* scale;
  int32_t scale_bf16;
  int32_t nrows;
  int32_t vpr;      // vectors per row (C / VEC)
  int64_t nvec;     // vectors in the whole tensor (a scalar scale's last row may be short)
  int64_t C;
  int64_t str_r;    // scale offset per row (0 for SL_SCALAR)
  int32_t shift;    // SL_2D: log2(block size)
  vq_rounder qr;
};

template <typename TIn, typename TOut, bool DEQ, int K, int SL, int U>
__global__ void __launch_bounds__(1024) k_rows(const __grid_constant__ RowsArgs a) {
  extern __shared__ __align__(16) uint16_t smem[];
  if (!DEQ) stage_table<K>(a.qr, smem);
  constexpr bool IN_BF = sizeof(TIn) == 2;
  constexpr bool OUT_BF = sizeof(TOut) == 2;
  constexpr int VEC = 16 / sizeof(TIn);
  float s = 1.f;
  Divisor dv = make_divisor(1.f);
  if (SL == SL_SCALAR) {
    s = ld_f(a.scale, 0, a.scale_bf16);
    if (!DEQ) dv = make_divisor(s);
  }
  int64_t cached = -1;
  for (int row = blockIdx.x; row < a.nrows; row += gridDim.x) {
    if (SL == SL_ROW) {
      s = ld_f(a.scale, (int64_t)row * a.str_r, a.scale_bf16);
      if (!DEQ) dv = make_divisor(s);
    }
    const TIn* src = reinterpret_cast<const TIn*>(a.in) + (int64_t)row * a.C;
    TOut* dst = reinterpret_cast<TOut*>(a.out) + (int64_t)row * a.C;
    const int vend = (int)min((int64_t)a.vpr, a.nvec - (int64_t)row * a.vpr);
    for (int v0 = threadIdx.x; v0 < vend; v0 += U * blockDim.x) {
      uint4 raws[U];
      int vv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        vv[u] = v0 + u * (int)blockDim.x;
        if (vv[u] < vend) raws[u] = __ldcs(reinterpret_cast<const uint4*>(src) + vv[u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = vv[u];
        if (v >= vend) break;
        const uint4 raw = raws[u];
        if (SL == SL_2D) {
          const int64_t off = (int64_t)row * a.str_r + (((int64_t)v * VEC) >> a.shift);
          if (off != cached) {
            cached = off;
            s = ld_f(a.scale, off, a.scale_bf16);
            if (!DEQ) dv = make_divisor(s);
          }
        }
        const TIn* x = reinterpret_cast<const TIn*>(&raw);
        uint32_t ob[VEC];
        float of[VEC];
        if (!DEQ) {
          bool exact = true;
          if (!IN_BF && K == VQ_R_TABLE && dv.fast) {
            // float32 input into a table (the index costs most): quotients
            // x * fl(1/s), bf16-rounded by the hardware, unless the FMA-pipe
            // tie test (q -+ |q| 2^-21 + 2^-146 round alike) or a NaN index
            // (the table wants 0xFFFF for it) sends the vector to the exact path
            float q[VEC];
            uint32_t flag = 0, c2v[VEC / 2];
#pragma unroll
            for (int j = 0; j < VEC; ++j) q[j] = __fmul_rn(*reinterpret_cast<const float*>(&x[j]), dv.r);
#pragma unroll
            for (int j = 0; j < VEC; j += 2) {
              const float d0 = __fmaf_rn(fabsf(q[j]), 0x1p-21f, 0x1p-146f);
              const float d1 = __fmaf_rn(fabsf(q[j + 1]), 0x1p-21f, 0x1p-146f);
              const uint32_t idx = bf16x2_rn(q[j], q[j + 1]);
              flag |= (bf16x2_rn(__fsub_rn(q[j], d0), __fsub_rn(q[j + 1], d1)) ^
                       bf16x2_rn(__fadd_rn(q[j], d0), __fadd_rn(q[j + 1], d1))) |
                      (((idx & 0x7FFF7FFFu) + 0x007F007Fu) & 0x80008000u);
              c2v[j / 2] = round_pair<K>(a.qr, idx, smem);
            }
            if (!flag) {
#pragma unroll
              for (int j = 0; j < VEC; j += 2) {
                const uint32_t c2 = c2v[j / 2];
                ob[j] = c2 & 0xFFFFu;
                ob[j + 1] = c2 >> 16;
                of[j] = __uint_as_float(c2 << 16);
                of[j + 1] = __uint_as_float(c2 & 0xFFFF0000u);
              }
              exact = false;
            }
          }
          if (exact) {
            float t[VEC];
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
              const float xf = IN_BF ? bf2f(*reinterpret_cast<const uint16_t*>(&x[j]))
                                     : *reinterpret_cast<const float*>(&x[j]);
              t[j] = div_to_bf16_domain(xf, dv);
            }
#pragma unroll
            for (int j = 0; j < VEC; j += 2) {
              const uint32_t c2 = round_pair<K>(a.qr, pair_index<K>(t[j], t[j + 1]), smem);
              ob[j] = c2 & 0xFFFFu;
              ob[j + 1] = c2 >> 16;
              of[j] = __uint_as_float(c2 << 16);
              of[j + 1] = __uint_as_float(c2 & 0xFFFF0000u);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            const float xf = IN_BF ? bf2f(*reinterpret_cast<const uint16_t*>(&x[j]))
                                   : *reinterpret_cast<const float*>(&x[j]);
            float w = fmul_rn(xf, s);
            if (OUT_BF) {
              ob[j] = f2bf(w);
            } else {
              of[j] = w;
            }
          }
        }
        if (OUT_BF) {
          uint4 o;
          uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int j = 0; j < VEC / 2; ++j) ow[j] = ob[2 * j] | (ob[2 * j + 1] << 16);
          if (VEC == 8) {
            __stcs(reinterpret_cast<uint4*>(dst) + v, o);
          } else {  // fp32 in, bf16 out does not arise (promotion)
            *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(dst) + (int64_t)v * VEC) =
                make_uint2(ow[0], ow[1]);
          }
        } else {
          TOut* d = dst + (int64_t)v * VEC;
          if (VEC == 4) {
            __stcs(reinterpret_cast<float4*>(d), make_float4(of[0], of[1], of[2], of[3]));
          } else {
            __stcs(reinterpret_cast<float4*>(d), make_float4(of[0], of[1], of[2], of[3]));
            __stcs(reinterpret_cast<float4*>(d) + 1, make_float4(of[4], of[5], of[6], of[7]));
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// k_elem: quantize / dequantize with broadcast or expand()ed operands
// ---------------------------------------------------------------------------
constexpr int kElemDims = 4;

struct OperandMap {  // offset = sum_d (i_d / div_d) * str_d
  const void* ptr;
  int32_t is_bf16;
  int32_t uniform_vec;  // scale constant across one vector
  FastDiv div[kElemDims];
  int64_t str[kElemDims];
};

struct ElemArgs {
  const void* in;
  void* out;
  uint32_t nvec;  // vectors in this launch
  uint32_t vec;   // elements per vector
  FastDiv D[kElemDims];  // collapsed output dims (D[3] innermost)
  OperandMap scale, zp;
  int32_t has_zp;
  // rounding of intermediates to bf16 (result dtypes of each binary op)
  int32_t r1_bf16, r2_bf16;
  // dequantize only
  int32_t has_inq, has_outq;
  const uint16_t* inq_table;
  const uint16_t* outq_table;
  vq_rounder inq, outq;
  vq_rounder qr;  // quantize element rounder
};

__device__ __forceinline__ int64_t op_offset(const OperandMap& m, const uint32_t* c) {
  int64_t off = 0;
#pragma unroll
  for (int d = 0; d < kElemDims; ++d) off += (int64_t)m.div[d].div(c[d]) * m.str[d];
  return off;
}

template <bool DEQ, int K>
__device__ __forceinline__ uint32_t elem_op(const ElemArgs& a, float x, uint32_t xbits_bf,
                                            bool x_is_bf, float s, float z,
                                            const uint16_t* stab, float* outf) {
  if (!DEQ) {
    float t = fdiv_rn(x, s);
    if (a.r1_bf16) t = round_bf(t);
    if (a.has_zp) {
      t = fadd_rn(t, z);
      if (a.r2_bf16) t = round_bf(t);
    }
    uint32_t code = round_elem<K>(a.qr, f2bf(t), stab);
    *outf = bf2f(code);
    return code;
  } else {
    float v = x;
    if (a.has_inq) {
      uint32_t idx = x_is_bf ? xbits_bf : f2bf(x);
      v = bf2f(round_any_dev(a.inq, idx, a.inq_table));
    }
    if (a.has_zp) {
      v = fsub_rn(v, z);
      if (a.r1_bf16) v = round_bf(v);
    }
    v = fmul_rn(v, s);
    if (a.r2_bf16) v = round_bf(v);
    if (a.has_outq) v = bf2f(round_any_dev(a.outq, f2bf(v), a.outq_table));
    *outf = v;
    return f2bf(v);
  }
}

template <typename TIn, typename TOut, bool DEQ, int K, int VEC>
__global__ void __launch_bounds__(1024) k_elem(const __grid_constant__ ElemArgs a) {
  extern __shared__ __align__(16) uint16_t smem[];
  if (!DEQ) stage_table<K>(a.qr, smem);
  constexpr bool IN_BF = sizeof(TIn) == 2;
  constexpr bool OUT_BF = sizeof(TOut) == 2;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < a.nvec; v += stride) {
    // coordinates of the vector's first element
    uint32_t e = v * VEC;
    uint32_t c[kElemDims];
    uint32_t q3 = a.D[3].div(e);
    c[3] = e - q3 * a.D[3].d;
    uint32_t q2 = a.D[2].div(q3);
    c[2] = q3 - q2 * a.D[2].d;
    uint32_t q1 = a.D[1].div(q2);
    c[1] = q2 - q1 * a.D[1].d;
    c[0] = q1;
    const uint64_t base = (uint64_t)v * VEC;
    TIn xin[VEC];
    if (VEC * sizeof(TIn) == 16) {
      *reinterpret_cast<uint4*>(xin) = __ldcs(reinterpret_cast<const uint4*>(
          reinterpret_cast<const TIn*>(a.in) + base));
    } else if (VEC * sizeof(TIn) == 8) {
      *reinterpret_cast<uint2*>(xin) =
          *reinterpret_cast<const uint2*>(reinterpret_cast<const TIn*>(a.in) + base);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) xin[j] = reinterpret_cast<const TIn*>(a.in)[base + j];
    }
    float s = 0.f, z = 0.f;
    if (a.scale.uniform_vec) s = ld_f(a.scale.ptr, op_offset(a.scale, c), a.scale.is_bf16);
    if (a.has_zp && a.zp.uniform_vec) z = ld_f(a.zp.ptr, op_offset(a.zp, c), a.zp.is_bf16);
    TOut res[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      if (!a.scale.uniform_vec || (a.has_zp && !a.zp.uniform_vec)) {
        uint32_t cj[kElemDims] = {c[0], c[1], c[2], c[3] + j};
        if (!a.scale.uniform_vec) s = ld_f(a.scale.ptr, op_offset(a.scale, cj), a.scale.is_bf16);
        if (a.has_zp && !a.zp.uniform_vec) z = ld_f(a.zp.ptr, op_offset(a.zp, cj), a.zp.is_bf16);
      }
      uint32_t xb;
      float x;
      if (IN_BF) {
        xb = (uint32_t)(*reinterpret_cast<const uint16_t*>(&xin[j]));
        x = bf2f(xb);
      } else {
        x = *reinterpret_cast<const float*>(&xin[j]);
        xb = 0;
      }
      float of;
      uint32_t ob = elem_op<DEQ, K>(a, x, xb, IN_BF, s, z, smem, &of);
      if (OUT_BF) *reinterpret_cast<uint16_t*>(&res[j]) = (uint16_t)ob;
      else *reinterpret_cast<float*>(&res[j]) = of;
    }
    TOut* op = reinterpret_cast<TOut*>(a.out) + base;
    if (VEC * sizeof(TOut) == 16) {
      __stcs(reinterpret_cast<uint4*>(op), *reinterpret_cast<uint4*>(res));
    } else if (VEC * sizeof(TOut) == 32) {
      __stcs(reinterpret_cast<uint4*>(op), reinterpret_cast<uint4*>(res)[0]);
      __stcs(reinterpret_cast<uint4*>(op) + 1, reinterpret_cast<uint4*>(res)[1]);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) op[j] = res[j];
    }
  }
}

}  // namespace vq

// ===========================================================================
// Host side: validation, broadcast plans, launches
// ===========================================================================
using namespace vq;

namespace {

bool is_float_dtype(int d) { return d == VQ_BF16 || d == VQ_F32; }
int64_t numel(const vq_tensor& t) {
  int64_t n = 1;
  for (int i = 0; i < t.ndim; ++i) n *= t.shape[i];
  return n;
}
size_t esize(int d) { return d == VQ_BF16 ? 2 : 4; }

// torch's result dtype for a binary op on float operands: a 0-d operand
// does not promote a dimensioned one.
int promote(int da, int na, int db, int nb) {
  if (nb == 0 && na > 0) return da;
  if (na == 0 && nb > 0) return db;
  return (da == VQ_F32 || db == VQ_F32) ? VQ_F32 : VQ_BF16;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int cuda_status(cudaError_t e) { return e == cudaSuccess ? VQ_OK : VQ_ERR_CUDA; }

// Rounders whose element form is the shared-memory table.
int elem_kind(const vq_rounder* r) {
  if (r == nullptr) return VQ_R_IDENTITY;
  if (r->kind == VQ_R_MINIFLOAT && r->hw == VQ_HW_E4M3) return K_HW_E4M3;
  if (r->kind == VQ_R_MINIFLOAT && r->hw == VQ_HW_E5M2) return K_HW_E5M2;
  if (r->kind == VQ_R_MINIFLOAT && r->hw == VQ_HW_E2M1) return K_HW_E2M1;
  if (r->kind == VQ_R_IDENTITY || r->kind == VQ_R_MINIFLOAT || r->kind == VQ_R_INT)
    return r->kind;
  return VQ_R_TABLE;
}

int check_rounder(const vq_rounder* r) {
  if (r == nullptr) return VQ_OK;
  if (r->kind < VQ_R_IDENTITY || r->kind > VQ_R_TABLE) return VQ_ERR_INVALID;
  if ((r->kind == VQ_R_TABLE || r->kind == VQ_R_POSIT || r->kind == VQ_R_STEP) &&
      r->table == nullptr)
    return VQ_ERR_NULL;
  if (r->kind == VQ_R_TABLE && !aligned16(r->table)) return VQ_ERR_ALIGNMENT;
  if (r->table8 && (!r->palette || !aligned16(r->table8) || !aligned16(r->palette)))
    return VQ_ERR_ALIGNMENT;
  if (r->kind == VQ_R_STEP && (r->nsteps < 0 || r->nsteps > VQ_STEP_MAX)) return VQ_ERR_INVALID;
  return VQ_OK;
}

// Per-dim map of an operand broadcast against an input shape, following
// expand() (quantized.py:158-171) when block_size > 0.
struct DimMap {
  int64_t div, str;
};

int operand_map(const vq_tensor& x, const vq_tensor& s, int64_t bs, DimMap* out) {
  const int n = x.ndim;
  if (s.ndim > n) return VQ_ERR_SHAPE;
  int64_t sshape[VQ_MAX_DIMS], sstride[VQ_MAX_DIMS];
  const int pad = n - s.ndim;
  for (int d = 0; d < n; ++d) sshape[d] = d < pad ? 1 : s.shape[d - pad];
  int64_t st = 1;
  for (int d = n - 1; d >= 0; --d) {
    sstride[d] = st;
    st *= sshape[d];
  }
  for (int d = 0; d < n; ++d) {
    const int64_t X = x.shape[d], S = sshape[d];
    if (S == X) {
      out[d] = {1, S == 1 ? 0 : sstride[d]};
    } else if (bs > 0) {
      if (S * bs < X) return VQ_ERR_SHAPE;  // repeat_interleave cannot reach X
      out[d] = {bs, S == 1 ? 0 : sstride[d]};
    } else if (S == 1) {
      out[d] = {1, 0};
    } else {
      return VQ_ERR_SHAPE;
    }
  }
  return VQ_OK;
}

// Collapse an n-d elementwise problem (contiguous output plus up to two
// mapped operands) to kElemDims dims.
struct Plan {
  int nd;
  int64_t D[VQ_MAX_DIMS];
  DimMap m[2][VQ_MAX_DIMS];
};

int make_plan(const vq_tensor& x, const DimMap* m0, const DimMap* m1, Plan* p) {
  p->nd = 0;
  for (int d = 0; d < x.ndim; ++d) {
    if (x.shape[d] == 1) continue;  // size-1 dims index nothing
    int k = p->nd;
    p->D[k] = x.shape[d];
    p->m[0][k] = m0[d];
    p->m[1][k] = m1 ? m1[d] : DimMap{1, 0};
    // merge with the previous dim when every operand is contiguous across it
    if (k > 0) {
      bool ok = true;
      for (int o = 0; o < 2; ++o) {
        const DimMap& a = p->m[o][k - 1];
        const DimMap& b = p->m[o][k];
        if (a.div != 1 || b.div != 1) ok = false;
        else if (!((a.str == 0 && b.str == 0) || a.str == b.str * p->D[k])) ok = false;
      }
      if (ok) {
        p->D[k - 1] *= p->D[k];
        for (int o = 0; o < 2; ++o) p->m[o][k - 1] = p->m[o][k];
        continue;
      }
    }
    p->nd++;
  }
  if (p->nd == 0) {  // a single element
    p->nd = 1;
    p->D[0] = 1;
    p->m[0][0] = {1, 0};
    p->m[1][0] = {1, 0};
  }
  if (p->nd > kElemDims) return VQ_ERR_UNSUPPORTED;
  // right-align into kElemDims dims
  const int sh = kElemDims - p->nd;
  for (int k = kElemDims - 1; k >= 0; --k) {
    if (k >= sh) {
      p->D[k] = p->D[k - sh];
      p->m[0][k] = p->m[0][k - sh];
      p->m[1][k] = p->m[1][k - sh];
    } else {
      p->D[k] = 1;
      p->m[0][k] = {1, 0};
      p->m[1][k] = {1, 0};
    }
  }
  p->nd = kElemDims;
  return VQ_OK;
}

template <typename TIn, typename TOut, bool DEQ, int K, int VEC>
int launch_elem(ElemArgs& a, cudaStream_t st) {
  auto kern = k_elem<TIn, TOut, DEQ, K, VEC>;
  int smem = (!DEQ && K == VQ_R_TABLE) ? table_smem(a.qr) : 0;
  int threads = 256;
  int sms = num_sms();
  int blocks;
  if (smem) {
    int per_sm = 1;  // 1024-thread CTAs, each holding the table
    if (int e = table_launch_shape(kern, smem, {1024}, &threads, &per_sm)) return e;
    blocks = sms * per_sm;
  } else {
    blocks = sms * resident_ctas(kern, threads);
  }
  int64_t need = ((int64_t)a.nvec + threads - 1) / threads;
  if (need < blocks) blocks = (int)std::max<int64_t>(need, 1);
  kern<<<blocks, threads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

template <typename TIn, typename TOut, bool DEQ, int VEC>
int dispatch_kind(ElemArgs& a, int K, cudaStream_t st) {
  if (DEQ) return launch_elem<TIn, TOut, DEQ, VQ_R_IDENTITY, VEC>(a, st);
  switch (K) {
    case VQ_R_IDENTITY: return launch_elem<TIn, TOut, DEQ, VQ_R_IDENTITY, VEC>(a, st);
    case VQ_R_MINIFLOAT: return launch_elem<TIn, TOut, DEQ, VQ_R_MINIFLOAT, VEC>(a, st);
    case VQ_R_INT: return launch_elem<TIn, TOut, DEQ, VQ_R_INT, VEC>(a, st);
    default: return launch_elem<TIn, TOut, DEQ, VQ_R_TABLE, VEC>(a, st);
  }
}

template <bool DEQ>
int dispatch_types(ElemArgs& a, int in_dt, int out_dt, int K, bool vec_ok, cudaStream_t st) {
  if (in_dt == VQ_BF16 && out_dt == VQ_BF16)
    return vec_ok ? dispatch_kind<uint16_t, uint16_t, DEQ, 8>(a, K, st)
                  : dispatch_kind<uint16_t, uint16_t, DEQ, 1>(a, K, st);
  if (in_dt == VQ_BF16 && out_dt == VQ_F32)
    return vec_ok ? dispatch_kind<uint16_t, float, DEQ, 8>(a, K, st)
                  : dispatch_kind<uint16_t, float, DEQ, 1>(a, K, st);
  if (in_dt == VQ_F32 && out_dt == VQ_F32)
    return vec_ok ? dispatch_kind<float, float, DEQ, 4>(a, K, st)
                  : dispatch_kind<float, float, DEQ, 1>(a, K, st);
  if (in_dt == VQ_F32 && out_dt == VQ_BF16)  // not produced by promotion
    return VQ_ERR_UNSUPPORTED;
  return VQ_ERR_UNSUPPORTED;
}

template <typename TIn, typename TOut, bool DEQ, int K, int VEC, int SL, bool QM>
int launch_2d(Elem2DArgs& a, cudaStream_t st) {
  constexpr int UNROLL = 2;
  auto kern = k_elem2d<TIn, TOut, DEQ, K, VEC, SL, QM, UNROLL>;
  const int smem = (!DEQ && K == VQ_R_TABLE) ? table_smem(a.qr) : 0;
  int threads = 256, sms = num_sms(), blocks;
  if (smem) {
    int per_sm = 1;
    if (int e = table_launch_shape(kern, smem, {1024}, &threads, &per_sm)) return e;
    blocks = sms * per_sm;
  } else {
    blocks = sms * resident_ctas(kern, threads);
  }
  int64_t need = ((int64_t)a.nvec + (int64_t)threads * UNROLL - 1) / ((int64_t)threads * UNROLL);
  if (need < blocks) blocks = (int)std::max<int64_t>(need, 1);
  kern<<<blocks, threads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

template <typename TIn, typename TOut, bool DEQ, int VEC, int SL>
int dispatch_2d_kind(Elem2DArgs& a, int K, cudaStream_t st) {
  if (DEQ) {
    if (a.has_inq || a.has_outq) return launch_2d<TIn, TOut, DEQ, VQ_R_IDENTITY, VEC, SL, true>(a, st);
    return launch_2d<TIn, TOut, DEQ, VQ_R_IDENTITY, VEC, SL, false>(a, st);
  }
  switch (K) {
    case VQ_R_IDENTITY: return launch_2d<TIn, TOut, DEQ, VQ_R_IDENTITY, VEC, SL, false>(a, st);
    case VQ_R_MINIFLOAT: return launch_2d<TIn, TOut, DEQ, VQ_R_MINIFLOAT, VEC, SL, false>(a, st);
    case VQ_R_INT: return launch_2d<TIn, TOut, DEQ, VQ_R_INT, VEC, SL, false>(a, st);
    case K_HW_E4M3: return launch_2d<TIn, TOut, DEQ, K_HW_E4M3, VEC, SL, false>(a, st);
    case K_HW_E5M2: return launch_2d<TIn, TOut, DEQ, K_HW_E5M2, VEC, SL, false>(a, st);
    case K_HW_E2M1: return launch_2d<TIn, TOut, DEQ, K_HW_E2M1, VEC, SL, false>(a, st);
    default: return launch_2d<TIn, TOut, DEQ, VQ_R_TABLE, VEC, SL, false>(a, st);
  }
}

template <typename TIn, typename TOut, bool DEQ, int VEC>
int dispatch_2d_layout(Elem2DArgs& a, int K, int SL, cudaStream_t st) {
  switch (SL) {
    case SL_SCALAR: return dispatch_2d_kind<TIn, TOut, DEQ, VEC, SL_SCALAR>(a, K, st);
    case SL_ROW: return dispatch_2d_kind<TIn, TOut, DEQ, VEC, SL_ROW>(a, K, st);
    default: return dispatch_2d_kind<TIn, TOut, DEQ, VEC, SL_2D>(a, K, st);
  }
}

template <bool DEQ>
int dispatch_2d(Elem2DArgs& a, int in_dt, int out_dt, int K, int SL, bool vec_ok,
                cudaStream_t st) {
  if (in_dt == VQ_BF16 && out_dt == VQ_BF16)
    return vec_ok ? dispatch_2d_layout<uint16_t, uint16_t, DEQ, 8>(a, K, SL, st)
                  : dispatch_2d_layout<uint16_t, uint16_t, DEQ, 1>(a, K, SL, st);
  if (in_dt == VQ_BF16 && out_dt == VQ_F32)
    return vec_ok ? dispatch_2d_layout<uint16_t, float, DEQ, 8>(a, K, SL, st)
                  : dispatch_2d_layout<uint16_t, float, DEQ, 1>(a, K, SL, st);
  if (in_dt == VQ_F32 && out_dt == VQ_F32)
    return vec_ok ? dispatch_2d_layout<float, float, DEQ, 4>(a, K, SL, st)
                  : dispatch_2d_layout<float, float, DEQ, 1>(a, K, SL, st);
  return VQ_ERR_UNSUPPORTED;
}

void fill_map2d(Map2D& m, const void* ptr, int dtype, const DimMap& r, const DimMap& c,
                int vec) {
  m.ptr = ptr;
  m.is_bf16 = dtype == VQ_BF16;
  m.div_r = FastDiv::make((uint32_t)r.div);
  m.div_c = FastDiv::make((uint32_t)c.div);
  m.str_r = r.str;
  m.str_c = c.str;
  m.uniform_vec = (c.str == 0) || (c.div % vec == 0);
}

template <typename TIn, typename TOut, bool DEQ, int K, int SL>
int launch_rows(RowsArgs& a, cudaStream_t st) {
  // the table kinds run one CTA per SM and need the second load in flight;
  // the analytic kinds keep eight CTAs per SM and do better without it
  constexpr int U = (!DEQ && K == VQ_R_TABLE) ? 2 : 1;
  auto kern = k_rows<TIn, TOut, DEQ, K, SL, U>;
  const int smem = (!DEQ && K == VQ_R_TABLE) ? table_smem(a.qr) : 0;
  const int sms = num_sms();
  int threads, blocks;
  if (smem) {
    int per_sm = 1;
    if (int e = table_launch_shape(kern, smem, {1024}, &threads, &per_sm)) return e;
    blocks = sms * per_sm;
  } else {
    threads = 256;
    blocks = sms * resident_ctas(kern, threads);
  }
  if (a.vpr < threads) threads = std::max(32, (a.vpr + 31) / 32 * 32);
  if (blocks > a.nrows) blocks = std::max(a.nrows, 1);
  kern<<<blocks, threads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

template <typename TIn, typename TOut, bool DEQ, int SL>
int dispatch_rows_kind(RowsArgs& a, int K, cudaStream_t st) {
  if (DEQ) return launch_rows<TIn, TOut, DEQ, VQ_R_IDENTITY, SL>(a, st);
  switch (K) {
    case VQ_R_IDENTITY: return launch_rows<TIn, TOut, DEQ, VQ_R_IDENTITY, SL>(a, st);
    case VQ_R_MINIFLOAT: return launch_rows<TIn, TOut, DEQ, VQ_R_MINIFLOAT, SL>(a, st);
    case VQ_R_INT: return launch_rows<TIn, TOut, DEQ, VQ_R_INT, SL>(a, st);
    case K_HW_E4M3: return launch_rows<TIn, TOut, DEQ, K_HW_E4M3, SL>(a, st);
    case K_HW_E5M2: return launch_rows<TIn, TOut, DEQ, K_HW_E5M2, SL>(a, st);
    case K_HW_E2M1: return launch_rows<TIn, TOut, DEQ, K_HW_E2M1, SL>(a, st);
    default: return launch_rows<TIn, TOut, DEQ, VQ_R_TABLE, SL>(a, st);
  }
}

template <bool DEQ, int SL>
int dispatch_rows(RowsArgs& a, int in_dt, int out_dt, int K, cudaStream_t st) {
  if (in_dt == VQ_BF16 && out_dt == VQ_BF16)
    return dispatch_rows_kind<uint16_t, uint16_t, DEQ, SL>(a, K, st);
  if (in_dt == VQ_BF16 && out_dt == VQ_F32)
    return dispatch_rows_kind<uint16_t, float, DEQ, SL>(a, K, st);
  if (in_dt == VQ_F32 && out_dt == VQ_F32)
    return dispatch_rows_kind<float, float, DEQ, SL>(a, K, st);
  return VQ_ERR_UNSUPPORTED;
}

void fill_operand(OperandMap& om, const vq_tensor* t, const DimMap* m, int vec) {
  om.ptr = t ? t->data : nullptr;
  om.is_bf16 = t ? (t->dtype == VQ_BF16) : 0;
  for (int d = 0; d < kElemDims; ++d) {
    om.div[d] = FastDiv::make((uint32_t)m[d].div);
    om.str[d] = m[d].str;
  }
  om.uniform_vec = (m[kElemDims - 1].str == 0) || (m[kElemDims - 1].div % vec == 0);
}

// dequantize(codes, scale, block_size) with bf16 codes and bf16 scales whose
// blocks of 2^shift elements run along the last dim (rows a multiple of the
// block): out = bf16(code * scale), the product exact in float32 and rounded
// once.  8 elements per 16-byte vector, 4 vectors per thread in flight.
__global__ void __launch_bounds__(256) k_deq_blocks_bf16(const uint16_t* __restrict__ in,
                                                         const uint16_t* __restrict__ scale,
                                                         uint16_t* __restrict__ out, uint32_t nvec,
                                                         int shift) {
  constexpr int U = 4;
  const uint32_t nthr = gridDim.x * blockDim.x;
  for (uint32_t v0 = blockIdx.x * blockDim.x + threadIdx.x; v0 < nvec; v0 += U * nthr) {
    uint4 q[U];
    float sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t v = v0 + u * nthr;
      if (v < nvec) {
        q[u] = __ldcs(reinterpret_cast<const uint4*>(in) + v);
        sc[u] = bf2f(scale[((uint64_t)v * 8) >> shift]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t v = v0 + u * nthr;
      if (v >= nvec) continue;
      const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __nv_bfloat162 b = __floats2bfloat162_rn(__fmul_rn(__uint_as_float(w[k] << 16), sc[u]),
                                                 __fmul_rn(__uint_as_float(w[k] & 0xFFFF0000u), sc[u]));
        o[k] = *reinterpret_cast<uint32_t*>(&b);
      }
      __stcs(reinterpret_cast<uint4*>(out) + v, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// The layout k_deq_blocks_bf16 takes; 0 when it does not apply.
int launch_deq_blocks(const vq_tensor* input, const vq_tensor* scale, const vq_tensor* zp,
                      int64_t bs, const vq_rounder* inq, const vq_rounder* outq,
                      const vq_tensor* out, cudaStream_t st, int* status) {
  if (zp || inq || outq || bs < 8 || (bs & (bs - 1))) return 0;
  if (input->dtype != VQ_BF16 || scale->dtype != VQ_BF16 || out->dtype != VQ_BF16) return 0;
  const int nd = input->ndim;
  if (nd < 1 || scale->ndim != nd) return 0;
  const int64_t C = input->shape[nd - 1];
  if (C % bs || scale->shape[nd - 1] != C / bs) return 0;
  for (int d = 0; d < nd - 1; ++d)
    if (scale->shape[d] != input->shape[d]) return 0;
  if (!aligned16(input->data) || !aligned16(out->data)) return 0;
  const int64_t nvec = numel(*input) / 8;
  if (nvec >= ((int64_t)1 << 31) || nvec == 0) return 0;
  int shift = 0;
  while ((1ll << shift) < bs) ++shift;
  const int blocks = (int)std::min<int64_t>(
      (nvec + 255) / 256, (int64_t)num_sms() * resident_ctas(k_deq_blocks_bf16, 256));
  k_deq_blocks_bf16<<<blocks, 256, 0, st>>>((const uint16_t*)input->data,
                                            (const uint16_t*)scale->data, (uint16_t*)out->data,
                                            (uint32_t)nvec, shift);
  *status = cuda_status(cudaGetLastError());
  return 1;
}

// Shared driver of quantize (DEQ=false) and dequantize (DEQ=true).
template <bool DEQ>
int run_elementwise(const vq_tensor* input, const vq_tensor* scale, const vq_tensor* zp,
                    int64_t bs, const vq_rounder* qr, const vq_rounder* inq,
                    const vq_rounder* outq, vq_tensor* out, void* stream) {
  if (!input || !scale || !out) return VQ_ERR_NULL;
  if (!is_float_dtype(input->dtype) || !is_float_dtype(scale->dtype)) return VQ_ERR_UNSUPPORTED;
  if (zp && !is_float_dtype(zp->dtype)) return VQ_ERR_UNSUPPORTED;
  if (input->ndim > VQ_MAX_DIMS || scale->ndim > VQ_MAX_DIMS || input->ndim < 0)
    return VQ_ERR_INVALID;
  int st;
  if ((st = check_rounder(qr)) || (st = check_rounder(inq)) || (st = check_rounder(outq)))
    return st;
  // result dtypes of the chain of binary ops, as eager torch computes them
  int r1, r2;
  if (!DEQ) {
    r1 = promote(input->dtype, input->ndim, scale->dtype, scale->ndim);  // x / s
    r2 = zp ? promote(r1, input->ndim, zp->dtype, zp->ndim) : r1;       // + zp
  } else {
    r1 = zp ? promote(input->dtype, input->ndim, zp->dtype, zp->ndim) : input->dtype;
    r2 = promote(r1, input->ndim, scale->dtype, scale->ndim);
  }
  if (out->dtype != r2) return VQ_ERR_INVALID;
  if (out->ndim != input->ndim) return VQ_ERR_SHAPE;
  for (int d = 0; d < input->ndim; ++d)
    if (out->shape[d] != input->shape[d]) return VQ_ERR_SHAPE;
  const int64_t n = numel(*input);
  if (n == 0) return VQ_OK;
  if (!input->data || !out->data || !scale->data || (zp && !zp->data)) return VQ_ERR_NULL;
  if (DEQ) {
    int dst = 0;
    if (launch_deq_blocks(input, scale, zp, bs, inq, outq, out,
                          reinterpret_cast<cudaStream_t>(stream), &dst))
      return dst;
  }

  DimMap ms[VQ_MAX_DIMS], mz[VQ_MAX_DIMS];
  if ((st = operand_map(*input, *scale, bs, ms))) return st;
  if (zp && (st = operand_map(*input, *zp, bs, mz))) return st;
  Plan p;
  if ((st = make_plan(*input, ms, zp ? mz : nullptr, &p))) return st;

  const int in_dt = input->dtype, out_dt = r2;
  const int vec = in_dt == VQ_BF16 ? 8 : 4;
  bool vec_ok = (p.D[kElemDims - 1] % vec == 0) && aligned16(input->data) && aligned16(out->data);

  if (p.D[0] == 1 && p.D[1] == 1) {
    // [R, C] view: the specialised kernel
    const int64_t R = p.D[2], C = p.D[3];
    const DimMap &sr = p.m[0][2], &sc = p.m[0][3], &zr = p.m[1][2], &zc = p.m[1][3];
    const int SL = (sr.str == 0 && sc.str == 0) ? SL_SCALAR : (sc.str == 0 ? SL_ROW : SL_2D);
    const int use_vec = vec_ok ? vec : 1;
    Elem2DArgs b;
    memset(&b, 0, sizeof(b));
    b.has_zp = zp != nullptr;
    b.r1_bf16 = r1 == VQ_BF16;
    b.r2_bf16 = r2 == VQ_BF16;
    b.exact_div = !DEQ && zp != nullptr && r1 != VQ_BF16;
    if (qr) b.qr = *qr;
    b.has_inq = inq != nullptr;
    b.has_outq = outq != nullptr;
    if (inq) {
      b.inq = *inq;
      b.inq_table = inq->table;
    }
    if (outq) {
      b.outq = *outq;
      b.outq_table = outq->table;
    }
    const int Kq = elem_kind(qr);
    cudaStream_t cs2 = reinterpret_cast<cudaStream_t>(stream);
    // the row kernel: no zero point, no qmaps, 16-byte vectors, scale per
    // tensor / per row / per power-of-two block along the row
    const bool pow2_blk = SL == SL_2D && sc.str == 1 && sc.div >= vec && (sc.div & (sc.div - 1)) == 0;
    if (!zp && !inq && !outq && vec_ok && R * (C / vec) < (1ll << 40) && C / vec < (1ll << 31) &&
        (SL == SL_SCALAR || ((SL == SL_ROW || pow2_blk) && R >= 4 * num_sms())) && sr.div == 1) {
      RowsArgs ra;
      memset(&ra, 0, sizeof(ra));
      ra.in = input->data;
      ra.out = out->data;
      ra.scale = scale->data;
      ra.scale_bf16 = scale->dtype == VQ_BF16;
      ra.nrows = (int32_t)R;
      ra.vpr = (int32_t)(C / vec);
      ra.nvec = R * (C / vec);
      ra.C = C;
      if (SL == SL_SCALAR) {
        // rows carry no meaning for a per-tensor scale: cut the tensor into
        // rows of 2048 vectors so every SM gets work
        const int64_t nv = R * (C / vec);
        ra.vpr = (int32_t)std::min<int64_t>(nv, 2048);
        ra.nrows = (int32_t)((nv + ra.vpr - 1) / ra.vpr);
        ra.C = (int64_t)ra.vpr * vec;
      }
      ra.str_r = sr.str;
      int sh = 0;
      while ((1ll << sh) < sc.div) ++sh;
      ra.shift = sh;
      if (qr) ra.qr = *qr;
      if (SL == SL_SCALAR) return dispatch_rows<DEQ, SL_SCALAR>(ra, in_dt, out_dt, Kq, cs2);
      if (SL == SL_ROW) return dispatch_rows<DEQ, SL_ROW>(ra, in_dt, out_dt, Kq, cs2);
      return dispatch_rows<DEQ, SL_2D>(ra, in_dt, out_dt, Kq, cs2);
    }
    if (C > ((int64_t)1 << 30)) return VQ_ERR_UNSUPPORTED;
    int64_t rows_per = std::max<int64_t>(1, ((int64_t)1 << 30) / C);
    const int64_t od = std::max(sr.div, zr.div);
    rows_per = std::max<int64_t>(od, rows_per - rows_per % od);
    for (int64_t r0 = 0; r0 < R; r0 += rows_per) {
      const int64_t rows = std::min(rows_per, R - r0);
      b.in = reinterpret_cast<const char*>(input->data) + r0 * C * esize(in_dt);
      b.out = reinterpret_cast<char*>(out->data) + r0 * C * esize(out_dt);
      b.nvec = (uint32_t)(rows * C / use_vec);
      b.C = FastDiv::make((uint32_t)C);
      fill_map2d(b.scale, (const char*)scale->data + (r0 / sr.div) * sr.str * esize(scale->dtype),
                 scale->dtype, sr, sc, use_vec);
      if (zp)
        fill_map2d(b.zp, (const char*)zp->data + (r0 / zr.div) * zr.str * esize(zp->dtype),
                   zp->dtype, zr, zc, use_vec);
      if ((st = dispatch_2d<DEQ>(b, in_dt, out_dt, Kq, SL, vec_ok, cs2))) return st;
    }
    return VQ_OK;
  }

  ElemArgs a;
  memset(&a, 0, sizeof(a));
  a.in = input->data;
  a.out = out->data;
  a.has_zp = zp != nullptr;
  // dequantize: r1 is the dtype after "- zp", r2 after "* scale";
  // quantize: r1 after "/ scale", r2 after "+ zp".
  a.r1_bf16 = r1 == VQ_BF16;
  a.r2_bf16 = r2 == VQ_BF16;
  if (qr) a.qr = *qr;
  a.has_inq = inq != nullptr;
  a.has_outq = outq != nullptr;
  if (inq) {
    a.inq = *inq;
    a.inq_table = inq->table;
  }
  if (outq) {
    a.outq = *outq;
    a.outq_table = outq->table;
  }
  const int K = elem_kind(qr);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  // Launch in chunks of whole outer rows so 32-bit indexing holds.
  const int64_t inner = p.D[1] * p.D[2] * p.D[3];
  const int use_vec = vec_ok ? vec : 1;
  int64_t rows_per = std::max<int64_t>(1, ((int64_t)1 << 30) / std::max<int64_t>(inner, 1));
  if (inner > ((int64_t)1 << 30)) return VQ_ERR_UNSUPPORTED;
  // chunk boundaries must keep the outer-dim block mapping intact
  const int64_t od0 = std::max(p.m[0][0].div, p.m[1][0].div);
  rows_per = std::max<int64_t>(od0, rows_per - rows_per % od0);
  for (int64_t r0 = 0; r0 < p.D[0]; r0 += rows_per) {
    const int64_t rows = std::min(rows_per, p.D[0] - r0);
    const int64_t elems = rows * inner;
    a.in = reinterpret_cast<const char*>(input->data) + r0 * inner * esize(in_dt);
    a.out = reinterpret_cast<char*>(out->data) + r0 * inner * esize(out_dt);
    a.nvec = (uint32_t)(elems / use_vec);
    a.vec = use_vec;
    a.D[0] = FastDiv::make((uint32_t)rows);
    for (int d = 1; d < kElemDims; ++d) a.D[d] = FastDiv::make((uint32_t)p.D[d]);
    // operand maps, shifted to this chunk's first outer row
    DimMap sm[kElemDims], zm[kElemDims];
    for (int d = 0; d < kElemDims; ++d) {
      sm[d] = p.m[0][d];
      zm[d] = p.m[1][d];
    }
    vq_tensor sc = *scale;
    sc.data = (char*)scale->data + (r0 / sm[0].div) * sm[0].str * esize(scale->dtype);
    fill_operand(a.scale, &sc, sm, use_vec);
    if (zp) {
      vq_tensor zc = *zp;
      zc.data = (char*)zp->data + (r0 / zm[0].div) * zm[0].str * esize(zp->dtype);
      fill_operand(a.zp, &zc, zm, use_vec);
    } else {
      fill_operand(a.zp, nullptr, zm, use_vec);
    }
    if ((st = dispatch_types<DEQ>(a, in_dt, out_dt, K, vec_ok, cs))) return st;
  }
  return VQ_OK;
}

// Normalised blocked axes (sorted, non-negative) or an error.
int norm_axes(const vq_tensor& x, const int64_t* axes, int naxes, int* out_blocked) {
  for (int d = 0; d < VQ_MAX_DIMS; ++d) out_blocked[d] = 0;
  if (naxes <= 0 || !axes) return VQ_ERR_INVALID;
  for (int i = 0; i < naxes; ++i) {
    int64_t a = axes[i] < 0 ? axes[i] + x.ndim : axes[i];
    if (a < 0 || a >= x.ndim) return VQ_ERR_INVALID;
    out_blocked[a] = 1;
  }
  return VQ_OK;
}

int blocked_shape(const vq_tensor& x, const int* blocked, int64_t bs, vq_tensor* s) {
  s->ndim = x.ndim;
  for (int d = 0; d < x.ndim; ++d)
    s->shape[d] = blocked[d] ? (x.shape[d] + bs - 1) / bs : x.shape[d];
  return VQ_OK;
}

int qmx_last_fast_ok(const vq_tensor& x, const int* blocked, int64_t bs) {
  if (x.ndim < 1) return 0;
  for (int d = 0; d < x.ndim - 1; ++d)
    if (blocked[d]) return 0;
  if (!blocked[x.ndim - 1]) return 0;
  const int vec = x.dtype == VQ_BF16 ? 8 : 4;
  const int64_t C = x.shape[x.ndim - 1];
  if (C % vec || bs % vec) return 0;
  const int64_t nv = bs / vec;
  if (nv > 32 || (nv & (nv - 1))) return 0;
  if (!aligned16(x.data)) return 0;
  const int64_t rows = numel(x) / std::max<int64_t>(C, 1);
  const int64_t nb = (C + bs - 1) / bs;
  if (rows * nb >= ((int64_t)1 << 31) || C >= ((int64_t)1 << 31)) return 0;
  return (int)nv;
}

template <typename TIn, int K, int SK, int TPB, int VPT>
int launch_qmx(QmxArgs& a, cudaStream_t st) {
  // float32 blocks through a staged table: one block per thread (registers
  // decide how many threads stay resident), the next one prefetched to L2
  constexpr int UNROLL = (sizeof(TIn) == 4 && K == VQ_R_TABLE && TPB >= 4) ? 1 : 2;
  auto kern = k_qmx_last<TIn, K, SK, TPB, VPT, UNROLL>;
  int smem = K == VQ_R_TABLE ? table_smem(a.qr) : 0;
  int threads = 256, sms = num_sms(), blocks;
  if (smem) {
    // each resident CTA holds the table: the CTA size that keeps the most
    // threads resident under the shared-memory and register limits
    int per_sm = 1;
    if (int e = table_launch_shape(kern, smem, {1024, 960, 896, 768, 640, 512}, &threads, &per_sm))
      return e;
    blocks = sms * per_sm;
  } else {
    blocks = sms * resident_ctas(kern, threads);
  }
  int64_t need = ((int64_t)a.ngroups * TPB + threads * UNROLL - 1) / (threads * UNROLL);
  if (need < blocks) blocks = (int)std::max<int64_t>(need, 1);
  kern<<<blocks, threads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

// nv = vectors per block: one thread per block up to two vectors, then two
// vectors per thread across nv/2 threads.
template <typename TIn, int K, int SK>
int launch_qmx_tpb(QmxArgs& a, int nv, cudaStream_t st) {
  switch (nv) {
    case 1: return launch_qmx<TIn, K, SK, 1, 1>(a, st);
    case 2: return launch_qmx<TIn, K, SK, 1, 2>(a, st);
    case 4: return launch_qmx<TIn, K, SK, 2, 2>(a, st);
    case 8: return launch_qmx<TIn, K, SK, 4, 2>(a, st);
    case 16: return launch_qmx<TIn, K, SK, 8, 2>(a, st);
    default: return launch_qmx<TIn, K, SK, 16, 2>(a, st);
  }
}

template <typename TIn, int K>
int launch_qmx_sk(QmxArgs& a, int nv, cudaStream_t st) {
  // the power-of-two path never rounds through scale_qmap
  if (a.pow2 || !a.has_sq) return launch_qmx_tpb<TIn, K, 0>(a, nv, st);
  if (a.sq.kind == VQ_R_MINIFLOAT) return launch_qmx_tpb<TIn, K, 1>(a, nv, st);
  return launch_qmx_tpb<TIn, K, 2>(a, nv, st);
}

template <typename TIn>
int launch_qmx_kind(QmxArgs& a, int K, int nv, cudaStream_t st) {
  switch (K) {
    case VQ_R_IDENTITY: return launch_qmx_sk<TIn, VQ_R_IDENTITY>(a, nv, st);
    case VQ_R_MINIFLOAT: return launch_qmx_sk<TIn, VQ_R_MINIFLOAT>(a, nv, st);
    case VQ_R_INT: return launch_qmx_sk<TIn, VQ_R_INT>(a, nv, st);
    case K_HW_E4M3: return launch_qmx_sk<TIn, K_HW_E4M3>(a, nv, st);
    case K_HW_E5M2: return launch_qmx_sk<TIn, K_HW_E5M2>(a, nv, st);
    case K_HW_E2M1: return launch_qmx_sk<TIn, K_HW_E2M1>(a, nv, st);
    default: return launch_qmx_sk<TIn, VQ_R_TABLE>(a, nv, st);
  }
}

// The NVFP4 configuration k_qmx_nvfp4 takes: returns 0 when it does not
// apply (the caller uses k_qmx_last).
int launch_qmx_nvfp4(const vq_tensor& x, const int* blocked, int64_t bs, int pow2,
                     const vq_rounder* qmap, const vq_rounder* sq, QmxArgs& a, cudaStream_t st,
                     int* status) {
  if (x.dtype != VQ_BF16 || bs != 16 || pow2 || !sq || !qmap) return 0;
  if (elem_kind(qmap) != K_HW_E2M1 || sq->kind != VQ_R_MINIFLOAT || sq->hw != VQ_HW_E4M3) return 0;
  for (int d = 0; d < x.ndim - 1; ++d)
    if (blocked[d]) return 0;
  if (!blocked[x.ndim - 1]) return 0;
  const int64_t C = x.shape[x.ndim - 1];
  if (C % 16 || !aligned16(x.data) || !aligned16(a.codes)) return 0;
  if (!(a.quant_max > 0.0f) || !std::isfinite(a.quant_max)) return 0;
  const int64_t groups = numel(x) / 16;
  if (groups >= ((int64_t)1 << 31)) return 0;
  a.ngroups = (uint32_t)groups;
  // a quant_max of at most 4 significant bits (6.0 for E2M1) divides
  // exactly enough by its reciprocal (see k_qmx_nvfp4)
  uint32_t qb;
  memcpy(&qb, &a.quant_max, 4);
  const bool normal = ((qb >> 23) & 0xFFu) != 0;
  a.rq = normal && (qb & 0x7FFFFu) == 0 ? 1.0f / a.quant_max : 0.0f;
  // exactly the CTAs that fit at once (one wave; the grid-stride loop takes
  // the rest), found once per device and kernel
  auto kern = a.mask_on ? k_qmx_nvfp4<true> : k_qmx_nvfp4<false>;
  int per_sm = 0, threads = 256;
  if (int e = table_launch_shape(kern, 0, {256}, &threads, &per_sm)) {
    *status = e;
    return 1;
  }
  const int blocks = (int)std::min<int64_t>((groups + 255) / 256, (int64_t)num_sms() * per_sm);
  kern<<<blocks, 256, 0, st>>>(a);
  *status = cuda_status(cudaGetLastError());
  return 1;
}

int run_qparam_generic(const vq_tensor* input, const int* blocked, int64_t bs, float qmax,
                       int pow2, int fl2q, const vq_rounder* sq, vq_tensor* scale_out,
                       cudaStream_t st) {
  QparamArgs a;
  memset(&a, 0, sizeof(a));
  int nbl = 0;
  for (int d = 0; d < input->ndim; ++d) nbl += blocked[d];
  if (nbl > 2) return VQ_ERR_UNSUPPORTED;
  a.in = input->data;
  a.scale = scale_out->data;
  a.is_bf16 = input->dtype == VQ_BF16;
  a.ndim = input->ndim;
  int64_t stride = 1;
  for (int d = input->ndim - 1; d >= 0; --d) {
    a.istride[d] = stride;
    stride *= input->shape[d];
    a.ishape[d] = input->shape[d];
    a.sshape[d] = scale_out->shape[d];
    a.blocked[d] = blocked[d];
  }
  a.nscale = numel(*scale_out);
  a.bs = bs;
  a.quant_max = qmax;
  a.pow2 = pow2;
  a.fl2q = fl2q;
  a.has_sq = sq != nullptr;
  if (sq) {
    a.sq = *sq;
    a.sq_table = sq->table;
  }
  if (a.nscale == 0) return VQ_OK;
  int64_t blocks = (a.nscale + 255) / 256;
  if (blocks > INT32_MAX) return VQ_ERR_UNSUPPORTED;
  k_qparam<<<(unsigned)blocks, 256, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

int validate_mx(const vq_tensor* input, const int64_t* axes, int naxes, int64_t bs,
                const vq_rounder* sq, vq_tensor* scale_out, int* blocked) {
  if (!input || !scale_out) return VQ_ERR_NULL;
  if (!is_float_dtype(input->dtype)) return VQ_ERR_UNSUPPORTED;
  if (input->ndim < 1 || input->ndim > VQ_MAX_DIMS) return VQ_ERR_INVALID;
  if (bs <= 0) return VQ_ERR_INVALID;
  int st;
  if ((st = norm_axes(*input, axes, naxes, blocked))) return st;
  if ((st = check_rounder(sq))) return st;
  vq_tensor want;
  blocked_shape(*input, blocked, bs, &want);
  if (scale_out->dtype != input->dtype) return VQ_ERR_INVALID;
  if (scale_out->ndim != want.ndim) return VQ_ERR_SHAPE;
  for (int d = 0; d < want.ndim; ++d)
    if (scale_out->shape[d] != want.shape[d]) return VQ_ERR_SHAPE;
  if (numel(*input) > 0 && (!input->data || !scale_out->data)) return VQ_ERR_NULL;
  return VQ_OK;
}

}  // namespace

extern "C" {

int vq_quantize(const vq_tensor* input, const vq_tensor* scale, const vq_tensor* zero_point,
                int64_t block_size, const vq_rounder* qmap, vq_tensor* out, void* stream) {
  if (!qmap) return VQ_ERR_NULL;
  return run_elementwise<false>(input, scale, zero_point, block_size, qmap, nullptr, nullptr,
                                out, stream);
}

int vq_dequantize(const vq_tensor* input, const vq_tensor* scale, const vq_tensor* zero_point,
                  int64_t block_size, const vq_rounder* input_qmap,
                  const vq_rounder* output_qmap, vq_tensor* out, void* stream) {
  return run_elementwise<true>(input, scale, zero_point, block_size, nullptr, input_qmap,
                               output_qmap, out, stream);
}

int vq_calculate_mx_qparam(const vq_tensor* input, const int64_t* axes, int32_t naxes,
                           int64_t block_size, float quant_max, int32_t pow2,
                           int32_t floor_log2_qmax, const vq_rounder* scale_qmap,
                           vq_tensor* scale_out, void* stream) {
  int blocked[VQ_MAX_DIMS];
  int st = validate_mx(input, axes, naxes, block_size, scale_qmap, scale_out, blocked);
  if (st) return st;
  if (numel(*input) == 0) return VQ_OK;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const int nv = qmx_last_fast_ok(*input, blocked, block_size);
  if (nv && aligned16(scale_out->data)) {
    QmxArgs a;
    memset(&a, 0, sizeof(a));
    const int64_t C = input->shape[input->ndim - 1];
    const int64_t nb = (C + block_size - 1) / block_size;
    a.in = input->data;
    a.codes = nullptr;
    a.scale = scale_out->data;
    a.C = (uint32_t)C;
    a.bs = (uint32_t)block_size;
    a.nb = FastDiv::make((uint32_t)nb);
    a.ngroups = (uint32_t)(numel(*input) / C * nb);
    a.quant_max = quant_max;
    a.pow2 = pow2;
    a.fl2q = floor_log2_qmax;
    a.has_sq = scale_qmap != nullptr;
    if (scale_qmap) {
      a.sq = *scale_qmap;
      a.sq_table = scale_qmap->table;
    }
    a.qr.kind = VQ_R_IDENTITY;
    return input->dtype == VQ_BF16 ? launch_qmx_kind<uint16_t>(a, VQ_R_IDENTITY, nv, cs)
                                   : launch_qmx_kind<float>(a, VQ_R_IDENTITY, nv, cs);
  }
  return run_qparam_generic(input, blocked, block_size, quant_max, pow2, floor_log2_qmax,
                            scale_qmap, scale_out, cs);
}

int vq_quantize_mx(const vq_tensor* input, const vq_rounder* qmap, const int64_t* axes,
                   int32_t naxes, int64_t block_size, float quant_max, int32_t pow2,
                   int32_t floor_log2_qmax, const vq_rounder* scale_qmap, vq_tensor* scale_out,
                   vq_tensor* codes_out, void* stream) {
  if (!qmap || !codes_out) return VQ_ERR_NULL;
  int blocked[VQ_MAX_DIMS];
  int st = validate_mx(input, axes, naxes, block_size, scale_qmap, scale_out, blocked);
  if (st) return st;
  if ((st = check_rounder(qmap))) return st;
  if (codes_out->dtype != input->dtype || codes_out->ndim != input->ndim) return VQ_ERR_SHAPE;
  for (int d = 0; d < input->ndim; ++d)
    if (codes_out->shape[d] != input->shape[d]) return VQ_ERR_SHAPE;
  if (numel(*input) == 0) return VQ_OK;
  if (!codes_out->data) return VQ_ERR_NULL;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const int nv = qmx_last_fast_ok(*input, blocked, block_size);
  if (nv && aligned16(codes_out->data)) {
    QmxArgs a;
    memset(&a, 0, sizeof(a));
    const int64_t C = input->shape[input->ndim - 1];
    const int64_t nb = (C + block_size - 1) / block_size;
    a.in = input->data;
    a.codes = codes_out->data;
    a.scale = scale_out->data;
    a.C = (uint32_t)C;
    a.bs = (uint32_t)block_size;
    a.nb = FastDiv::make((uint32_t)nb);
    a.ngroups = (uint32_t)(numel(*input) / C * nb);
    a.quant_max = quant_max;
    a.pow2 = pow2;
    a.fl2q = floor_log2_qmax;
    a.has_sq = scale_qmap != nullptr;
    if (scale_qmap) {
      a.sq = *scale_qmap;
      a.sq_table = scale_qmap->table;
    }
    a.qr = *qmap;
    const int K = elem_kind(qmap);
    int nst = 0;
    if (launch_qmx_nvfp4(*input, blocked, block_size, pow2, qmap, scale_qmap, a, cs, &nst))
      return nst;
    return input->dtype == VQ_BF16 ? launch_qmx_kind<uint16_t>(a, K, nv, cs)
                                   : launch_qmx_kind<float>(a, K, nv, cs);
  }
  // generic: scales, then an expand()ed quantize
  if ((st = run_qparam_generic(input, blocked, block_size, quant_max, pow2, floor_log2_qmax,
                               scale_qmap, scale_out, cs)))
    return st;
  return run_elementwise<false>(input, scale_out, nullptr, block_size, qmap, nullptr, nullptr,
                                codes_out, stream);
}

int vq_quantize_mx_packed(const vq_tensor* input, const vq_rounder* qmap, int32_t floor_log2_qmax,
                          vq_tensor* scale_out, vq_tensor* codes_out, void* packed_codes,
                          void* packed_sf, void* stream) {
  if (!input || !qmap || !scale_out || !codes_out || !packed_codes || !packed_sf)
    return VQ_ERR_NULL;
  if (input->dtype != VQ_BF16 || input->ndim != 2) return VQ_ERR_UNSUPPORTED;
  if (elem_kind(qmap) != K_HW_E4M3) return VQ_ERR_UNSUPPORTED;
  const int64_t R = input->shape[0], C = input->shape[1];
  if (C % 128 != 0 || R <= 0) return VQ_ERR_UNSUPPORTED;
  const int64_t axes[1] = {-1};
  int blocked[VQ_MAX_DIMS];
  int st = validate_mx(input, axes, 1, 32, nullptr, scale_out, blocked);
  if (st) return st;
  if (codes_out->dtype != VQ_BF16 || codes_out->ndim != 2 || codes_out->shape[0] != R ||
      codes_out->shape[1] != C)
    return VQ_ERR_SHAPE;
  const int nv = qmx_last_fast_ok(*input, blocked, 32);
  if (!nv || !aligned16(codes_out->data) || !aligned16(packed_codes) || !aligned16(packed_sf))
    return VQ_ERR_ALIGNMENT;
  QmxArgs a;
  memset(&a, 0, sizeof(a));
  a.in = input->data;
  a.codes = codes_out->data;
  a.scale = scale_out->data;
  a.C = (uint32_t)C;
  a.bs = 32;
  a.nb = FastDiv::make((uint32_t)(C / 32));
  a.ngroups = (uint32_t)(R * (C / 32));
  a.quant_max = 448.0f;
  a.pow2 = 1;
  a.fl2q = floor_log2_qmax;
  a.qr = *qmap;
  a.packed = (uint8_t*)packed_codes;
  a.packed_sf = (uint8_t*)packed_sf;
  a.packed_rt = (int32_t)((R + 127) / 128);
  return launch_qmx_kind<uint16_t>(a, K_HW_E4M3, nv, reinterpret_cast<cudaStream_t>(stream));
}

int vq_quantize_mx_masked(const vq_tensor* input, const vq_rounder* qmap, int64_t block_size,
                          float quant_max, int32_t pow2, int32_t floor_log2_qmax,
                          const vq_rounder* scale_qmap, double threshold, vq_tensor* scale_out,
                          vq_tensor* codes_out, void* packed_codes, void* packed_sf,
                          void* stream) {
  if (!input || !qmap || !codes_out) return VQ_ERR_NULL;
  const int64_t axes[1] = {-1};
  int blocked[VQ_MAX_DIMS];
  int st = validate_mx(input, axes, 1, block_size, scale_qmap, scale_out, blocked);
  if (st) return st;
  if ((st = check_rounder(qmap))) return st;
  if (codes_out->dtype != input->dtype || codes_out->ndim != input->ndim) return VQ_ERR_SHAPE;
  for (int d = 0; d < input->ndim; ++d)
    if (codes_out->shape[d] != input->shape[d]) return VQ_ERR_SHAPE;
  if (numel(*input) == 0) return VQ_OK;
  if (!codes_out->data) return VQ_ERR_NULL;
  const int nv = qmx_last_fast_ok(*input, blocked, block_size);
  if (!nv || !aligned16(codes_out->data)) return VQ_ERR_UNSUPPORTED;
  const int K = elem_kind(qmap);
  const int64_t C = input->shape[input->ndim - 1];
  const int64_t rows = numel(*input) / C;
  const bool pack = packed_codes || packed_sf;
  if (pack) {
    // the MXFP8 GEMM operand, as vq_quantize_mx_packed writes it
    if (!packed_codes || !packed_sf) return VQ_ERR_NULL;
    if (input->dtype != VQ_BF16 || K != K_HW_E4M3 || block_size != 32 || !pow2 || scale_qmap ||
        C % 128 != 0)
      return VQ_ERR_UNSUPPORTED;
    if (!aligned16(packed_codes) || !aligned16(packed_sf)) return VQ_ERR_ALIGNMENT;
  }
  QmxArgs a;
  memset(&a, 0, sizeof(a));
  const int64_t nb = (C + block_size - 1) / block_size;
  a.in = input->data;
  a.codes = codes_out->data;
  a.scale = scale_out->data;
  a.C = (uint32_t)C;
  a.bs = (uint32_t)block_size;
  a.nb = FastDiv::make((uint32_t)nb);
  a.ngroups = (uint32_t)(rows * nb);
  a.quant_max = quant_max;
  a.pow2 = pow2;
  a.fl2q = floor_log2_qmax;
  a.has_sq = scale_qmap != nullptr;
  if (scale_qmap) {
    a.sq = *scale_qmap;
    a.sq_table = scale_qmap->table;
  }
  a.qr = *qmap;
  if (pack) {
    a.packed = (uint8_t*)packed_codes;
    a.packed_sf = (uint8_t*)packed_sf;
    a.packed_rt = (int32_t)((rows + 127) / 128);
  }
  a.mask_on = 1;
  a.mask_lo1 = vq_outlier_threshold_bits(threshold, input->dtype);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  int nst = 0;
  if (!pack && launch_qmx_nvfp4(*input, blocked, block_size, pow2, qmap, scale_qmap, a, cs, &nst))
    return nst;
  return input->dtype == VQ_BF16 ? launch_qmx_kind<uint16_t>(a, K, nv, cs)
                                 : launch_qmx_kind<float>(a, K, nv, cs);
}

int vq_rounder_check_hw(const vq_rounder* r, int32_t* d_mismatches, void* stream) {
  if (!r || !d_mismatches || !r->table) return VQ_ERR_NULL;
  if (r->kind != VQ_R_MINIFLOAT || r->hw < VQ_HW_E4M3 || r->hw > VQ_HW_E2M1) return VQ_ERR_INVALID;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(d_mismatches, 0, sizeof(int32_t), cs) != cudaSuccess) return VQ_ERR_CUDA;
  k_check_hw<<<128, 256, 0, cs>>>(*r, d_mismatches);
  return cuda_status(cudaGetLastError());
}

int vq_quantize_affine_qparams(const vq_tensor* input, const int64_t* axes, int32_t naxes,
                               int64_t block_size, float quant_min, float quant_max,
                               const vq_rounder* scale_qmap, vq_tensor* scale_out,
                               vq_tensor* zero_point_out, void* stream) {
  if (naxes != 1) return VQ_ERR_INVALID;
  if (!zero_point_out) return VQ_ERR_NULL;
  int blocked[VQ_MAX_DIMS];
  int st = validate_mx(input, axes, naxes, block_size, scale_qmap, scale_out, blocked);
  if (st) return st;
  if (zero_point_out->dtype != scale_out->dtype || zero_point_out->ndim != scale_out->ndim)
    return VQ_ERR_SHAPE;
  for (int d = 0; d < scale_out->ndim; ++d)
    if (zero_point_out->shape[d] != scale_out->shape[d]) return VQ_ERR_SHAPE;
  if (numel(*input) == 0) return VQ_OK;
  if (!zero_point_out->data) return VQ_ERR_NULL;
  AffineArgs aa;
  memset(&aa, 0, sizeof(aa));
  QparamArgs& a = aa.q;
  a.in = input->data;
  a.scale = scale_out->data;
  a.is_bf16 = input->dtype == VQ_BF16;
  a.ndim = input->ndim;
  int64_t stride = 1;
  for (int d = input->ndim - 1; d >= 0; --d) {
    a.istride[d] = stride;
    stride *= input->shape[d];
    a.ishape[d] = input->shape[d];
    a.sshape[d] = scale_out->shape[d];
    a.blocked[d] = blocked[d];
  }
  a.nscale = numel(*scale_out);
  a.bs = block_size;
  a.has_sq = scale_qmap != nullptr;
  if (scale_qmap) {
    a.sq = *scale_qmap;
    a.sq_table = scale_qmap->table;
  }
  aa.zp = zero_point_out->data;
  aa.qmin = quant_min;
  aa.qmax = quant_max;
  int64_t blocks = (a.nscale + 255) / 256;
  if (blocks > INT32_MAX) return VQ_ERR_UNSUPPORTED;
  k_affine_qparam<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(aa);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
