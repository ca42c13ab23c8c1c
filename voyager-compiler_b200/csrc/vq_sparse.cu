// The outlier CSR side-stream of quantized_ops (quantized.py:958-1327):
//
//   k_outlier_count / k_outlier_scan / k_outlier_scatter
//                      filter_outlier in three launches with no waits between
//                      CTAs: outliers (|x| > threshold, x != 0) counted per
//                      tile of 8192 (bf16) / 4096 (f32) elements, the counts
//                      scanned per matrix, then each tile writes its CSR
//                      entries (values, columns) in row-major order, the row
//                      pointers of the rows starting in it, the inliers
//                      (outliers replaced by +0) and its share of the unused
//                      slots -- the order to_sparse_csr produces.
//   k_spmm_rows        spmm_csr's row bounds: cummax(clamp(indptr - indptr[0],
//                      0, L)), exactly the reference's rebasing.
//   k_spmm_csr         spmm_csr: out[r, :] = sum_j data[j] * B[col_j, :] with
//                      B row-major [K, N], accumulated in float32 in CSR order
//                      as the reference's CPU sparse mm does: a chain of fused
//                      multiply-adds, or for widths 4..24 (multiples of 4)
//                      rounded products added in pairs, four entries per
//                      step; rounded once to B's dtype.
//   k_slice_rows       slice_csr_tensor along dim 0
//   k_slice_count / k_slice_scan / k_slice_write
//                      slice_csr_tensor along dim 1 (column window)
//   k_transpose        [.., R, C] -> [.., C, R] (a KC-stored weight becomes the
//                      row-major B of spmm_csr once, then stays cached)
//
// Overflow follows _pad_csr (quantized.py:964-990): entries past the
// capacity are dropped, row pointers clamped to it, unused slots hold
// value 0 and column -1.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <cmath>

#include "voyager_b200.h"
#include "vq_numerics.cuh"

namespace vq {
namespace sparse {

constexpr uint32_t FULL = 0xFFFFFFFFu;
constexpr int F_THREADS = 256;
constexpr int F_WARPS = F_THREADS / 32;
// elements per thread (64 bytes) and per tile
__host__ __device__ constexpr int f_ept(bool bf) { return bf ? 32 : 16; }
__host__ __device__ constexpr int f_tile(bool bf) { return F_THREADS * f_ept(bf); }
__device__ __forceinline__ int64_t imin(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ int64_t imax(int64_t a, int64_t b) { return a > b ? a : b; }

int cuda_status(cudaError_t e) { return e == cudaSuccess ? VQ_OK : VQ_ERR_CUDA; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
int64_t numel(const vq_tensor& t) {
  int64_t n = 1;
  for (int d = 0; d < t.ndim; ++d) n *= t.shape[d];
  return n;
}
int esize(int dt) { return dt == VQ_BF16 ? 2 : 4; }
int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

// ---------------------------------------------------------------------------
// filter_outlier
// ---------------------------------------------------------------------------
struct FilterArgs {
  const void* in;
  void* inliers;  // may be null
  void* data;
  int32_t* indices;
  int32_t* indptr;
  uint32_t* tile_cnt;  // [nb * tiles] outliers per tile
  uint32_t* tile_off;  // [nb * tiles] exclusive prefix within the matrix
  uint32_t* total;     // [nb] outliers per matrix
  uint64_t RC;  // elements per matrix
  uint32_t R, C;
  uint32_t tiles;  // tiles per matrix
  int64_t max_nnz;
  uint32_t offset;  // indptr_offset (added modulo 2^32, as int32 addition wraps)
  uint32_t lo1;     // outlier <=> lo1 <= |x| bits <= +inf bits
  int32_t vec;      // 16-byte loads and stores allowed
};

// Thread `tid` of tile `t` of matrix `b`: its EPT elements (from element e0
// of the matrix) as 16 words of raw bits, and how many of them exist.
template <bool BF>
__device__ __forceinline__ void load_tile(const FilterArgs& a, uint32_t b, uint32_t t, int tid,
                                          uint32_t (&w)[16], uint64_t& e0, uint32_t& nvalid,
                                          uint64_t& first) {
  constexpr int F_EPT = f_ept(BF);
  constexpr int VE = BF ? 8 : 4;
  constexpr int ES = BF ? 2 : 4;
  e0 = (uint64_t)t * f_tile(BF) + (uint64_t)tid * F_EPT;
  nvalid = e0 < a.RC ? (uint32_t)imin(F_EPT, (int64_t)(a.RC - e0)) : 0u;
  first = (uint64_t)b * a.RC + e0;
#pragma unroll
  for (int k = 0; k < 16; ++k) w[k] = 0;
  if (a.vec) {
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(a.in) + first * ES);
#pragma unroll
    for (int v = 0; v < 4; ++v)
      if ((uint32_t)(v * VE) < nvalid) {
        const uint4 q = src[v];
        w[4 * v] = q.x, w[4 * v + 1] = q.y, w[4 * v + 2] = q.z, w[4 * v + 3] = q.w;
      }
  } else {
#pragma unroll
    for (int i = 0; i < F_EPT; ++i)
      if ((uint32_t)i < nvalid) {
        if (BF) {
          const uint32_t h = reinterpret_cast<const uint16_t*>(a.in)[first + i];
          w[i / 2] |= h << (16 * (i & 1));
        } else {
          w[i] = reinterpret_cast<const uint32_t*>(a.in)[first + i];
        }
      }
  }
}

// Bit i set <=> element i is stored in the CSR (outlier and nonzero); with
// INL the words become the inliers (outliers replaced by +0).
template <bool BF, bool INL>
__device__ __forceinline__ uint32_t csr_bits(uint32_t (&w)[16], uint32_t lo1, uint32_t nvalid) {
  const uint32_t lo1c = max(lo1, 1u);
  uint32_t bits = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    if (BF) {
      const uint32_t ab = w[k] & 0x7FFF7FFFu;
      const uint32_t fin = __vcmpleu2(ab, 0x7F807F80u);
      const uint32_t mc = __vcmpgeu2(ab, lo1c * 0x10001u) & fin;
      bits |= ((mc & 1u) | ((mc >> 15) & 2u)) << (2 * k);
      if (INL) w[k] &= ~(__vcmpgeu2(ab, lo1 * 0x10001u) & fin);
    } else {
      const uint32_t ab = w[k] & 0x7FFFFFFFu;
      const bool fin = ab <= 0x7F800000u;
      bits |= (uint32_t)(fin && ab >= lo1c) << k;
      if (INL && fin && ab >= lo1) w[k] = 0;
    }
  }
  if ((uint32_t)f_ept(BF) > nvalid) bits &= (1u << nvalid) - 1u;
  return bits;
}

// block-wide sum (F_THREADS threads)
__device__ __forceinline__ uint32_t block_sum(uint32_t x, uint32_t* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(FULL, x, o);
  if (lane == 0) s_warp[warp] = x;
  __syncthreads();
  uint32_t t = 0;
#pragma unroll
  for (int i = 0; i < F_WARPS; ++i) t += s_warp[i];
  return t;
}

// Persistent: CTA c counts tiles c, c + grid, ...; the next tile's loads
// are in flight while the current one is reduced.
template <bool BF>
__global__ void __launch_bounds__(F_THREADS) k_outlier_count(const __grid_constant__ FilterArgs a,
                                                             uint32_t ntiles) {
  __shared__ uint32_t s_warp[2][F_WARPS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t g = blockIdx.x;
  if (g >= ntiles) return;
  uint32_t w[16];
  uint64_t e0, first;
  uint32_t nvalid;
  load_tile<BF>(a, g / a.tiles, g % a.tiles, threadIdx.x, w, e0, nvalid, first);
  for (int buf = 0; g < ntiles; buf ^= 1) {
    uint32_t n = __popc(csr_bits<BF, false>(w, a.lo1, nvalid));
    const uint32_t gn = g + gridDim.x;
    if (gn < ntiles) load_tile<BF>(a, gn / a.tiles, gn % a.tiles, threadIdx.x, w, e0, nvalid, first);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) n += __shfl_xor_sync(FULL, n, o);
    if (lane == 0) s_warp[buf][warp] = n;
    __syncthreads();  // s_warp[buf] complete; s_warp[buf ^ 1] free again
    if (threadIdx.x == 0) {
      uint32_t t = 0;
#pragma unroll
      for (int i = 0; i < F_WARPS; ++i) t += s_warp[buf][i];
      a.tile_cnt[g] = t;
    }
    g = gn;
  }
}

// exclusive prefix of the tile counts of matrix blockIdx.x; one CTA each
__global__ void __launch_bounds__(1024) k_outlier_scan(const __grid_constant__ FilterArgs a) {
  __shared__ uint32_t s_w[32];
  __shared__ uint32_t s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint64_t base = (uint64_t)blockIdx.x * a.tiles;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (uint32_t c = 0; c < a.tiles; c += 1024) {
    const uint32_t i = c + tid;
    const uint32_t x = i < a.tiles ? a.tile_cnt[base + i] : 0u;
    uint32_t v = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(FULL, v, o);
      if (lane >= o) v += y;
    }
    if (lane == 31) s_w[warp] = v;
    __syncthreads();
    if (warp == 0) {
      uint32_t z = s_w[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(FULL, z, o);
        if (lane >= o) z += y;
      }
      s_w[lane] = z;
    }
    __syncthreads();
    const uint32_t carry = s_carry;
    const uint32_t incl = v + (warp > 0 ? s_w[warp - 1] : 0u) + carry;
    if (i < a.tiles) a.tile_off[base + i] = incl - x;
    __syncthreads();
    if (tid == 1023) s_carry = incl;
    __syncthreads();
  }
  if (tid == 0) a.total[blockIdx.x] = s_carry;
}

// One tile per CTA; thread i holds elements [EPT i, EPT i + EPT) of the tile.
template <bool BF>
__global__ void __launch_bounds__(F_THREADS) k_outlier_scatter(const __grid_constant__ FilterArgs a) {
  constexpr int F_EPT = f_ept(BF);
  constexpr int VE = BF ? 8 : 4;
  constexpr int ES = BF ? 2 : 4;
  __shared__ uint32_t s_warp[F_WARPS];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t g = blockIdx.x, b = g / a.tiles, t = g - b * a.tiles;
  uint32_t w[16];
  uint64_t e0, first;
  uint32_t nvalid;
  load_tile<BF>(a, b, t, tid, w, e0, nvalid, first);
  const uint32_t csrbits = a.inliers ? csr_bits<BF, true>(w, a.lo1, nvalid)
                                     : csr_bits<BF, false>(w, a.lo1, nvalid);
  // block-wide exclusive scan of the per-thread counts
  const uint32_t cnt = __popc(csrbits);
  uint32_t inc = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(FULL, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  uint32_t wofs = 0;
#pragma unroll
  for (int i = 0; i < F_WARPS; ++i) wofs += i < warp ? s_warp[i] : 0u;
  const uint32_t pos0 = a.tile_off[g] + wofs + inc - cnt;
  const uint64_t slot0 = (uint64_t)b * (uint64_t)a.max_nnz;

  // unused slots of this matrix: value 0, column -1 (each tile a share)
  {
    const int64_t nse = a.total[b];
    for (int64_t p = nse + (int64_t)t * F_THREADS + tid; p < a.max_nnz;
         p += (int64_t)a.tiles * F_THREADS) {
      if (BF) reinterpret_cast<uint16_t*>(a.data)[slot0 + p] = 0;
      else reinterpret_cast<uint32_t*>(a.data)[slot0 + p] = 0;
      a.indices[slot0 + p] = -1;
    }
  }
  if (!nvalid) return;

  if (a.inliers) {
    if (a.vec) {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.inliers) + first * ES);
#pragma unroll
      for (int v = 0; v < 4; ++v)
        if ((uint32_t)(v * VE) < nvalid)
          dst[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < F_EPT; ++i)
        if ((uint32_t)i < nvalid) {
          if (BF)
            reinterpret_cast<uint16_t*>(a.inliers)[first + i] =
                (uint16_t)(w[i / 2] >> (16 * (i & 1)));
          else
            reinterpret_cast<uint32_t*>(a.inliers)[first + i] = w[i];
        }
    }
  }

  const uint64_t r0 = e0 / a.C;
  const uint32_t c0 = (uint32_t)(e0 - r0 * a.C);
  // the CSR entries of this thread's elements (few: outliers are rare)
  if (csrbits) {
    uint32_t bits = csrbits, p = pos0;
    while (bits) {
      const int i = __ffs(bits) - 1;
      bits &= bits - 1;
      if ((int64_t)p < a.max_nnz) {
        uint32_t col = c0 + (uint32_t)i;
        while (col >= a.C) col -= a.C;
        // the value is the input element, re-read (the register copy may
        // already hold the inlier's zero)
        if (BF)
          reinterpret_cast<uint16_t*>(a.data)[slot0 + p] =
              reinterpret_cast<const uint16_t*>(a.in)[first + i];
        else
          reinterpret_cast<uint32_t*>(a.data)[slot0 + p] =
              reinterpret_cast<const uint32_t*>(a.in)[first + i];
        a.indices[slot0 + p] = (int32_t)col;
      }
      ++p;
    }
  }
  // row pointers of the rows that start inside this thread's elements
  int32_t* ip = a.indptr + (uint64_t)b * (a.R + 1ull);
  uint32_t i = c0 == 0 ? 0u : (a.C - c0 < (uint32_t)F_EPT ? a.C - c0 : (uint32_t)F_EPT);
  uint64_t r = c0 == 0 ? r0 : r0 + 1;
  for (; i < nvalid; i += a.C, ++r) {
    const uint32_t before = pos0 + __popc(csrbits & ((1u << i) - 1u));
    ip[r] = (int32_t)((uint32_t)imin(before, a.max_nnz) + a.offset);
    if (a.C > (uint32_t)F_EPT) break;
  }
  if (e0 + nvalid == a.RC)
    ip[a.R] = (int32_t)((uint32_t)imin(pos0 + cnt, a.max_nnz) + a.offset);
}

__global__ void k_fill_i32(int32_t* p, int64_t n, int32_t v) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// ---------------------------------------------------------------------------
// spmm_csr
// ---------------------------------------------------------------------------
// crow[b][r] = cummax over r' <= r of clamp(indptr[b][r'] - indptr[b][0], 0, L);
// one CTA per matrix, 8 consecutive rows per thread per step.
__global__ void __launch_bounds__(1024) k_spmm_rows(const int32_t* indptr, int64_t rows1, int64_t L,
                                                    int32_t* crow) {
  __shared__ int32_t s_w[32];
  __shared__ int32_t s_carry;
  constexpr int PER = 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int32_t* ip = indptr + (int64_t)blockIdx.x * rows1;
  int32_t* out = crow + (int64_t)blockIdx.x * rows1;
  const int64_t base = ip[0];
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int64_t c = 0; c < rows1; c += 1024 * PER) {
    const int64_t r0 = c + (int64_t)tid * PER;
    int32_t v[PER];
    int32_t m = 0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int64_t r = r0 + k;
      v[k] = r < rows1 ? (int32_t)imin(imax((int64_t)ip[r] - base, 0), L) : 0;
      m = max(m, v[k]);
      v[k] = m;  // running max within the thread's rows
    }
    int32_t x = m;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(FULL, x, o);
      if (lane >= o) x = max(x, y);
    }
    if (lane == 31) s_w[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int32_t z = s_w[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(FULL, z, o);
        if (lane >= o) z = max(z, y);
      }
      s_w[lane] = z;
    }
    __syncthreads();
    // max over everything before this thread's rows
    int32_t before = max(s_carry, warp > 0 ? s_w[warp - 1] : 0);
    const int32_t xl = __shfl_up_sync(FULL, x, 1);
    if (lane > 0) before = max(before, xl);
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int64_t r = r0 + k;
      if (r < rows1) out[r] = max(v[k], before);
    }
    __syncthreads();
    if (tid == 1023) s_carry = max(before, x);
    __syncthreads();
  }
}

struct SpmmArgs {
  const void* data;  // [nb, L]
  const int32_t* indices;
  const int32_t* crow;  // [nb, X + 1] from k_spmm_rows
  const void* B;        // [Kc, N] or [nb, Kc, N]
  void* out;            // [nb, X, N]
  int64_t L, X, Kc, N;
  int32_t b_batched;
  int32_t chunks;  // column chunks per row
  int32_t pairs;   // the CPU kernel's order for widths 4..24 (multiples of 4)
};

constexpr int S_THREADS = 256;

// VEC consecutive elements of row `row` of B, widened to float32
template <bool BBF, int VEC>
__device__ __forceinline__ void b_row(const SpmmArgs& a, int64_t bb, int32_t row, int64_t n0,
                                      float (&x)[VEC]) {
  const int64_t e = bb + (int64_t)row * a.N + n0;
  if (VEC == 8) {  // bf16, 16-byte vectors
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(a.B) + e));
    const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[2 * k] = __uint_as_float(qq[k] << 16);
      x[2 * k + 1] = __uint_as_float(qq[k] & 0xFFFF0000u);
    }
  } else if (VEC == 4) {  // float32, 16-byte vectors
    const float4 q = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.B) + e));
    x[0] = q.x, x[1] = q.y, x[2] = q.z, x[3] = q.w;
  } else {
    x[0] = BBF ? bf2f(reinterpret_cast<const uint16_t*>(a.B)[e]) : reinterpret_cast<const float*>(a.B)[e];
  }
}

// a * b + c rounded once, a and b bfloat16 (exact product), c float32
__device__ __forceinline__ float fma_bf16(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.bf16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
__device__ __forceinline__ void halves(uint32_t w, uint16_t& lo, uint16_t& hi) {
  asm("mov.b32 {%0, %1}, %2;" : "=h"(lo), "=h"(hi) : "r"(w));
}

// One CTA per (row, chunk of S_THREADS * VEC columns), chunk-major so the
// CTAs running together read one column slice of B (kept in L2); the row's
// entries are staged in shared memory 256 at a time and every thread
// accumulates its VEC columns over them in CSR order, 8 B rows in flight.
template <bool DBF, bool BBF, int VEC>
__global__ void __launch_bounds__(S_THREADS) k_spmm_csr(const __grid_constant__ SpmmArgs a) {
  __shared__ float s_v[S_THREADS];
  __shared__ uint16_t s_vb[S_THREADS];
  __shared__ int32_t s_c[S_THREADS];
  const int tid = threadIdx.x;
  const int64_t bid = blockIdx.x;
  const int64_t rows_all = (int64_t)gridDim.x / a.chunks;
  const int64_t chunk = bid / rows_all, rest = bid - chunk * rows_all;
  const int64_t r = rest % a.X, b = rest / a.X;
  const int32_t* cr = a.crow + b * (a.X + 1);
  const int64_t start = cr[r], end = cr[r + 1];
  const int64_t n0 = (chunk * S_THREADS + tid) * VEC;
  const bool live = n0 < a.N;
  const int64_t boff = b * a.L;
  const int64_t bb = a.b_batched ? b * a.Kc * a.N : 0;
  const int64_t q4 = (end - start) / 4 * 4;  // entries in whole groups of four (pairs mode)
  constexpr bool MIXED = DBF && BBF && VEC == 8;
  float acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.0f;
  for (int64_t s0 = start; s0 < end; s0 += S_THREADS) {
    const int cnt = (int)imin(S_THREADS, end - s0);
    __syncthreads();
    if (tid < cnt) {
      const int64_t j = boff + s0 + tid;
      if (DBF) {
        const uint16_t vb = reinterpret_cast<const uint16_t*>(a.data)[j];
        s_vb[tid] = vb;
        s_v[tid] = bf2f(vb);
      } else {
        s_v[tid] = reinterpret_cast<const float*>(a.data)[j];
      }
      const int64_t c = reinterpret_cast<const int32_t*>(a.indices)[j];
      s_c[tid] = (int32_t)imin(imax(c, 0), a.Kc - 1);
    }
    __syncthreads();
    if (!live) continue;
    if (!a.pairs) {
      // fused multiply-add chain
      if (MIXED) {
        const uint16_t* B16 = reinterpret_cast<const uint16_t*>(a.B) + bb + n0;
        int j = 0;
        for (; j + 8 <= cnt; j += 8) {
          uint4 q[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            q[u] = __ldg(reinterpret_cast<const uint4*>(B16 + (int64_t)s_c[j + u] * a.N));
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint16_t v = s_vb[j + u];
            const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint16_t lo, hi;
              halves(w[k], lo, hi);
              acc[2 * k] = fma_bf16(v, lo, acc[2 * k]);
              acc[2 * k + 1] = fma_bf16(v, hi, acc[2 * k + 1]);
            }
          }
        }
        for (; j < cnt; ++j) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(B16 + (int64_t)s_c[j] * a.N));
          const uint16_t v = s_vb[j];
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint16_t lo, hi;
            halves(w[k], lo, hi);
            acc[2 * k] = fma_bf16(v, lo, acc[2 * k]);
            acc[2 * k + 1] = fma_bf16(v, hi, acc[2 * k + 1]);
          }
        }
      } else {
#pragma unroll 4
        for (int j = 0; j < cnt; ++j) {
          float x[VEC];
          b_row<BBF, VEC>(a, bb, s_c[j], n0, x);
          const float v = s_v[j];
#pragma unroll
          for (int i = 0; i < VEC; ++i) acc[i] = fmaf(v, x[i], acc[i]);
        }
      }
      continue;
    }
    // rounded products added in pairs, four entries per step; chunks start
    // at multiples of 256 entries, so only the last holds the 1-3 left over
    const int full = (int)imin(cnt, imax(q4 - (s0 - start), 0));
    for (int j = 0; j < full; j += 4) {
      float x0[VEC], x1[VEC], x2[VEC], x3[VEC];
      b_row<BBF, VEC>(a, bb, s_c[j], n0, x0);
      b_row<BBF, VEC>(a, bb, s_c[j + 1], n0, x1);
      b_row<BBF, VEC>(a, bb, s_c[j + 2], n0, x2);
      b_row<BBF, VEC>(a, bb, s_c[j + 3], n0, x3);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        acc[i] = __fadd_rn(acc[i], __fadd_rn(__fmul_rn(s_v[j], x0[i]), __fmul_rn(s_v[j + 1], x1[i])));
        acc[i] = __fadd_rn(acc[i], __fadd_rn(__fmul_rn(s_v[j + 2], x2[i]), __fmul_rn(s_v[j + 3], x3[i])));
      }
    }
    const int left = cnt - full;
    if (left > 0) {
      float x0[VEC], x1[VEC], x2[VEC];
      b_row<BBF, VEC>(a, bb, s_c[full], n0, x0);
      if (left > 1) b_row<BBF, VEC>(a, bb, s_c[full + 1], n0, x1);
      if (left > 2) b_row<BBF, VEC>(a, bb, s_c[full + 2], n0, x2);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float p0 = __fmul_rn(s_v[full], x0[i]);
        if (left == 1) {
          acc[i] = __fadd_rn(acc[i], p0);
        } else if (left == 2) {
          acc[i] = __fadd_rn(__fadd_rn(acc[i], p0), __fmul_rn(s_v[full + 1], x1[i]));
        } else {
          const float p1 = __fmul_rn(s_v[full + 1], x1[i]), p2 = __fmul_rn(s_v[full + 2], x2[i]);
          acc[i] = __fadd_rn(__fadd_rn(acc[i], p2), __fadd_rn(p0, p1));
        }
      }
    }
  }
  if (!live) return;
  const int64_t o = (b * a.X + r) * a.N + n0;
  if (VEC == 8) {
    uint32_t p[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = (uint32_t)f2bf(acc[2 * k]) | ((uint32_t)f2bf(acc[2 * k + 1]) << 16);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.out) + o) = make_uint4(p[0], p[1], p[2], p[3]);
  } else if (VEC == 4) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + o) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
  } else if (BBF) {
    reinterpret_cast<uint16_t*>(a.out)[o] = (uint16_t)f2bf(acc[0]);
  } else {
    reinterpret_cast<float*>(a.out)[o] = acc[0];
  }
}

template <bool DBF, bool BBF, int VEC>
int launch_spmm(SpmmArgs& a, int64_t nb, cudaStream_t st) {
  a.chunks = (int32_t)((a.N + (int64_t)S_THREADS * VEC - 1) / ((int64_t)S_THREADS * VEC));
  const int64_t blocks = nb * a.X * a.chunks;  // chunk-major: [chunks][nb][X]
  if (blocks == 0) return VQ_OK;
  if (blocks > INT32_MAX) return VQ_ERR_TOO_LARGE;
  k_spmm_csr<DBF, BBF, VEC><<<(unsigned)blocks, S_THREADS, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// slice_csr_tensor
// ---------------------------------------------------------------------------
// Python's slice bounds: a negative bound counts from the end, then both are
// clamped to [0, L].
__device__ __forceinline__ int64_t py_bound(int64_t x, int64_t L) {
  if (x < 0) x += L;
  return x < 0 ? 0 : (x > L ? L : x);
}

template <int ES>
__global__ void k_slice_rows(const void* data, const int32_t* indices, const int32_t* indptr,
                             int64_t L, int64_t start, int64_t end, int64_t max_out,
                             void* new_data, int32_t* new_indices, int32_t* new_indptr) {
  const int64_t s = indptr[start], e = indptr[end];
  const int64_t nse = e - s;
  const int64_t a0 = py_bound(s, L), a1 = py_bound(e, L);
  const int64_t len = a1 > a0 ? a1 - a0 : 0;
  const int64_t n = imax(max_out, end - start + 1);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i <= end - start) {
      const int64_t v = (int64_t)indptr[start + i] - s;
      new_indptr[i] = (int32_t)(nse > max_out ? imin(v, max_out) : v);
    }
    if (i < max_out) {
      const bool in = i < len;
      if (ES == 2)
        reinterpret_cast<uint16_t*>(new_data)[i] =
            in ? reinterpret_cast<const uint16_t*>(data)[a0 + i] : (uint16_t)0;
      else
        reinterpret_cast<uint32_t*>(new_data)[i] =
            in ? reinterpret_cast<const uint32_t*>(data)[a0 + i] : 0u;
      new_indices[i] = in ? indices[a0 + i] : -1;
    }
  }
}

// one warp per row: entries of the row whose column lies in [start, end)
__global__ void k_slice_count(const int32_t* indices, const int32_t* indptr, int64_t rows, int64_t L,
                              int64_t start, int64_t end, int32_t* counts) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t a0 = imax(indptr[r], 0), a1 = imin(indptr[r + 1], L);
  uint32_t n = 0;
  for (int64_t j0 = a0; j0 < a1; j0 += 32) {
    const int64_t j = j0 + lane;
    const bool p = j < a1 && indices[j] >= start && indices[j] < end;
    n += __popc(__ballot_sync(FULL, p));
  }
  if (lane == 0) counts[r] = (int32_t)n;
}

// exclusive prefix of counts -> excl[0..rows] (uncapped) and new_indptr
// (capped at max_out when the total exceeds it); one CTA
__global__ void __launch_bounds__(1024) k_slice_scan(const int32_t* counts, int64_t rows,
                                                     int64_t max_out, int32_t* excl,
                                                     int32_t* new_indptr) {
  __shared__ int32_t s_w[32];
  __shared__ int32_t s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int64_t c = 0; c < rows; c += 1024) {
    const int64_t r = c + tid;
    const int32_t x = r < rows ? counts[r] : 0;
    int32_t v = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(FULL, v, o);
      if (lane >= o) v += y;
    }
    if (lane == 31) s_w[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int32_t z = s_w[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t y = __shfl_up_sync(FULL, z, o);
        if (lane >= o) z += y;
      }
      s_w[lane] = z;
    }
    __syncthreads();
    const int32_t carry = s_carry;
    const int32_t incl = v + (warp > 0 ? s_w[warp - 1] : 0) + carry;
    if (r < rows) excl[r + 1] = incl;
    __syncthreads();
    if (tid == 1023) s_carry = incl;
    __syncthreads();
  }
  if (tid == 0) excl[0] = 0;
  __syncthreads();
  const int64_t total = excl[rows];
  for (int64_t r = tid; r <= rows; r += 1024) {
    const int64_t v = excl[r];
    new_indptr[r] = (int32_t)(total > max_out ? imin(v, max_out) : v);
  }
}

template <int ES>
__global__ void k_slice_write(const void* data, const int32_t* indices, const int32_t* indptr,
                              int64_t rows, int64_t L, int64_t start, int64_t end,
                              const int32_t* excl, int64_t max_out, void* new_data,
                              int32_t* new_indices) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t a0 = imax(indptr[r], 0), a1 = imin(indptr[r + 1], L);
  int64_t pos = excl[r];
  for (int64_t j0 = a0; j0 < a1; j0 += 32) {
    const int64_t j = j0 + lane;
    const int32_t c = j < a1 ? indices[j] : -1;
    const bool p = j < a1 && c >= start && c < end;
    const uint32_t m = __ballot_sync(FULL, p);
    const int64_t q = pos + __popc(m & ((1u << lane) - 1u));
    if (p && q < max_out) {
      if (ES == 2)
        reinterpret_cast<uint16_t*>(new_data)[q] = reinterpret_cast<const uint16_t*>(data)[j];
      else
        reinterpret_cast<uint32_t*>(new_data)[q] = reinterpret_cast<const uint32_t*>(data)[j];
      new_indices[q] = (int32_t)(c - start);
    }
    pos += __popc(m);
  }
}

// ---------------------------------------------------------------------------
// transpose [nb, R, C] -> [nb, C, R] through 32 x 32 shared tiles
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) k_transpose(const T* src, T* dst, int64_t R, int64_t C,
                                                   int64_t tiles_r, int64_t tiles_c) {
  __shared__ T tile[32][33];
  const int64_t t = blockIdx.x;
  const int64_t per = tiles_r * tiles_c;
  const int64_t b = t / per, rem = t - b * per;
  const int64_t tr = rem / tiles_c, tc = rem - tr * tiles_c;
  const T* s = src + b * R * C;
  T* d = dst + b * R * C;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
#pragma unroll
  for (int k = 0; k < 32; k += 8) {
    const int64_t r = tr * 32 + ty + k, c = tc * 32 + tx;
    if (r < R && c < C) tile[ty + k][tx] = s[r * C + c];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 32; k += 8) {
    const int64_t c = tc * 32 + ty + k, r = tr * 32 + tx;
    if (r < R && c < C) d[c * R + r] = tile[tx][ty + k];
  }
}

}  // namespace sparse
}  // namespace vq

using namespace vq::sparse;

namespace {

// The reference compares |x| with the Python float threshold in the
// tensor's dtype: the double is rounded to float32 and, for bfloat16 input,
// again to bfloat16 (round-half-even each time).  Returns lo1 with
// |x| > threshold <=> lo1 <= bits(|x|) <= bits(+inf) for every non-NaN x.
uint32_t outlier_lo1(double threshold, int dtype) {
  const float tf = (float)threshold;
  uint32_t bits;
  memcpy(&bits, &tf, 4);
  const bool bf = dtype == VQ_BF16;
  if (std::isnan(tf)) return bf ? 0x8000u : 0x80000000u;
  if (bf) {
    bits = (bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16;  // finite or inf: RNE to bf16
    if ((bits & 0x8000u) && (bits & 0x7FFFu)) return 0;  // negative: every non-NaN
    return (bits & 0x7FFFu) + 1u;
  }
  if ((bits & 0x80000000u) && (bits & 0x7FFFFFFFu)) return 0;
  return (bits & 0x7FFFFFFFu) + 1u;
}

int matrix_dims(const vq_tensor* t, int64_t* nb, int64_t* R, int64_t* C) {
  if (t->ndim < 2 || t->ndim > VQ_MAX_DIMS) return VQ_ERR_INVALID;
  int64_t n = 1;
  for (int d = 0; d < t->ndim - 2; ++d) n *= t->shape[d];
  *nb = n;
  *R = t->shape[t->ndim - 2];
  *C = t->shape[t->ndim - 1];
  return VQ_OK;
}

int64_t filter_tiles(int64_t R, int64_t C, int dtype) {
  const int64_t tile = f_tile(dtype == VQ_BF16);
  return (R * C + tile - 1) / tile;
}

}  // namespace

extern "C" {

uint32_t vq_outlier_threshold_bits(double threshold, int32_t dtype) {
  return outlier_lo1(threshold, dtype);
}

size_t vq_filter_outlier_workspace_bytes(const vq_tensor* input) {
  int64_t nb, R, C;
  if (!input || matrix_dims(input, &nb, &R, &C)) return 0;
  return (size_t)(2 * nb * filter_tiles(R, C, input->dtype) + nb) * 4 + 16;
}

int vq_filter_outlier(const vq_tensor* input, double threshold, int64_t max_nnz,
                      int32_t indptr_offset, void* data, int32_t* indices, int32_t* indptr,
                      void* inliers, void* workspace, size_t workspace_bytes, int32_t* d_err,
                      void* stream) {
  (void)d_err;  // no device waits: nothing to report
  if (!input || !indptr || !workspace) return VQ_ERR_NULL;
  if (input->dtype != VQ_BF16 && input->dtype != VQ_F32) return VQ_ERR_UNSUPPORTED;
  int64_t nb, R, C;
  int st = matrix_dims(input, &nb, &R, &C);
  if (st) return st;
  if (max_nnz < 0 || nb < 0 || R < 0 || C < 0) return VQ_ERR_INVALID;
  if (R * C >= ((int64_t)1 << 31) || R >= INT32_MAX ||
      nb * filter_tiles(R, C, input->dtype) >= INT32_MAX)
    return VQ_ERR_TOO_LARGE;
  if (nb * max_nnz > 0 && (!data || !indices)) return VQ_ERR_NULL;
  if (nb * R * C > 0 && !input->data) return VQ_ERR_NULL;
  const int64_t tiles = filter_tiles(R, C, input->dtype);
  if (workspace_bytes < (size_t)(2 * nb * tiles + nb) * 4 + 16) return VQ_ERR_TOO_LARGE;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const int es = esize(input->dtype);
  if (nb == 0) return VQ_OK;
  if (R * C == 0) {
    // no elements: every slot unused, every row pointer the offset
    if (nb * max_nnz > 0 &&
        (cudaMemsetAsync(data, 0, (size_t)(nb * max_nnz) * es, cs) != cudaSuccess ||
         cudaMemsetAsync(indices, 0xFF, (size_t)(nb * max_nnz) * 4, cs) != cudaSuccess))
      return VQ_ERR_CUDA;
    const int64_t n = nb * (R + 1);
    k_fill_i32<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, cs>>>(
        indptr, n, indptr_offset);
    return cuda_status(cudaGetLastError());
  }
  FilterArgs a;
  memset(&a, 0, sizeof(a));
  a.in = input->data;
  a.inliers = inliers;
  a.data = data;
  a.indices = indices;
  a.indptr = indptr;
  a.tile_cnt = reinterpret_cast<uint32_t*>(workspace);
  a.tile_off = a.tile_cnt + nb * tiles;
  a.total = a.tile_off + nb * tiles;
  a.RC = (uint64_t)(R * C);
  a.R = (uint32_t)R;
  a.C = (uint32_t)C;
  a.tiles = (uint32_t)tiles;
  a.max_nnz = max_nnz;
  a.offset = (uint32_t)indptr_offset;
  a.lo1 = outlier_lo1(threshold, input->dtype);
  const int ve = 16 / es;
  a.vec = (R * C) % ve == 0 && aligned16(input->data) && (!inliers || aligned16(inliers));
  const unsigned blocks = (unsigned)(nb * tiles);
  const unsigned cblocks = (unsigned)std::min<int64_t>(nb * tiles, (int64_t)num_sms() * 6);
  if (input->dtype == VQ_BF16) k_outlier_count<true><<<cblocks, F_THREADS, 0, cs>>>(a, blocks);
  else k_outlier_count<false><<<cblocks, F_THREADS, 0, cs>>>(a, blocks);
  k_outlier_scan<<<(unsigned)nb, 1024, 0, cs>>>(a);
  if (input->dtype == VQ_BF16) k_outlier_scatter<true><<<blocks, F_THREADS, 0, cs>>>(a);
  else k_outlier_scatter<false><<<blocks, F_THREADS, 0, cs>>>(a);
  return cuda_status(cudaGetLastError());
}

int vq_spmm_csr(const vq_tensor* data, const int32_t* indices, const int32_t* indptr,
                int64_t rows, const vq_tensor* b, vq_tensor* out, int32_t* workspace,
                void* stream) {
  if (!data || !b || !out || !indptr || !workspace) return VQ_ERR_NULL;
  if ((data->dtype != VQ_BF16 && data->dtype != VQ_F32) ||
      (b->dtype != VQ_BF16 && b->dtype != VQ_F32) || out->dtype != b->dtype)
    return VQ_ERR_UNSUPPORTED;
  if (data->ndim != 2 || (b->ndim != 2 && b->ndim != 3) || out->ndim != 3 || rows < 0)
    return VQ_ERR_INVALID;
  const int64_t nb = data->shape[0], L = data->shape[1];
  const int64_t Kc = b->shape[b->ndim - 2], N = b->shape[b->ndim - 1];
  const int b_batched = b->ndim == 3;
  if (b_batched && b->shape[0] != nb) return VQ_ERR_SHAPE;
  if (out->shape[0] != nb || out->shape[1] != rows || out->shape[2] != N) return VQ_ERR_SHAPE;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (nb * rows * N == 0) return VQ_OK;
  if (!out->data) return VQ_ERR_NULL;
  if (Kc == 0 || L == 0) {
    // no column can be addressed: every product is empty
    const int64_t bytes = nb * rows * N * esize(out->dtype);
    return cuda_status(cudaMemsetAsync(out->data, 0, (size_t)bytes, cs));
  }
  if (!data->data || !indices || !b->data) return VQ_ERR_NULL;
  if (nb > INT32_MAX) return VQ_ERR_TOO_LARGE;
  k_spmm_rows<<<(unsigned)nb, 1024, 0, cs>>>(indptr, rows + 1, L, workspace);
  int st = cuda_status(cudaGetLastError());
  if (st) return st;
  SpmmArgs a;
  memset(&a, 0, sizeof(a));
  a.data = data->data;
  a.indices = indices;
  a.crow = workspace;
  a.B = b->data;
  a.out = out->data;
  a.L = L;
  a.X = rows;
  a.Kc = Kc;
  a.N = N;
  a.b_batched = b_batched;
  a.pairs = N % 4 == 0 && N >= 4 && N <= 24;
  const bool dbf = data->dtype == VQ_BF16, bbf = b->dtype == VQ_BF16;
  const int ve = bbf ? 8 : 4;
  const bool vec = N % ve == 0 && aligned16(b->data) && aligned16(out->data);
  if (dbf) {
    if (bbf) return vec ? launch_spmm<true, true, 8>(a, nb, cs) : launch_spmm<true, true, 1>(a, nb, cs);
    return vec ? launch_spmm<true, false, 4>(a, nb, cs) : launch_spmm<true, false, 1>(a, nb, cs);
  }
  if (bbf) return vec ? launch_spmm<false, true, 8>(a, nb, cs) : launch_spmm<false, true, 1>(a, nb, cs);
  return vec ? launch_spmm<false, false, 4>(a, nb, cs) : launch_spmm<false, false, 1>(a, nb, cs);
}

int vq_slice_csr(const vq_tensor* data, const int32_t* indices, const int32_t* indptr,
                 int64_t rows, int32_t dim, int64_t start, int64_t end, int64_t max_out,
                 void* new_data, int32_t* new_indices, int32_t* new_indptr, int32_t* workspace,
                 void* stream) {
  if (!data || !indptr || !new_indptr) return VQ_ERR_NULL;
  if (data->dtype != VQ_BF16 && data->dtype != VQ_F32) return VQ_ERR_UNSUPPORTED;
  if (data->ndim != 1 || rows < 0 || max_out < 0) return VQ_ERR_INVALID;
  if (max_out > 0 && (!new_data || !new_indices)) return VQ_ERR_NULL;
  const int64_t L = data->shape[0];
  if (L > 0 && (!data->data || !indices)) return VQ_ERR_NULL;
  const int es = esize(data->dtype);
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (dim == 0) {
    if (start < 0 || end < start || end > rows) return VQ_ERR_INVALID;
    const int64_t n = std::max<int64_t>(max_out, end - start + 1);
    const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 8192);
    if (es == 2)
      k_slice_rows<2><<<blocks, 256, 0, cs>>>(data->data, indices, indptr, L, start, end, max_out,
                                              new_data, new_indices, new_indptr);
    else
      k_slice_rows<4><<<blocks, 256, 0, cs>>>(data->data, indices, indptr, L, start, end, max_out,
                                              new_data, new_indices, new_indptr);
    return cuda_status(cudaGetLastError());
  }
  if (dim != 1) return VQ_ERR_INVALID;
  if (!workspace) return VQ_ERR_NULL;
  if (start < 0) return VQ_ERR_INVALID;
  if (max_out > 0) {
    if (cudaMemsetAsync(new_data, 0, (size_t)max_out * es, cs) != cudaSuccess ||
        cudaMemsetAsync(new_indices, 0xFF, (size_t)max_out * 4, cs) != cudaSuccess)
      return VQ_ERR_CUDA;
  }
  int32_t* counts = workspace;             // [rows]
  int32_t* excl = workspace + rows;        // [rows + 1]
  const unsigned wblocks = (unsigned)std::max<int64_t>((rows * 32 + 255) / 256, 1);
  if (rows > 0)
    k_slice_count<<<wblocks, 256, 0, cs>>>(indices, indptr, rows, L, start, end, counts);
  k_slice_scan<<<1, 1024, 0, cs>>>(counts, rows, max_out, excl, new_indptr);
  int st = cuda_status(cudaGetLastError());
  if (st || rows == 0) return st;
  if (es == 2)
    k_slice_write<2><<<wblocks, 256, 0, cs>>>(data->data, indices, indptr, rows, L, start, end, excl,
                                              max_out, new_data, new_indices);
  else
    k_slice_write<4><<<wblocks, 256, 0, cs>>>(data->data, indices, indptr, rows, L, start, end, excl,
                                              max_out, new_data, new_indices);
  return cuda_status(cudaGetLastError());
}

int vq_transpose(const vq_tensor* src, vq_tensor* dst, void* stream) {
  if (!src || !dst) return VQ_ERR_NULL;
  int64_t nb, R, C;
  int st = matrix_dims(src, &nb, &R, &C);
  if (st) return st;
  if (dst->dtype != src->dtype || dst->ndim != src->ndim) return VQ_ERR_SHAPE;
  for (int d = 0; d < src->ndim - 2; ++d)
    if (dst->shape[d] != src->shape[d]) return VQ_ERR_SHAPE;
  if (dst->shape[src->ndim - 2] != C || dst->shape[src->ndim - 1] != R) return VQ_ERR_SHAPE;
  if (nb * R * C == 0) return VQ_OK;
  if (!src->data || !dst->data) return VQ_ERR_NULL;
  const int64_t tr = (R + 31) / 32, tc = (C + 31) / 32;
  const int64_t blocks = nb * tr * tc;
  if (blocks > INT32_MAX) return VQ_ERR_TOO_LARGE;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  if (esize(src->dtype) == 2)
    k_transpose<uint16_t><<<(unsigned)blocks, 256, 0, cs>>>(
        (const uint16_t*)src->data, (uint16_t*)dst->data, R, C, tr, tc);
  else
    k_transpose<uint32_t><<<(unsigned)blocks, 256, 0, cs>>>(
        (const uint32_t*)src->data, (uint32_t*)dst->data, R, C, tr, tc);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
