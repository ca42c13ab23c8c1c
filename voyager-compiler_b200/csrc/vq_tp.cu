// Tensor-parallel decoder collectives over NVLink / NVSwitch, written by the
// kernels that produce the data (no separate collective launch).
//
// The decoder's column-parallel layout keeps the residual stream split by
// hidden columns; every rank needs the full rows of the MXFP8 operands its
// GEMMs read.  Each producer kernel therefore quantizes its own column shard
// and stores the tcgen05 operand (E4M3 bytes + UE8M0 scale words) through
// the NVLS multicast address of a symmetric buffer (multimem.st): one store
// lands in every rank's copy.  A rank waits for the others with
// k_tp_barrier: release / acquire flags in the same symmetric buffer, the
// wait bounded by %globaltimer (a wait that gives up sets *err and returns).
//
//   k_tp_sumsq    partial sum of squares of this rank's columns of each row
//                 -> slot [rank][row] of every rank's stats buffer
//   k_tp_norm_qmx RMSNorm of this rank's columns (row statistic = the sum of
//                 the ranks' partials in rank order) -> MXFP8 operand columns
//   k_tp_qmx      MXFP8 quantization of a bf16 [rows, C] shard -> operand
//                 columns (the attention output before o_proj)
//   k_tp_swiglu_qmx  bf16(silu(gate)) * up -> operand columns, zero padded
//                 from the shard's width to the next multiple of 128
//
// Quantization is quantize_mx's (E4M3 table, power-of-two block-32 scales
// along the row): the same pow2_scale_bf16 and hardware E4M3 rounding as
// k_qmx_last.  Each thread handles 16 consecutive columns; 8 threads cover a
// 128-column K tile and assemble its 4 scale bytes into one 32-bit word.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "vq_hw.cuh"
#include "vq_numerics.cuh"
#include "vq_tc.cuh"

namespace vq {
namespace tp {

constexpr uint64_t WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_rn(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// Stores through a multicast address: every rank's copy receives the data.
__device__ __forceinline__ void mc_st_v4(void* addr, uint32_t a, uint32_t b, uint32_t c,
                                         uint32_t d) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr),
               "f"(__uint_as_float(a)), "f"(__uint_as_float(b)), "f"(__uint_as_float(c)),
               "f"(__uint_as_float(d))
               : "memory");
}
__device__ __forceinline__ void mc_st_f32(void* addr, uint32_t a) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(addr), "f"(__uint_as_float(a))
               : "memory");
}

// ---------------------------------------------------------------------------
// Barrier: thread j tells rank j "rank `rank` reached epoch", then waits for
// rank j's flag in this rank's array.  Flags only grow (epoch is the
// caller's call counter), so no reset is needed.  A wait that has not seen
// its flag after timeout_ns of %globaltimer time records 100 + j and ends.
__global__ void k_tp_barrier(const uint64_t* peer_flags, uint32_t* my_flags, int rank, int world,
                             uint32_t epoch, uint64_t timeout_ns, int* err) {
  const int j = threadIdx.x;
  if (j < world) {
    __threadfence_system();
    uint32_t* dst = reinterpret_cast<uint32_t*>(peer_flags[j]) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
    const uint32_t* src = my_flags + j;
    const uint64_t t0 = now_ns();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(src) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (now_ns() - t0 > timeout_ns) {
        vq::tc::note_err(err, 100 + j);
        break;
      }
    }
    __threadfence_system();
  }
}

// The same barrier with the epoch kept on the device: *counter + 1 (0 is
// skipped), stored back for the next call.  Every rank makes the same
// sequence of barrier calls, so the counters stay equal across the ranks
// whether the launches come from the host one by one or from a replayed
// CUDA graph (where an epoch passed as a kernel argument would repeat).
__global__ void k_tp_barrier_dev(const uint64_t* peer_flags, uint32_t* my_flags, int rank,
                                 int world, uint32_t* counter, uint64_t timeout_ns, int* err) {
  __shared__ uint32_t ep;
  if (threadIdx.x == 0) {
    uint32_t e = *counter + 1u;
    if (e == 0u) e = 1u;
    *counter = e;
    ep = e;
  }
  __syncthreads();
  const uint32_t epoch = ep;
  const int j = threadIdx.x;
  if (j < world) {
    __threadfence_system();
    uint32_t* dst = reinterpret_cast<uint32_t*>(peer_flags[j]) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(epoch) : "memory");
    const uint32_t* src = my_flags + j;
    const uint64_t t0 = now_ns();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(src) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (now_ns() - t0 > timeout_ns) {
        vq::tc::note_err(err, 100 + j);
        break;
      }
    }
    __threadfence_system();
  }
}

// ---------------------------------------------------------------------------
struct SumsqArgs {
  const uint16_t* x;  // bf16 [T, C] (this rank's columns)
  float* stats_mc;    // multicast address of float [world][T]
  int T, C, rank;
};

// One warp per row.
__global__ void __launch_bounds__(256) k_tp_sumsq(const __grid_constant__ SumsqArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.T) return;
  const uint16_t* xr = a.x + row * a.C;
  float acc = 0.f;
  for (int c = lane * 8; c < a.C; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float f0 = lo_f(w[k]), f1 = hi_f(w[k]);
      acc = __fmaf_rn(f0, f0, acc);
      acc = __fmaf_rn(f1, f1, acc);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (lane == 0) mc_st_f32(a.stats_mc + (int64_t)a.rank * a.T + row, __float_as_uint(acc));
}

// ---------------------------------------------------------------------------
// Where a shard's operand columns go: E4M3 bytes at packed + row * ld +
// col_off, scale words at atoms + ((kt_off + kt) * RT + row / 128) * 512 +
// (row % 32) * 16 + (row / 32 % 4) * 4 (multicast addresses).
struct Dest {
  uint8_t* packed;
  uint8_t* atoms;
  int64_t ld;
  int col_off;
  int kt_off;
  int RT;
};

// 16 bf16 values of one lane (8 packed pairs) -> MXFP8: two blocks of 32
// span lane pairs, a K tile spans 8 lanes.  Stores the lane's 16 bytes and,
// from the tile's first lane, the tile's scale word.
__device__ __forceinline__ void quant16_store(const uint32_t (&v)[8], int64_t row, int c16,
                                              const Dest& d, int fl2q, uint32_t nan_bits) {
  const int lane = threadIdx.x & 31;
  uint32_t m = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) m = __vmaxu2(m, v[k] & 0x7FFF7FFFu);
  m = max(m & 0xFFFFu, m >> 16);
  const unsigned grp8 = 0xFFu << (lane & 24);
  m = max(m, __shfl_xor_sync(grp8, m, 1));
  const uint32_t sbits = pow2_scale_bf16(m, fl2q);
  const uint32_t E = (sbits >> 7) & 0xFFu;
  const bool fast = E >= 1u && E <= 253u;
  const float inv = __uint_as_float((254u - min(max(E, 1u), 253u)) << 23);
  const float s = bf2f(sbits);
  uint32_t bytes[4];
#pragma unroll
  for (int k = 0; k < 8; k += 2) {
    uint32_t c2[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float x0 = lo_f(v[k + h]), x1 = hi_f(v[k + h]);
      const float q0 = fast ? x0 * inv : __fdiv_rn(x0, s);
      const float q1 = fast ? x1 * inv : __fdiv_rn(x1, s);
      c2[h] = hw_pair<K_HW_E4M3>(pair_index<K_HW_E4M3>(q0, q1), nan_bits);
    }
    uint16_t b0, b1;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b0) : "f"(hi_f(c2[0])), "f"(lo_f(c2[0])));
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b1) : "f"(hi_f(c2[1])), "f"(lo_f(c2[1])));
    bytes[k / 2] = (uint32_t)b0 | ((uint32_t)b1 << 16);
  }
  mc_st_v4(d.packed + row * d.ld + d.col_off + c16 * 16, bytes[0], bytes[1], bytes[2], bytes[3]);
  // scale bytes of the tile's 4 blocks (lanes 0, 2, 4, 6 of the 8-lane group)
  const uint32_t e8 = E;
  const int base = lane & 24;
  const uint32_t w0 = __shfl_sync(grp8, e8, base + 0), w1 = __shfl_sync(grp8, e8, base + 2);
  const uint32_t w2 = __shfl_sync(grp8, e8, base + 4), w3 = __shfl_sync(grp8, e8, base + 6);
  if ((lane & 7) == 0) {
    const int kt = c16 / 8;
    const size_t off = ((size_t)(d.kt_off + kt) * d.RT + (row >> 7)) * 512 + (row & 31) * 16 +
                       ((row >> 5) & 3) * 4;
    mc_st_f32(d.atoms + off, w0 | (w1 << 8) | (w2 << 16) | (w3 << 24));
  }
}

// ---------------------------------------------------------------------------
struct NormArgs {
  const uint16_t* x;    // bf16 [T, C]
  const float* stats;   // float [world][T] (local copy)
  const uint16_t* w;    // bf16 [C]: this rank's slice of the norm weight
  Dest d;
  int T, C, world, H;   // H = full row length (the mean's divisor)
  float eps;
  int fl2q;
  uint32_t nan_bits;
};

__global__ void __launch_bounds__(256) k_tp_norm_qmx(const __grid_constant__ NormArgs a) {
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int per_row = a.C / 16;
  if (gid >= (int64_t)a.T * per_row) return;  // per_row % 8 == 0: tiles stay whole
  const int64_t row = gid / per_row;
  const int c16 = (int)(gid % per_row);
  float ss = 0.f;
  for (int r = 0; r < a.world; ++r) ss += a.stats[(int64_t)r * a.T + row];
  const float rs = rsqrtf(__fdiv_rn(ss, (float)a.H) + a.eps);
  const uint16_t* xr = a.x + row * a.C + c16 * 16;
  uint32_t v[8];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + 8 * h);
    const uint4 g = *reinterpret_cast<const uint4*>(a.w + c16 * 16 + 8 * h);
    const uint32_t xw[4] = {u.x, u.y, u.z, u.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t y = pack_rn(lo_f(xw[k]) * rs, hi_f(xw[k]) * rs);
      v[4 * h + k] = pack_rn(lo_f(gw[k]) * lo_f(y), hi_f(gw[k]) * hi_f(y));
    }
  }
  quant16_store(v, row, c16, a.d, a.fl2q, a.nan_bits);
}

// ---------------------------------------------------------------------------
struct QmxArgs {
  const uint16_t* x;  // bf16 [T, ldx] (C used)
  int64_t ldx;
  Dest d;
  int T, C;
  int fl2q;
  uint32_t nan_bits;
};

__global__ void __launch_bounds__(256) k_tp_qmx(const __grid_constant__ QmxArgs a) {
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int per_row = a.C / 16;
  if (gid >= (int64_t)a.T * per_row) return;
  const int64_t row = gid / per_row;
  const int c16 = (int)(gid % per_row);
  const uint16_t* xr = a.x + row * a.ldx + c16 * 16;
  const uint4 u0 = *reinterpret_cast<const uint4*>(xr);
  const uint4 u1 = *reinterpret_cast<const uint4*>(xr + 8);
  const uint32_t v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  quant16_store(v, row, c16, a.d, a.fl2q, a.nan_bits);
}

// ---------------------------------------------------------------------------
struct SwigluArgs {
  const uint16_t* gu;  // bf16 [T, ld]: gate [0, F), up [up_off, up_off + F)
  int64_t ld, up_off;
  Dest d;
  int T, F, Fp;        // Fp = F rounded up to 128 (the shard's operand width)
  int fl2q;
  uint32_t nan_bits;
};

__global__ void __launch_bounds__(256) k_tp_swiglu_qmx(const __grid_constant__ SwigluArgs a) {
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int per_row = a.Fp / 16;
  if (gid >= (int64_t)a.T * per_row) return;
  const int64_t row = gid / per_row;
  const int c16 = (int)(gid % per_row);
  uint32_t v[8];
  const int c0 = c16 * 16;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = c0 + 8 * h;  // F % 8 == 0: a group of 8 is all real or all padding
    if (c < a.F) {
      const uint4 g4 = *reinterpret_cast<const uint4*>(a.gu + row * a.ld + c);
      const uint4 u4 = *reinterpret_cast<const uint4*>(a.gu + row * a.ld + a.up_off + c);
      const uint32_t g[4] = {g4.x, g4.y, g4.z, g4.w}, u[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float g0 = lo_f(g[k]), g1 = hi_f(g[k]);
        const uint32_t s = pack_rn(g0 / (1.0f + expf(-g0)), g1 / (1.0f + expf(-g1)));
        v[4 * h + k] = pack_rn(lo_f(s) * lo_f(u[k]), hi_f(s) * hi_f(u[k]));
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) v[4 * h + k] = 0u;  // padding: code 0, scale 1
    }
  }
  quant16_store(v, row, c16, a.d, a.fl2q, a.nan_bits);
}

// ---------------------------------------------------------------------------
// A [rows, bytes] block copied into every rank's copy of a symmetric buffer:
// consecutive threads take consecutive 16-byte pieces of a row, so each warp
// store is 512 contiguous bytes through the multicast address.
__global__ void __launch_bounds__(256) k_tp_copy_mc(const uint8_t* src, int64_t lds, uint8_t* dst,
                                                    int64_t ldd, int64_t rows, int64_t bytes) {
  const int64_t per_row = bytes / 16;
  const int64_t total = rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * 256) {
    const int64_t r = i / per_row, c = (i % per_row) * 16;
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src + r * lds + c));
    mc_st_v4(dst + r * ldd + c, v.x, v.y, v.z, v.w);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_dest(const Dest& d, int C) {
  if (!d.packed || !d.atoms) return VQ_ERR_NULL;
  if (!al16(d.packed) || (reinterpret_cast<uintptr_t>(d.atoms) & 3)) return VQ_ERR_ALIGNMENT;
  if (C % 128 || d.col_off % 128 || d.ld % 16 || d.col_off + C > d.ld) return VQ_ERR_UNSUPPORTED;
  if (d.kt_off != d.col_off / 128 || d.RT <= 0) return VQ_ERR_INVALID;
  return VQ_OK;
}

// This file's sticky wait-timeout word (vq_device_errors).
int sticky_tp(int* out, int clear, cudaStream_t st) { return vq::tc::sticky_read(out, clear, st); }

int e4m3(const vq_rounder* r) {
  if (!r) return VQ_ERR_NULL;
  return (r->kind == VQ_R_MINIFLOAT && r->hw == VQ_HW_E4M3) ? VQ_OK : VQ_ERR_UNSUPPORTED;
}

}  // namespace tp
}  // namespace vq

using namespace vq::tp;

extern "C" {

int vq_tp_barrier_ex(const void* peer_flag_ptrs, void* my_flags, int32_t rank, int32_t world,
                     uint32_t epoch, uint64_t timeout_ns, int32_t* d_err, void* stream) {
  if (!peer_flag_ptrs || !my_flags || !d_err) return VQ_ERR_NULL;
  if (world < 1 || world > 64 || rank < 0 || rank >= world) return VQ_ERR_INVALID;
  if (timeout_ns < 1000 || timeout_ns > 10000000000ull) return VQ_ERR_INVALID;
  k_tp_barrier<<<1, 64, 0, (cudaStream_t)stream>>>((const uint64_t*)peer_flag_ptrs,
                                                   (uint32_t*)my_flags, rank, world, epoch,
                                                   timeout_ns, d_err);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_tp_barrier(const void* peer_flag_ptrs, void* my_flags, int32_t rank, int32_t world,
                  uint32_t epoch, int32_t* d_err, void* stream) {
  return vq_tp_barrier_ex(peer_flag_ptrs, my_flags, rank, world, epoch, WAIT_NS, d_err, stream);
}

int vq_tp_barrier_dev(const void* peer_flag_ptrs, void* my_flags, int32_t rank, int32_t world,
                      uint32_t* d_counter, uint64_t timeout_ns, int32_t* d_err, void* stream) {
  if (!peer_flag_ptrs || !my_flags || !d_counter || !d_err) return VQ_ERR_NULL;
  if (world < 1 || world > 64 || rank < 0 || rank >= world) return VQ_ERR_INVALID;
  if (timeout_ns < 1000 || timeout_ns > 10000000000ull) return VQ_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(d_counter) & 3) return VQ_ERR_ALIGNMENT;
  k_tp_barrier_dev<<<1, 64, 0, (cudaStream_t)stream>>>((const uint64_t*)peer_flag_ptrs,
                                                       (uint32_t*)my_flags, rank, world, d_counter,
                                                       timeout_ns, d_err);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_tp_copy_multicast(const void* src, int64_t src_ld, int64_t rows, int64_t row_bytes,
                         void* dst_mc, int64_t dst_ld, void* stream) {
  if (!src || !dst_mc) return VQ_ERR_NULL;
  if (rows <= 0 || row_bytes <= 0 || row_bytes % 16 || src_ld % 16 || dst_ld % 16 ||
      src_ld < row_bytes || dst_ld < row_bytes)
    return VQ_ERR_INVALID;
  if (!al16(src) || !al16(dst_mc)) return VQ_ERR_ALIGNMENT;
  const int64_t total = rows * (row_bytes / 16);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  k_tp_copy_mc<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)src, src_ld, (uint8_t*)dst_mc, dst_ld, rows, row_bytes);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_tp_sumsq(const void* x, int64_t rows, int64_t cols, void* stats_mc, int32_t rank,
                void* stream) {
  if (!x || !stats_mc) return VQ_ERR_NULL;
  if (rows <= 0 || cols <= 0 || cols % 8 || rows >= (1ll << 31)) return VQ_ERR_INVALID;
  if (!al16(x) || (reinterpret_cast<uintptr_t>(stats_mc) & 3)) return VQ_ERR_ALIGNMENT;
  SumsqArgs a{(const uint16_t*)x, (float*)stats_mc, (int)rows, (int)cols, rank};
  k_tp_sumsq<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_tp_norm_quantize(const void* x, int64_t rows, int64_t cols, const void* stats,
                        int32_t world, int64_t full_cols, const void* weight, float eps,
                        const vq_rounder* qmap, int32_t floor_log2_qmax, void* packed_mc,
                        void* atoms_mc, int64_t ld, int64_t col_off, int64_t row_tiles,
                        void* stream) {
  int st = e4m3(qmap);
  if (st) return st;
  if (!x || !stats || !weight) return VQ_ERR_NULL;
  if (rows <= 0 || rows >= (1ll << 31) || world < 1 || full_cols <= 0) return VQ_ERR_INVALID;
  Dest d{(uint8_t*)packed_mc, (uint8_t*)atoms_mc, ld, (int)col_off, (int)(col_off / 128),
         (int)row_tiles};
  if ((st = check_dest(d, (int)cols))) return st;
  if (row_tiles * 128 < rows || !al16(x) || !al16(weight)) return VQ_ERR_INVALID;
  NormArgs a{(const uint16_t*)x, (const float*)stats, (const uint16_t*)weight, d, (int)rows,
             (int)cols, world, (int)full_cols, eps, floor_log2_qmax, qmap->nan_bits};
  const int64_t total = rows * (cols / 16);
  k_tp_norm_qmx<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_tp_quantize(const void* x, int64_t ldx, int64_t rows, int64_t cols, const vq_rounder* qmap,
                   int32_t floor_log2_qmax, void* packed_mc, void* atoms_mc, int64_t ld,
                   int64_t col_off, int64_t row_tiles, void* stream) {
  int st = e4m3(qmap);
  if (st) return st;
  if (!x) return VQ_ERR_NULL;
  if (rows <= 0 || rows >= (1ll << 31) || ldx < cols || ldx % 8) return VQ_ERR_INVALID;
  Dest d{(uint8_t*)packed_mc, (uint8_t*)atoms_mc, ld, (int)col_off, (int)(col_off / 128),
         (int)row_tiles};
  if ((st = check_dest(d, (int)cols))) return st;
  if (row_tiles * 128 < rows || !al16(x)) return VQ_ERR_INVALID;
  QmxArgs a{(const uint16_t*)x, ldx, d, (int)rows, (int)cols, floor_log2_qmax, qmap->nan_bits};
  const int64_t total = rows * (cols / 16);
  k_tp_qmx<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_tp_swiglu_quantize(const void* gate_up, int64_t ld_in, int64_t up_off, int64_t rows,
                          int64_t cols, const vq_rounder* qmap, int32_t floor_log2_qmax,
                          void* packed_mc, void* atoms_mc, int64_t ld, int64_t col_off,
                          int64_t row_tiles, void* stream) {
  int st = e4m3(qmap);
  if (st) return st;
  if (!gate_up) return VQ_ERR_NULL;
  if (rows <= 0 || rows >= (1ll << 31) || cols <= 0 || cols % 32 || ld_in % 8 || up_off % 8 ||
      up_off < cols || up_off + cols > ld_in)
    return VQ_ERR_INVALID;
  const int64_t Fp = (cols + 127) / 128 * 128;
  Dest d{(uint8_t*)packed_mc, (uint8_t*)atoms_mc, ld, (int)col_off, (int)(col_off / 128),
         (int)row_tiles};
  if ((st = check_dest(d, (int)Fp))) return st;
  if (row_tiles * 128 < rows || !al16(gate_up)) return VQ_ERR_INVALID;
  SwigluArgs a{(const uint16_t*)gate_up, ld_in, up_off, d, (int)rows, (int)cols, (int)Fp,
               floor_log2_qmax, qmap->nan_bits};
  const int64_t total = rows * (Fp / 16);
  k_tp_swiglu_qmx<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
