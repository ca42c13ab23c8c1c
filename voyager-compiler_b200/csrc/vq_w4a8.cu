// W4A8 linear for few tokens: NVFP4 weights (E2M1 codes, E4M3 scales per 16
// along K) times MXFP8 activations (E4M3 codes, power-of-two scales per 32).
//
// The reference has no single op for this pair (linear_mx takes one block
// size); its result is aten.linear of the two operands dequantized with their
// own block sizes (src/voyager_compiler/ops/quantized.py:455-472, 522-586).
// With M <= 16 tokens the product streams the weights once and is bound by
// HBM (arithmetic intensity ~4-56 FLOP/B), so this kernel reads the packed
// weights (0.5 B + 1/16 B per weight) instead of a dequantized bf16 copy.
//
// Per warp: 32 weight rows x 16 tokens, mma.sync.m16n8k16 with f16 operands:
//   weights  16-byte loads; each nibble pair -> f16x2 (cvt.rn.f16x2.e2m1x2)
//            times its E4M3 block scale (exact in f16: at most 6 significant
//            bits in [2^-10, 2688]);
//   tokens   the E4M3 codes themselves (exact in f16), staged once per CTA in
//            shared memory; their power-of-two block scale multiplies the
//            float32 sum of the two MMA steps of each 32-wide block.
// The packed weight rows are permuted within each 128-wide K chunk
// (vq_w4_pack_weights) so that thread t of a quad finds in its 16 contiguous
// bytes exactly its fragment values: for each 32-block b, k = 32b + 16h +
// {2t, 2t+1, 2t+8, 2t+9} for the two MMA steps h, so every MMA covers one
// weight scale block of 16 and one token scale block of 32.  The K range is
// split over CTAs; partial sums meet in a float32 workspace, and the last CTA
// of each row block adds the bias, rounds to bf16 and leaves the workspace
// zero (one launch per call).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "vq_numerics.cuh"

namespace vq {
namespace w4 {

constexpr int WARPS = 8;
constexpr int WROWS = 32;             // weight rows per warp
constexpr int ROWS = WARPS * WROWS;   // 256 weight rows per CTA

struct Args {
  const uint8_t* wq;   // [N, K/2] E2M1 nibbles, even k in the low nibble
  const uint8_t* ws;   // [N, K/16] E4M3 scale bytes
  const uint16_t* ac;  // bf16 [M, K] token codes
  const uint16_t* as;  // bf16 [M, K/32] token block scales
  const uint16_t* bias;  // bf16 [N] or null
  uint16_t* out;       // bf16 [M, N]
  float* acc;          // [M, N] float32 workspace: zero on entry, left zero
  int* done;           // [row blocks] split counters: zero on entry, left zero
  int M, N, K, chunks_per_split, splits;
};

__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(r) : "r"(byte));
  return r;
}
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(r) : "r"(two_bytes));
  return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

constexpr int MAX_CHUNKS = 8;  // K chunks of 128 per CTA (the split size)

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

__global__ void __launch_bounds__(WARPS * 32, 2) k_w4a8(const __grid_constant__ Args p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * ROWS + warp * WROWS + g;  // rows row0 + 8i, i = 0..3
  const int nch = p.K / 128;
  const int c0 = blockIdx.y * p.chunks_per_split, c1 = min(c0 + p.chunks_per_split, nch);
  const bool two = p.M > 8;
  const size_t wrow = (size_t)p.K / 2, srow = (size_t)p.K / 16;
  bool ok[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) ok[i] = row0 + 8 * i < p.N;
  float acc[2][2][4] = {};
  // weights of the next chunk are loaded while this one is used
  uint4 w[4];
  uint2 sc[4];
  auto load = [&](int c) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const size_t r = (size_t)(row0 + 8 * i);
      w[i] = ok[i] ? ld_stream(p.wq + r * wrow + c * 64 + t * 16) : make_uint4(0, 0, 0, 0);
      sc[i] = ok[i] ? *reinterpret_cast<const uint2*>(p.ws + r * srow + c * 8) : make_uint2(0, 0);
    }
  };
  if (c0 < c1) load(c0);  // in flight while the tokens are staged
  // this CTA's K range of the 16 tokens: E4M3 codes as f16 [16][kw] and the
  // block scales as float [16][kw / 32] (zero past M)
  // rows padded by 8 halves so the 8 token rows a warp reads fall in
  // different banks
  __shared__ __align__(16) uint16_t tok[16 * (MAX_CHUNKS * 128 + 8)];
  __shared__ float tsc[16 * MAX_CHUNKS * 4];
  const int kw = (c1 - c0) * 128;
  const int ks = kw + 8;  // staged row stride (halves)
  for (int i = threadIdx.x; i < 16 * kw / 8; i += blockDim.x) {
    const int m = i / (kw / 8), k = c0 * 128 + (i % (kw / 8)) * 8;
    uint4 o = make_uint4(0, 0, 0, 0);
    if (m < p.M) {
      const uint4 v = *reinterpret_cast<const uint4*>(p.ac + (size_t)m * p.K + k);
      const uint32_t cv[4] = {v.x, v.y, v.z, v.w};
      uint32_t r[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        __half2 h = __floats2half2_rn(__uint_as_float(cv[q] << 16),
                                      __uint_as_float(cv[q] & 0xFFFF0000u));
        r[q] = *reinterpret_cast<uint32_t*>(&h);
      }
      o = make_uint4(r[0], r[1], r[2], r[3]);
    }
    *reinterpret_cast<uint4*>(tok + m * ks + (k - c0 * 128)) = o;
  }
  for (int i = threadIdx.x; i < 16 * kw / 32; i += blockDim.x) {
    const int m = i / (kw / 32), kb = c0 * 4 + i % (kw / 32);
    tsc[i] = m < p.M ? __uint_as_float((uint32_t)p.as[(size_t)m * (p.K / 32) + kb] << 16) : 0.f;
  }
  __syncthreads();
  for (int c = c0; c < c1; ++c) {
    const uint4 wc[4] = {w[0], w[1], w[2], w[3]};
    const uint2 scc[4] = {sc[0], sc[1], sc[2], sc[3]};
    if (c + 1 < c1) load(c + 1);
    const int kc = (c - c0) * 128;  // chunk offset in the staged tokens
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      // token fragments of block b (f16 pairs): tokens g and g + 8
      uint32_t bt[2][2][2];  // [nt][h][pair lo / hi]
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint16_t* tp = tok + (8 * nt + g) * ks + kc + 32 * b + 16 * h + 2 * t;
          bt[nt][h][0] = *reinterpret_cast<const uint32_t*>(tp);
          bt[nt][h][1] = *reinterpret_cast<const uint32_t*>(tp + 8);
        }
      float d[2][2][4] = {};  // [mt][nt]: this block's sums
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint32_t wa = (&wc[2 * mt].x)[b], wb = (&wc[2 * mt + 1].x)[b];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = 2 * b + h;  // 16-block of the chunk
          const uint32_t sa = j < 4 ? byte_of(scc[2 * mt].x, j) : byte_of(scc[2 * mt].y, j - 4);
          const uint32_t sb = j < 4 ? byte_of(scc[2 * mt + 1].x, j) : byte_of(scc[2 * mt + 1].y, j - 4);
          const uint32_t sa2 = e4m3x2_to_f16x2(sa * 0x101u), sb2 = e4m3x2_to_f16x2(sb * 0x101u);
          const uint32_t a0 = hmul2(e2m1x2_to_f16x2(byte_of(wa, 2 * h)), sa2);
          const uint32_t a2 = hmul2(e2m1x2_to_f16x2(byte_of(wa, 2 * h + 1)), sa2);
          const uint32_t a1 = hmul2(e2m1x2_to_f16x2(byte_of(wb, 2 * h)), sb2);
          const uint32_t a3 = hmul2(e2m1x2_to_f16x2(byte_of(wb, 2 * h + 1)), sb2);
          mma_f16(d[mt][0], a0, a1, a2, a3, bt[0][h][0], bt[0][h][1]);
          if (two) mma_f16(d[mt][1], a0, a1, a2, a3, bt[1][h][0], bt[1][h][1]);
        }
      }
      // token block scales: C columns are tokens 8 nt + 2t, + 1
      const int kb = (kc + 32 * b) / 32;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        if (nt == 1 && !two) break;
        const float s0 = tsc[(8 * nt + 2 * t) * (kw / 32) + kb];
        const float s1 = tsc[(8 * nt + 2 * t + 1) * (kw / 32) + kb];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          acc[mt][nt][0] = fmaf(d[mt][nt][0], s0, acc[mt][nt][0]);
          acc[mt][nt][1] = fmaf(d[mt][nt][1], s1, acc[mt][nt][1]);
          acc[mt][nt][2] = fmaf(d[mt][nt][2], s0, acc[mt][nt][2]);
          acc[mt][nt][3] = fmaf(d[mt][nt][3], s1, acc[mt][nt][3]);
        }
      }
    }
  }
  // C fragment: rows (weight) g / g + 8 of the m-tile, tokens 8 nt + 2t, + 1
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const int rA = row0 + 16 * mt, rB = rA + 8;
    const bool okA = ok[2 * mt], okB = ok[2 * mt + 1];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int ta = 8 * nt + 2 * t, tb = ta + 1;
      if (okA && ta < p.M) atomicAdd(p.acc + (size_t)ta * p.N + rA, acc[mt][nt][0]);
      if (okA && tb < p.M) atomicAdd(p.acc + (size_t)tb * p.N + rA, acc[mt][nt][1]);
      if (okB && ta < p.M) atomicAdd(p.acc + (size_t)ta * p.N + rB, acc[mt][nt][2]);
      if (okB && tb < p.M) atomicAdd(p.acc + (size_t)tb * p.N + rB, acc[mt][nt][3]);
    }
  }
  // the last split of this row block to finish writes the rows out (+ bias,
  // bf16) and leaves the workspace and its counter at zero for the next call
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.done + blockIdx.x, 1);
    last = prev == p.splits - 1;
    if (last) p.done[blockIdx.x] = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int r0 = blockIdx.x * ROWS;
  const int nrows = min(ROWS, p.N - r0);
  for (int i = threadIdx.x; i < p.M * nrows; i += blockDim.x) {
    const int m = i / nrows, r = r0 + i % nrows;
    float v = atomicExch(p.acc + (size_t)m * p.N + r, 0.f);
    if (p.bias) v += bf2f(p.bias[r]);
    p.out[(size_t)m * p.N + r] = (uint16_t)f2bf(v);
  }
}

// Packing --------------------------------------------------------------------
// weights: bf16 E2M1 codes [N, K] -> nibbles [N, K/2] (even k in the low
// nibble; bytes permuted within each 64-byte chunk as k_w4a8 reads them);
// bf16 E4M3 scales [N, K/16] -> bytes.  Counts codes / scales that are not
// such values.
__global__ void k_w4_pack(const uint16_t* codes, const uint16_t* scales, uint8_t* wq, uint8_t* ws,
                          int N, int K, int* inexact) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one byte of wq
  const int64_t total = (int64_t)N * (K / 2);
  if (i < total) {
    const float f0 = bf2f(codes[2 * i]), f1 = bf2f(codes[2 * i + 1]);
    uint32_t q;
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
        : "=r"(q) : "f"(f1), "f"(f0));
    // byte o = 16b + 4ii + t of a row's 64-byte chunk goes to 16t + 4b + ii
    const int64_t row = i / (K / 2), o = i % (K / 2);
    const int c = (int)(o / 64), oo = (int)(o % 64);
    const int b = oo / 16, ii = (oo % 16) / 4, t = oo % 4;
    wq[row * (K / 2) + c * 64 + t * 16 + 4 * b + ii] = (uint8_t)q;
    const uint32_t back = e2m1x2_to_f16x2(q);
    const float g0 = __half2float(__ushort_as_half((unsigned short)(back & 0xFFFF)));
    const float g1 = __half2float(__ushort_as_half((unsigned short)(back >> 16)));
    const int bad = (g0 != f0) + (g1 != f1);  // -0 == +0 counts as equal
    if (bad && inexact) atomicAdd(inexact, bad);
  }
  const int64_t ns = (int64_t)N * (K / 16);
  if (i < ns) {
    const float f = bf2f(scales[i]);
    uint16_t b;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b) : "f"(0.f), "f"(f));
    ws[i] = (uint8_t)(b & 0xFF);
    const uint32_t back = e4m3x2_to_f16x2(b & 0xFF);
    const float g = __half2float(__ushort_as_half((unsigned short)(back & 0xFFFF)));
    if (g != f && inexact) atomicAdd(inexact, 1);
  }
}

int sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

}  // namespace w4
}  // namespace vq

using namespace vq::w4;

extern "C" {

int vq_w4_pack_weights(const vq_tensor* codes, const vq_tensor* scales, void* wq, void* ws,
                       int32_t* d_inexact, void* stream) {
  if (!codes || !scales || !wq || !ws) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || scales->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (codes->ndim != 2 || scales->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t N = codes->shape[0], K = codes->shape[1];
  if (K % 128 || N <= 0 || scales->shape[0] != N || scales->shape[1] != K / 16) return VQ_ERR_SHAPE;
  if (N * K >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_inexact && cudaMemsetAsync(d_inexact, 0, 4, st) != cudaSuccess) return VQ_ERR_CUDA;
  const int64_t n = N * (K / 2);
  k_w4_pack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      (const uint16_t*)codes->data, (const uint16_t*)scales->data, (uint8_t*)wq, (uint8_t*)ws,
      (int)N, (int)K, d_inexact);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_w4a8_linear_small(const vq_tensor* a_codes, const vq_tensor* a_scales, const void* wq,
                         const void* ws, int64_t N, const void* bias, float* workspace,
                         int32_t* counters, void* out, void* stream) {
  if (!a_codes || !a_scales || !wq || !ws || !workspace || !counters || !out) return VQ_ERR_NULL;
  if (a_codes->dtype != VQ_BF16 || a_scales->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (a_codes->ndim != 2 || a_scales->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t M = a_codes->shape[0], K = a_codes->shape[1];
  if (a_scales->shape[0] != M || a_scales->shape[1] != K / 32) return VQ_ERR_SHAPE;
  if (M <= 0 || M > 16 || N <= 0 || K <= 0 || K % 128) return VQ_ERR_UNSUPPORTED;
  if (N * K >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  const void* ptrs[3] = {a_codes->data, wq, ws};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15) return VQ_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Args p;
  p.wq = (const uint8_t*)wq;
  p.ws = (const uint8_t*)ws;
  p.ac = (const uint16_t*)a_codes->data;
  p.as = (const uint16_t*)a_scales->data;
  p.bias = (const uint16_t*)bias;
  p.out = (uint16_t*)out;
  p.acc = workspace;
  p.done = counters;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  const int rb = (int)((N + ROWS - 1) / ROWS), chunks = (int)(K / 128);
  // one wave of two CTAs per SM when the rows allow, at most MAX_CHUNKS
  // chunks (the shared-memory token slice) per CTA
  int splits = std::max(1, (2 * sms()) / rb);
  splits = std::min(splits, std::max(1, chunks / 2));
  p.chunks_per_split = std::min((chunks + splits - 1) / splits, MAX_CHUNKS);
  p.splits = (chunks + p.chunks_per_split - 1) / p.chunks_per_split;
  if (p.splits > 65535) return VQ_ERR_UNSUPPORTED;
  k_w4a8<<<dim3(rb, p.splits), WARPS * 32, 0, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
