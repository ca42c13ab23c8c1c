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
// Per warp: 16 weight rows x 16 tokens, mma.sync.m16n8k16 with f16 operands:
//   weights  E2M1 nibble pairs -> f16x2 (cvt.rn.f16x2.e2m1x2), times the E4M3
//            block scale as f16x2 (exact: every E2M1 x E4M3 product is an f16);
//   tokens   E4M3 bytes -> f16x2 (exact), their power-of-two block scale
//            applied in float32 to the partial sum of each 32-wide K block.
// Within a 64-wide K group, thread t's fragment elements are the 8 K values
// 32b + 8t .. 32b + 8t + 7 of block b: a permutation of K that both operands
// share, so every MMA stays inside one activation-scale block.  The K range is
// split over CTAs; partial sums meet in a float32 workspace (red.add), then
// a finalize pass adds the bias and rounds to bf16.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "vq_numerics.cuh"

namespace vq {
namespace w4 {

constexpr int WARPS = 8;              // 128 weight rows per CTA
constexpr int ROWS = WARPS * 16;

struct Args {
  const uint8_t* wq;  // [N, K/2] E2M1 nibbles, even k in the low nibble
  const uint8_t* ws;  // [N, K/16] E4M3 scale bytes
  const uint8_t* aq;  // [M, K] E4M3 bytes
  const float* as;    // [M, K/32] activation scales
  float* acc;         // [M, N] float32 workspace, zeroed
  int M, N, K, groups_per_split;
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
__device__ __forceinline__ void mma_f16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(WARPS * 32) k_w4a8(const __grid_constant__ Args p) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane >> 2, t = lane & 3;
  const int rA = blockIdx.x * ROWS + warp * 16 + g, rB = rA + 8;
  const bool okA = rA < p.N, okB = rB < p.N;
  const int ngroups = p.K / 64;
  const int grp0 = blockIdx.y * p.groups_per_split;
  const int grp1 = min(grp0 + p.groups_per_split, ngroups);
  const int tok0 = g, tok1 = 8 + g;  // the B-fragment token of each 8-token tile
  const bool okT0 = tok0 < p.M, okT1 = tok1 < p.M;
  float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  const size_t wrow = (size_t)p.K / 2, srow = (size_t)p.K / 16;
  for (int grp = grp0; grp < grp1; ++grp) {
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const int kb = grp * 64 + 32 * b + 8 * t;  // this thread's 8 K values
      const uint32_t wa = okA ? *reinterpret_cast<const uint32_t*>(p.wq + rA * wrow + kb / 2) : 0u;
      const uint32_t wb = okB ? *reinterpret_cast<const uint32_t*>(p.wq + rB * wrow + kb / 2) : 0u;
      const uint32_t sa = okA ? p.ws[rA * srow + kb / 16] : 0u;
      const uint32_t sb = okB ? p.ws[rB * srow + kb / 16] : 0u;
      const uint32_t sa2 = e4m3x2_to_f16x2(sa | (sa << 8)), sb2 = e4m3x2_to_f16x2(sb | (sb << 8));
      uint32_t fa[4], fb[4];  // f16x2 of k pairs (0,1) (2,3) (4,5) (6,7)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        fa[i] = hmul2(e2m1x2_to_f16x2((wa >> (8 * i)) & 0xFF), sa2);
        fb[i] = hmul2(e2m1x2_to_f16x2((wb >> (8 * i)) & 0xFF), sb2);
      }
      const uint2 x0 = okT0 ? *reinterpret_cast<const uint2*>(p.aq + (size_t)tok0 * p.K + kb)
                            : make_uint2(0, 0);
      const uint2 x1 = okT1 ? *reinterpret_cast<const uint2*>(p.aq + (size_t)tok1 * p.K + kb)
                            : make_uint2(0, 0);
      const uint32_t b00 = e4m3x2_to_f16x2(x0.x & 0xFFFF), b01 = e4m3x2_to_f16x2(x0.x >> 16);
      const uint32_t b02 = e4m3x2_to_f16x2(x0.y & 0xFFFF), b03 = e4m3x2_to_f16x2(x0.y >> 16);
      const uint32_t b10 = e4m3x2_to_f16x2(x1.x & 0xFFFF), b11 = e4m3x2_to_f16x2(x1.x >> 16);
      const uint32_t b12 = e4m3x2_to_f16x2(x1.y & 0xFFFF), b13 = e4m3x2_to_f16x2(x1.y >> 16);
      // step 0: k 0..3 of the thread's 8; step 1: k 4..7
      const uint32_t a_s0[4] = {fa[0], fb[0], fa[1], fb[1]};
      const uint32_t a_s1[4] = {fa[2], fb[2], fa[3], fb[3]};
      float d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};
      mma_f16(d0, a_s0, b00, b01);
      mma_f16(d0, a_s1, b02, b03);
      if (p.M > 8) {
        mma_f16(d1, a_s0, b10, b11);
        mma_f16(d1, a_s1, b12, b13);
      }
      // the activation block scale of this 32-wide block, per token
      const int kblk = (grp * 64 + 32 * b) / 32, nkb = p.K / 32;
      const int c0 = 2 * t, c1 = 2 * t + 1;
      const float s00 = c0 < p.M ? p.as[c0 * nkb + kblk] : 0.f;
      const float s01 = c1 < p.M ? p.as[c1 * nkb + kblk] : 0.f;
      acc[0][0] += d0[0] * s00;
      acc[0][1] += d0[1] * s01;
      acc[0][2] += d0[2] * s00;
      acc[0][3] += d0[3] * s01;
      if (p.M > 8) {
        const float s10 = 8 + c0 < p.M ? p.as[(8 + c0) * nkb + kblk] : 0.f;
        const float s11 = 8 + c1 < p.M ? p.as[(8 + c1) * nkb + kblk] : 0.f;
        acc[1][0] += d1[0] * s10;
        acc[1][1] += d1[1] * s11;
        acc[1][2] += d1[2] * s10;
        acc[1][3] += d1[3] * s11;
      }
    }
  }
  // C fragment: rows rA (c0, c1) and rB (c2, c3), tokens 8j + 2t, 8j + 2t + 1
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int ta = 8 * j + 2 * t, tb = ta + 1;
    if (okA && ta < p.M) atomicAdd(p.acc + (size_t)ta * p.N + rA, acc[j][0]);
    if (okA && tb < p.M) atomicAdd(p.acc + (size_t)tb * p.N + rA, acc[j][1]);
    if (okB && ta < p.M) atomicAdd(p.acc + (size_t)ta * p.N + rB, acc[j][2]);
    if (okB && tb < p.M) atomicAdd(p.acc + (size_t)tb * p.N + rB, acc[j][3]);
  }
}

// float32 workspace (+ bias) -> bf16 out [M, N]
__global__ void k_w4a8_finalize(const float* acc, const uint16_t* bias, uint16_t* out, int M, int N) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * N) return;
  float v = acc[i];
  if (bias) v += bf2f(bias[i % N]);
  out[i] = (uint16_t)f2bf(v);
}

// Packing --------------------------------------------------------------------
// weights: bf16 E2M1 codes [N, K] -> nibbles [N, K/2]; bf16 E4M3 scales
// [N, K/16] -> bytes.  Counts codes / scales that are not such values.
__global__ void k_w4_pack(const uint16_t* codes, const uint16_t* scales, uint8_t* wq, uint8_t* ws,
                          int N, int K, int* inexact) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one byte of wq
  const int64_t total = (int64_t)N * (K / 2);
  if (i < total) {
    const float f0 = bf2f(codes[2 * i]), f1 = bf2f(codes[2 * i + 1]);
    uint32_t q;
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
        : "=r"(q) : "f"(f1), "f"(f0));
    wq[i] = (uint8_t)q;
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

// activations: bf16 E4M3 codes [M, K] -> bytes; bf16 scales -> float
__global__ void k_a8_pack(const uint16_t* codes, const uint16_t* scales, uint8_t* aq, float* as,
                          int M, int K, int* inexact) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one pair
  const int64_t total = (int64_t)M * K / 2;
  if (i < total) {
    const float f0 = bf2f(codes[2 * i]), f1 = bf2f(codes[2 * i + 1]);
    uint16_t b;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b) : "f"(f1), "f"(f0));
    *reinterpret_cast<uint16_t*>(aq + 2 * i) = b;
    const uint32_t back = e4m3x2_to_f16x2(b);
    const float g0 = __half2float(__ushort_as_half((unsigned short)(back & 0xFFFF)));
    const float g1 = __half2float(__ushort_as_half((unsigned short)(back >> 16)));
    const int bad = (g0 != f0) + (g1 != f1);
    if (bad && inexact) atomicAdd(inexact, bad);
  }
  if (i < (int64_t)M * (K / 32)) as[i] = bf2f(scales[i]);
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
  if (K % 64 || N <= 0 || scales->shape[0] != N || scales->shape[1] != K / 16) return VQ_ERR_SHAPE;
  if (N * K >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_inexact && cudaMemsetAsync(d_inexact, 0, 4, st) != cudaSuccess) return VQ_ERR_CUDA;
  const int64_t n = N * (K / 2);
  k_w4_pack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      (const uint16_t*)codes->data, (const uint16_t*)scales->data, (uint8_t*)wq, (uint8_t*)ws,
      (int)N, (int)K, d_inexact);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_a8_pack(const vq_tensor* codes, const vq_tensor* scales, void* aq, float* as,
               int32_t* d_inexact, void* stream) {
  if (!codes || !scales || !aq || !as) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || scales->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (codes->ndim != 2 || scales->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t M = codes->shape[0], K = codes->shape[1];
  if (K % 64 || M <= 0 || scales->shape[0] != M || scales->shape[1] != K / 32) return VQ_ERR_SHAPE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (d_inexact && cudaMemsetAsync(d_inexact, 0, 4, st) != cudaSuccess) return VQ_ERR_CUDA;
  const int64_t n = M * K / 2;
  k_a8_pack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      (const uint16_t*)codes->data, (const uint16_t*)scales->data, (uint8_t*)aq, as, (int)M,
      (int)K, d_inexact);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_w4a8_linear_small(const void* aq, const float* as, const void* wq, const void* ws,
                         int64_t M, int64_t N, int64_t K, const void* bias, float* workspace,
                         void* out, void* stream) {
  if (!aq || !as || !wq || !ws || !workspace || !out) return VQ_ERR_NULL;
  if (M <= 0 || M > 16 || N <= 0 || K <= 0 || K % 64) return VQ_ERR_UNSUPPORTED;
  if (N * K >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(workspace, 0, sizeof(float) * M * N, st) != cudaSuccess) return VQ_ERR_CUDA;
  Args p;
  p.wq = (const uint8_t*)wq;
  p.ws = (const uint8_t*)ws;
  p.aq = (const uint8_t*)aq;
  p.as = as;
  p.acc = workspace;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  const int rb = (int)((N + ROWS - 1) / ROWS), groups = (int)(K / 64);
  int splits = std::max(1, (2 * sms() + rb - 1) / rb);
  splits = std::min(splits, std::max(1, groups / 4));
  p.groups_per_split = (groups + splits - 1) / splits;
  splits = (groups + p.groups_per_split - 1) / p.groups_per_split;
  k_w4a8<<<dim3(rb, splits), WARPS * 32, 0, st>>>(p);
  const int64_t n = M * N;
  k_w4a8_finalize<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(workspace, (const uint16_t*)bias,
                                                             (uint16_t*)out, (int)M, (int)N);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
