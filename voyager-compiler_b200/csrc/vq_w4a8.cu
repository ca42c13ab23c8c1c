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
// Per warp: 32 weight rows x 16 tokens, mma.sync.m16n8k16 with bf16 operands
// that carry their block scales exactly:
//   weights  16-byte loads (32 E2M1 codes of one row), each nibble pair ->
//            f16x2 (cvt.rn.f16x2.e2m1x2) times its E4M3 block scale (exact in
//            f16), then bf16 (exact: at most 6 significant bits);
//   tokens   dequantized once to bf16 [16, K] exactly as _dequantize_mx
//            does (one bf16 rounding of code x scale), rows past M zero.
// With both operands exact, every MMA sums exact products in float32, so K
// can be permuted freely: thread t of a quad holds the 32 consecutive K values
// 32t..32t+31 of each 128-wide chunk, and MMA step s takes its logical k
// {2t, 2t+1, 2t+8, 2t+9} from physical 32t + 4s + {0, 1, 2, 3} in both
// operands.  The K range is split over CTAs; partial sums meet in a float32
// workspace (red.add), then a finalize pass adds the bias and rounds to bf16.
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
  const uint16_t* a;   // bf16 [16, K] dequantized tokens (rows >= M zero)
  float* acc;          // [M, N] float32 workspace, zeroed
  int M, N, K, chunks_per_split;
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
// an f16x2 whose values are exact in bf16 -> bf16x2
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
  const float2 f = __half22float2(*reinterpret_cast<__half2*>(&h));
  __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<uint32_t*>(&b);
}
__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

// 16 bytes of E2M1 codes (32 k) with the two E4M3 scales of their blocks of
// 16 -> 16 bf16x2 (k pairs in order).
__device__ __forceinline__ void dequant32(const uint4 w, uint32_t sc2, uint32_t (&o)[16]) {
  const uint32_t s0 = e4m3x2_to_f16x2((sc2 & 0xFFu) * 0x101u);
  const uint32_t s1 = e4m3x2_to_f16x2(((sc2 >> 8) & 0xFFu) * 0x101u);
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int b = 0; b < 4; ++b)
      o[4 * q + b] = f16x2_to_bf16x2(hmul2(e2m1x2_to_f16x2((ww[q] >> (8 * b)) & 0xFFu),
                                           q < 2 ? s0 : s1));
}

__global__ void __launch_bounds__(WARPS * 32) k_w4a8(const __grid_constant__ Args p) {
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
  uint32_t sc[4];
  auto load = [&](int c) {
    const int k0 = c * 128 + 32 * t;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const size_t r = (size_t)(row0 + 8 * i);
      w[i] = ok[i] ? ld_stream(p.wq + r * wrow + k0 / 2) : make_uint4(0, 0, 0, 0);
      sc[i] = ok[i] ? *reinterpret_cast<const uint16_t*>(p.ws + r * srow + k0 / 16) : 0u;
    }
  };
  if (c0 < c1) load(c0);
  for (int c = c0; c < c1; ++c) {
    const uint4 wc[4] = {w[0], w[1], w[2], w[3]};
    const uint32_t scc[4] = {sc[0], sc[1], sc[2], sc[3]};
    if (c + 1 < c1) load(c + 1);
    const int k0 = c * 128 + 32 * t;
    // tokens g and g + 8: their 32 values at k0 (bf16 pairs in k order)
    uint32_t b0[16], b1[16];
    const uint4* a0p = reinterpret_cast<const uint4*>(p.a + (size_t)g * p.K + k0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = a0p[j];
      b0[4 * j] = v.x; b0[4 * j + 1] = v.y; b0[4 * j + 2] = v.z; b0[4 * j + 3] = v.w;
    }
    if (two) {
      const uint4* a1p = reinterpret_cast<const uint4*>(p.a + (size_t)(g + 8) * p.K + k0);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = a1p[j];
        b1[4 * j] = v.x; b1[4 * j + 1] = v.y; b1[4 * j + 2] = v.z; b1[4 * j + 3] = v.w;
      }
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      uint32_t ra[16], rb[16];  // rows row0 + 16 mt and + 8
      dequant32(wc[2 * mt], scc[2 * mt], ra);
      dequant32(wc[2 * mt + 1], scc[2 * mt + 1], rb);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        mma_bf16(acc[mt][0], ra[2 * s], rb[2 * s], ra[2 * s + 1], rb[2 * s + 1], b0[2 * s],
                 b0[2 * s + 1]);
        if (two)
          mma_bf16(acc[mt][1], ra[2 * s], rb[2 * s], ra[2 * s + 1], rb[2 * s + 1], b1[2 * s],
                   b1[2 * s + 1]);
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

// activations: bf16 codes [M, K] x bf16 scales [M, K/32] -> bf16 [16, K] (rows
// >= M zero): the reference's _dequantize_mx, one bf16 rounding of the
// float32 product, so the MMA operand is the reference's own value.
__global__ void k_a8_dequant(const uint16_t* codes, const uint16_t* scales, uint16_t* out, int M,
                             int K) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one element of [16, K]
  if (i >= (int64_t)16 * K) return;
  const int m = (int)(i / K), k = (int)(i % K);
  uint16_t v = 0;
  if (m < M)
    v = (uint16_t)f2bf(bf2f(codes[(int64_t)m * K + k]) * bf2f(scales[(int64_t)m * (K / 32) + k / 32]));
  out[i] = v;
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

int vq_a8_dequant(const vq_tensor* codes, const vq_tensor* scales, void* out16, void* stream) {
  if (!codes || !scales || !out16) return VQ_ERR_NULL;
  if (codes->dtype != VQ_BF16 || scales->dtype != VQ_BF16) return VQ_ERR_UNSUPPORTED;
  if (codes->ndim != 2 || scales->ndim != 2) return VQ_ERR_SHAPE;
  const int64_t M = codes->shape[0], K = codes->shape[1];
  if (K % 128 || M <= 0 || M > 16 || scales->shape[0] != M || scales->shape[1] != K / 32)
    return VQ_ERR_SHAPE;
  if (K >= (1ll << 26)) return VQ_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n = 16 * K;
  k_a8_dequant<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      (const uint16_t*)codes->data, (const uint16_t*)scales->data, (uint16_t*)out16, (int)M,
      (int)K);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_w4a8_linear_small(const void* a16, const void* wq, const void* ws, int64_t M, int64_t N,
                         int64_t K, const void* bias, float* workspace, void* out, void* stream) {
  if (!a16 || !wq || !ws || !workspace || !out) return VQ_ERR_NULL;
  if (M <= 0 || M > 16 || N <= 0 || K <= 0 || K % 128) return VQ_ERR_UNSUPPORTED;
  if (N * K >= (1ll << 31)) return VQ_ERR_UNSUPPORTED;
  const void* ptrs[3] = {a16, wq, ws};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15) return VQ_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(workspace, 0, sizeof(float) * M * N, st) != cudaSuccess) return VQ_ERR_CUDA;
  Args p;
  p.wq = (const uint8_t*)wq;
  p.ws = (const uint8_t*)ws;
  p.a = (const uint16_t*)a16;
  p.acc = workspace;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  const int rb = (int)((N + ROWS - 1) / ROWS), chunks = (int)(K / 128);
  // about two CTAs per SM, at least 2 chunks per CTA
  int splits = std::max(1, (2 * sms() + rb - 1) / rb);
  splits = std::min(splits, std::max(1, chunks / 2));
  p.chunks_per_split = (chunks + splits - 1) / splits;
  splits = (chunks + p.chunks_per_split - 1) / p.chunks_per_split;
  k_w4a8<<<dim3(rb, splits), WARPS * 32, 0, st>>>(p);
  const int64_t n = M * N;
  k_w4a8_finalize<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(workspace, (const uint16_t*)bias,
                                                             (uint16_t*)out, (int)M, (int)N);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
