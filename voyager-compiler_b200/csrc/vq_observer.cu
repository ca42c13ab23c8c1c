// The amax observer behind per-tensor and per-channel fake quantization:
// FusedAmaxObsFakeQuantize._update_amax_scale
// (src/voyager_compiler/quantization/fake_quantize.py:494-527).
//
// One call folds the input's absolute maximum (over every axis, or every
// axis but ch_axis) into the amax history [L, C] and recomputes the scale
// [C] from the history as it was BEFORE the fold:
//
//   amax     = max over l of history[l]                (NaN propagates)
//   history  = roll(history, -1, 0); history[0] = amax_cur
//   sf       = amax / quant_max                        (float32 division)
//   sf       = amax > 0 and finite(amax) ? sf : scale
//   pow2:  sf = 2 ^ ceil(log2(sf))
//   scale    = sf
//
// The roll-then-overwrite keeps history[0] = amax_cur, history[i] = the old
// history[i + 1] for 1 <= i <= L - 2 and history[L - 1] = the old
// history[0]: the old history[1] is the one dropped.
//
// Kernels: the input is viewed as [O, C, I] (C channels, I contiguous
// elements per channel run; per-tensor is C = 1).  Long runs (I >= 32, or
// C = 1) are cut into segments of at most SEG elements, one warp each, 16-byte
// loads where the run is aligned; short runs (channel-last, I < 32) go
// column-wise over the [O, C * I] view with each thread keeping one column.
// Partial maxima meet in a float32 workspace [C] by integer atomicMax on the
// magnitudes' bit patterns: for non-negative floats the unsigned order is
// the float order, and every NaN pattern sorts above +inf, so a NaN anywhere
// in a channel makes its amax NaN, as torch.amax does.  A second launch, one
// thread per channel, updates the history and the scale.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "vq_numerics.cuh"
#include "voyager_b200.h"

namespace vq {
namespace obs {

constexpr int SEG = 2048;  // elements per warp segment of a long run

// |x| as float32 bit patterns
__device__ __forceinline__ uint32_t mag_f32(uint32_t bits) { return bits & 0x7FFFFFFFu; }
__device__ __forceinline__ uint32_t mag_bf16(uint32_t bits16) { return (bits16 << 16) & 0x7FFFFFFFu; }

struct ObsArgs {
  const void* in;
  int is_bf16;
  int64_t C, I;          // channels, contiguous run length
  int64_t runs;          // O * C
  int64_t segs_per_run;  // ceil(I / SEG)
  int64_t W;             // C * I (column view)
  int64_t rows;          // O (column view)
  int64_t stride;        // column view: threads, a multiple of W
  int vec;               // every run starts 16-byte aligned: 16-byte loads
  uint32_t* ws;          // [C] float32 bit patterns of the amax, zeroed
};

// Long runs: warp per segment, grid-stride.
__global__ void __launch_bounds__(256) k_amax_runs(const __grid_constant__ ObsArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t nseg = a.runs * a.segs_per_run;
  const bool vec = a.vec != 0;
  for (int64_t s = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; s < nseg; s += warps) {
    const int64_t run = s / a.segs_per_run, off = (s % a.segs_per_run) * SEG;
    const int64_t n = min((int64_t)SEG, a.I - off);
    const int64_t base = run * a.I + off;
    uint32_t m = 0;
    if (vec && n == SEG) {
      // a whole aligned segment: every load of the lane in flight at once
      constexpr int NV = SEG * 2 / (32 * 16);  // bf16: 8 x 16 bytes a lane
      if (a.is_bf16) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.in) + base);
        uint4 v[NV];
#pragma unroll
        for (int u = 0; u < NV; ++u) v[u] = __ldcs(p + lane + 32 * u);
#pragma unroll
        for (int u = 0; u < NV; ++u) {
          const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) m = max(m, max(mag_bf16(w[j] & 0xFFFFu), mag_bf16(w[j] >> 16)));
        }
      } else {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint32_t*>(a.in) + base);
        uint4 v[2 * NV];
#pragma unroll
        for (int u = 0; u < 2 * NV; ++u) v[u] = __ldcs(p + lane + 32 * u);
#pragma unroll
        for (int u = 0; u < 2 * NV; ++u)
          m = max(max(m, max(mag_f32(v[u].x), mag_f32(v[u].y))), max(mag_f32(v[u].z), mag_f32(v[u].w)));
      }
    } else if (a.is_bf16) {
      const uint16_t* p = static_cast<const uint16_t*>(a.in) + base;
      if (vec) {
        for (int64_t i = (int64_t)lane * 8; i < n; i += 256) {
          const uint4 v = *reinterpret_cast<const uint4*>(p + i);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) m = max(m, max(mag_bf16(w[j] & 0xFFFFu), mag_bf16(w[j] >> 16)));
        }
      } else {
        for (int64_t i = lane; i < n; i += 32) m = max(m, mag_bf16(p[i]));
      }
    } else {
      const uint32_t* p = static_cast<const uint32_t*>(a.in) + base;
      if (vec) {
        for (int64_t i = (int64_t)lane * 4; i < n; i += 128) {
          const uint4 v = *reinterpret_cast<const uint4*>(p + i);
          m = max(max(m, max(mag_f32(v.x), mag_f32(v.y))), max(mag_f32(v.z), mag_f32(v.w)));
        }
      } else {
        for (int64_t i = lane; i < n; i += 32) m = max(m, mag_f32(p[i]));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0 && m) atomicMax(a.ws + run % a.C, m);
  }
}

// Short runs: thread g keeps column g % W of the [rows, W] view (stride is
// a multiple of W), rows g / W, g / W + stride / W, ...
__global__ void __launch_bounds__(256) k_amax_cols(const __grid_constant__ ObsArgs a) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= a.stride) return;
  const int64_t col = g % a.W, rstep = a.stride / a.W;
  uint32_t m = 0;
  for (int64_t r = g / a.W; r < a.rows; r += rstep) {
    const int64_t e = r * a.W + col;
    m = max(m, a.is_bf16 ? mag_bf16(static_cast<const uint16_t*>(a.in)[e])
                         : mag_f32(static_cast<const uint32_t*>(a.in)[e]));
  }
  if (m) atomicMax(a.ws + col / a.I, m);
}

// ceil(log2(sf)) as torch's float32 log2 gives it: the logarithm rounded to
// float32, then its ceiling (log2 is taken in double precision and rounded
// once; for every float32 the double result lies far closer to the exact
// value than the float32 rounding boundaries it is compared with).
__device__ __forceinline__ float pow2_ceil(float sf) {
  if (!(sf > 0.0f)) return sf == 0.0f ? 0.0f : __int_as_float(0x7FC00000);  // log2 of 0 / < 0 / NaN
  if (isinf(sf)) return sf;
  const float t = ceilf(__double2float_rn(log2((double)sf)));
  if (t > 127.0f) return __int_as_float(0x7F800000);
  if (t < -149.0f) return 0.0f;
  return ldexpf(1.0f, (int)t);  // exact: a power of two in float32's range
}

__device__ __forceinline__ float nanmax(float a, float b) {
  return (isnan(a) || isnan(b)) ? __int_as_float(0x7FC00000) : fmaxf(a, b);
}

__global__ void k_amax_update(const uint32_t* ws, float* hist, int64_t L, int64_t C, float* scale,
                              float qmax, int pow2, int reset) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  if (reset) {  // lazily sized: history zero, scale one
    for (int64_t l = 0; l < L; ++l) hist[l * C + c] = 0.0f;
    scale[c] = 1.0f;
  }
  float amax = hist[c];
  for (int64_t l = 1; l < L; ++l) amax = nanmax(amax, hist[l * C + c]);
  const float old0 = hist[c];
  for (int64_t l = 0; l + 1 < L; ++l) hist[l * C + c] = hist[(l + 1) * C + c];
  hist[(L - 1) * C + c] = old0;
  hist[c] = __uint_as_float(ws[c]);
  float sf = __fdiv_rn(amax, qmax);
  if (!(amax > 0.0f) || !isfinite(amax)) sf = scale[c];
  if (pow2) sf = pow2_ceil(sf);
  scale[c] = sf;
}

}  // namespace obs
}  // namespace vq

using namespace vq::obs;

extern "C" {

int vq_amax_observe(const vq_tensor* input, int32_t per_channel, int32_t ch_axis, float* amax_history,
                    int64_t history_len, float* scale, float quant_max, int32_t power_of_two,
                    int32_t reset, float* workspace, void* stream) {
  if (!input || !amax_history || !scale || !workspace) return VQ_ERR_NULL;
  if (!input->data) return VQ_ERR_NULL;
  if (input->dtype != VQ_BF16 && input->dtype != VQ_F32) return VQ_ERR_UNSUPPORTED;
  if (input->ndim < 0 || input->ndim > VQ_MAX_DIMS || history_len <= 0) return VQ_ERR_INVALID;
  int64_t numel = 1;
  for (int d = 0; d < input->ndim; ++d) {
    if (input->shape[d] < 0) return VQ_ERR_INVALID;
    numel *= input->shape[d];
  }
  if (numel == 0) return VQ_ERR_INVALID;  // torch.amax of an empty reduction raises
  int64_t C = 1, I = numel;
  if (per_channel) {
    if (input->ndim == 0 || ch_axis < 0 || ch_axis >= input->ndim) return VQ_ERR_INVALID;
    C = input->shape[ch_axis];
    I = 1;
    for (int d = ch_axis + 1; d < input->ndim; ++d) I *= input->shape[d];
  }
  const int esz = input->dtype == VQ_BF16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(input->data) & (esz - 1)) ||
      (reinterpret_cast<uintptr_t>(workspace) & 3) || (reinterpret_cast<uintptr_t>(amax_history) & 3) ||
      (reinterpret_cast<uintptr_t>(scale) & 3))
    return VQ_ERR_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(workspace, 0, (size_t)C * sizeof(float), st) != cudaSuccess) return VQ_ERR_CUDA;
  ObsArgs a = {};
  a.in = input->data;
  a.is_bf16 = input->dtype == VQ_BF16;
  a.C = C;
  a.I = I;
  a.runs = numel / I;
  a.ws = reinterpret_cast<uint32_t*>(workspace);
  a.vec = ((I * esz) & 15) == 0 && (reinterpret_cast<uintptr_t>(input->data) & 15) == 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  if (I >= 32 || C == 1) {
    a.segs_per_run = (I + SEG - 1) / SEG;
    const int64_t nseg = a.runs * a.segs_per_run;
    // exactly the CTAs that fit at once: the grid-stride loop takes the rest
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_amax_runs, 256, 0) != cudaSuccess ||
        per_sm <= 0)
      per_sm = 8;
    const int64_t blocks = std::min<int64_t>((nseg + 7) / 8, (int64_t)sms * per_sm);
    k_amax_runs<<<(unsigned)blocks, 256, 0, st>>>(a);
  } else {
    a.W = C * I;
    a.rows = numel / a.W;
    const int64_t target = (int64_t)sms * 2048;
    a.stride = a.W * std::max<int64_t>(1, std::min<int64_t>(a.rows, target / a.W));
    k_amax_cols<<<(unsigned)((a.stride + 255) / 256), 256, 0, st>>>(a);
  }
  if (cudaGetLastError() != cudaSuccess) return VQ_ERR_CUDA;
  k_amax_update<<<(unsigned)((C + 255) / 256), 256, 0, st>>>(a.ws, amax_history, history_len, C, scale,
                                                             quant_max, power_of_two ? 1 : 0,
                                                             reset ? 1 : 0);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
