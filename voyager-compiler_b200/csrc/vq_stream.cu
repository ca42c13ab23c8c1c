// The streaming floor of one launch: read R bytes and write W bytes of HBM
// with nothing else to do.  A measurement aid with no counterpart in the
// reference: the time of this kernel on a kernel's own byte counts is the
// least that kernel can take as one launch (launch latency, ramp-up and
// drain included), which for the microsecond-scale calls of few-token
// linears and small quantizations sits well below the long-copy bandwidth
// the roofline's peak is measured with.
//
// Up to eight CTAs of 256 threads per SM (as many as fit at once); each
// thread keeps eight 16-byte loads in flight (grid-stride), folds them into one word and, where it has a store
// to make, writes 16 bytes derived from it (so no load is optimized away).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "voyager_b200.h"

namespace vq {
namespace stream {

constexpr int U = 8;

__global__ void __launch_bounds__(256) k_stream(const uint4* __restrict__ src, int64_t r16,
                                                uint4* __restrict__ dst, int64_t w16) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n = r16 > w16 ? r16 : w16;
  uint32_t acc = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += U * stride) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = i + u * stride;
      v[u] = j < r16 ? __ldcs(src + j) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = i + u * stride;
      acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
      if (j < w16) __stcs(dst + j, make_uint4(acc, v[u].y, v[u].z, v[u].w));
    }
  }
}

}  // namespace stream
}  // namespace vq

extern "C" {

int vq_stream_probe(const void* src, int64_t read_bytes, void* dst, int64_t write_bytes,
                    void* stream) {
  if (read_bytes < 0 || write_bytes < 0) return VQ_ERR_INVALID;
  if ((read_bytes && !src) || (write_bytes && !dst)) return VQ_ERR_NULL;
  if ((read_bytes | write_bytes) & 15) return VQ_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15)
    return VQ_ERR_ALIGNMENT;
  if (!read_bytes && !write_bytes) return VQ_OK;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  const int64_t n16 = std::max(read_bytes, write_bytes) / 16;
  // exactly the CTAs that fit at once (no partial second wave)
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, vq::stream::k_stream, 256, 0) !=
          cudaSuccess || per_sm <= 0)
    per_sm = 8;
  const int64_t blocks = std::min<int64_t>((int64_t)sms * std::min(per_sm, 8), (n16 + 255) / 256);
  vq::stream::k_stream<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), read_bytes / 16, static_cast<uint4*>(dst), write_bytes / 16);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
