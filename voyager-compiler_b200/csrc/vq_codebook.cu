// Codebooks with one table per region of the tensor (quantized.py:211-337):
// a codebook [*counts, k] splits axis d of the tensor into counts[d] equal
// regions; an element's region picks the table its value is encoded against
// (or its index decoded through).  Both encode and decode are functions of
// the element's bfloat16 pattern within its region, so each region's table
// is built once on the host as 65,536 entries of the output dtype, and
// k_codebook_lookup gathers out[i] = table[region(i)][bf16 pattern of in[i]].
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>

#include "voyager_b200.h"
#include "vq_numerics.cuh"

namespace vq {
namespace cb {

struct LookupArgs {
  const void* in;
  void* out;
  const void* tables;  // [regions][65536], the output dtype
  int64_t n;
  int32_t ndim;
  int32_t in_bf16, out_bf16;
  int64_t shape[VQ_MAX_DIMS];
  int64_t tile[VQ_MAX_DIMS];     // extent of one region along each dim
  int64_t rstride[VQ_MAX_DIMS];  // region index stride of each dim
};

__global__ void __launch_bounds__(256) k_codebook_lookup(const __grid_constant__ LookupArgs a) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += step) {
    int64_t rem = i, r = 0;
    for (int d = a.ndim - 1; d >= 0; --d) {
      const int64_t c = rem % a.shape[d];
      rem /= a.shape[d];
      r += (c / a.tile[d]) * a.rstride[d];
    }
    const uint32_t p = a.in_bf16 ? (uint32_t)reinterpret_cast<const uint16_t*>(a.in)[i]
                                 : f2bf(reinterpret_cast<const float*>(a.in)[i]);
    const int64_t e = (r << 16) + p;
    if (a.out_bf16)
      reinterpret_cast<uint16_t*>(a.out)[i] = reinterpret_cast<const uint16_t*>(a.tables)[e];
    else
      reinterpret_cast<float*>(a.out)[i] = reinterpret_cast<const float*>(a.tables)[e];
  }
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? VQ_OK : VQ_ERR_CUDA; }

}  // namespace cb
}  // namespace vq

using namespace vq::cb;

extern "C" {

int vq_codebook_lookup(const vq_tensor* input, const int64_t* counts, int32_t ncounts,
                       const void* tables, int64_t nregions, vq_tensor* out, void* stream) {
  if (!input || !counts || !tables || !out) return VQ_ERR_NULL;
  if ((input->dtype != VQ_BF16 && input->dtype != VQ_F32) ||
      (out->dtype != VQ_BF16 && out->dtype != VQ_F32))
    return VQ_ERR_UNSUPPORTED;
  if (input->ndim < 1 || input->ndim > VQ_MAX_DIMS || ncounts != input->ndim ||
      out->ndim != input->ndim)
    return VQ_ERR_INVALID;
  LookupArgs a;
  memset(&a, 0, sizeof(a));
  int64_t n = 1, regions = 1;
  for (int d = 0; d < input->ndim; ++d) {
    if (out->shape[d] != input->shape[d]) return VQ_ERR_SHAPE;
    if (counts[d] < 1 || input->shape[d] % counts[d]) return VQ_ERR_SHAPE;
    a.shape[d] = input->shape[d];
    a.tile[d] = std::max<int64_t>(input->shape[d] / counts[d], 1);
    n *= input->shape[d];
  }
  for (int d = input->ndim - 1; d >= 0; --d) {
    a.rstride[d] = regions;
    regions *= counts[d];
  }
  if (regions != nregions) return VQ_ERR_SHAPE;
  if (n == 0) return VQ_OK;
  if (!input->data || !out->data) return VQ_ERR_NULL;
  a.in = input->data;
  a.out = out->data;
  a.tables = tables;
  a.n = n;
  a.ndim = input->ndim;
  a.in_bf16 = input->dtype == VQ_BF16;
  a.out_bf16 = out->dtype == VQ_BF16;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 16);
  k_codebook_lookup<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
