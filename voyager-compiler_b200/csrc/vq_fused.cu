// Decoder-graph fusions around quantize_mx (MXFP8 activations: E4M3 table,
// power-of-two block-32 scales along the last dim).  Each kernel computes
// the bf16 graph ops that feed a quantize_mx in a converted LLaMA layer and
// quantizes the result in the same pass, writing what quantize_mx returns
// (bf16 codes, bf16 scales) and the tcgen05 operand (E4M3 bytes + UE8M0
// scale atoms, the layout vq_mx_pack writes):
//
//   k_rms_qmx      RMSNorm (float32 statistics, bf16 cast, times the bf16
//                  weight) -> quantize_mx                 (input_layernorm)
//   k_rope_qmx     rotate-half RoPE of q and k heads -> quantize_mx along
//                  head_dim, written head-major [B, H, S, 128]
//   k_vt_qmx       v heads quantized along the tokens (blocks of 32 tokens),
//                  written transposed [B, H, 128, S]
//   k_swiglu_qmx   bf16(silu(gate)) * up -> quantize_mx   (MLP act_fn)
//
// The element quantization is the one quantize_mx does: scale =
// pow2_scale_bf16(block amax), code = E4M3(bf16(x / scale)) by the hardware
// conversion (exact for E4M3 tables, -0 -> +0, NaN -> the table's NaN).
// bf16 ops round as torch's CUDA kernels do (float math, one rounding per
// op; silu as x / (1 + expf(-x))).  RMSNorm's sum of squares is reduced in
// this kernel's own order.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "vq_hw.cuh"
#include "vq_numerics.cuh"

namespace vq {
namespace fused {

constexpr uint32_t FULL = 0xFFFFFFFFu;

__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_rn(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

// x / s for a power-of-two bf16 scale s (bits sbits), exactly: a product
// with 1 / s where that is a normal float, the IEEE division otherwise.
__device__ __forceinline__ float div_pow2(float x, uint32_t sbits) {
  const uint32_t E = (sbits >> 7) & 0xFFu;
  if (E >= 1u && E <= 253u) return x * __uint_as_float((254u - E) << 23);
  return __fdiv_rn(x, bf2f(sbits));
}

// The two E4M3 bytes of two E4M3 values held as bf16 (lo, hi halves).
__device__ __forceinline__ uint32_t e4m3_bytes(uint32_t codes2) {
  uint16_t b;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(b) : "f"(hi_f(codes2)), "f"(lo_f(codes2)));
  return b;
}

// MXFP8 quantization of 8 consecutive bf16 values (4 packed pairs) held by
// each of 4 consecutive lanes (lane % 4 = 0..3, all four active) that
// together cover one block of 32.  Returns
// the block's scale (bf16 bits); codes as bf16 pairs and E4M3 bytes.
__device__ __forceinline__ uint32_t mx8_quant8(const uint32_t (&v)[4], int fl2q, uint32_t nan_bits,
                                               uint32_t (&codes)[4], uint32_t (&bytes)[2]) {
  const uint32_t a0 = v[0] & 0x7FFF7FFFu, a1 = v[1] & 0x7FFF7FFFu, a2 = v[2] & 0x7FFF7FFFu,
                 a3 = v[3] & 0x7FFF7FFFu;
  uint32_t m = __vmaxu2(__vmaxu2(a0, a1), __vmaxu2(a2, a3));
  uint32_t mn = __vminu2(__vminu2(a0, a1), __vminu2(a2, a3));
  m = max(m & 0xFFFFu, m >> 16);
  mn = min(mn & 0xFFFFu, mn >> 16);
  const uint32_t lane_max = m;
  const unsigned quad = 0xFu << ((threadIdx.x & 31) & 28);  // the block's 4 lanes
  m = max(m, __shfl_xor_sync(quad, m, 1));
  m = max(m, __shfl_xor_sync(quad, m, 2));
  const uint32_t sbits = pow2_scale_bf16(m, fl2q);
  const uint32_t E = (sbits >> 7) & 0xFFu;
  const float inv = __uint_as_float((254u - E) << 23);
  uint32_t b16[4];
  if (plain_quotients(E, inv, mn, lane_max)) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      b16[k] = e4m3_pair(pack_rn(lo_f(v[k]) * inv, hi_f(v[k]) * inv), codes[k]);
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float q0 = div_pow2(lo_f(v[k]), sbits), q1 = div_pow2(hi_f(v[k]), sbits);
      codes[k] = hw_pair<K_HW_E4M3>(pair_index<K_HW_E4M3>(q0, q1), nan_bits);
      b16[k] = e4m3_bytes(codes[k]);
    }
  }
  bytes[0] = b16[0] | (b16[1] << 16);
  bytes[1] = b16[2] | (b16[3] << 16);
  return sbits;
}

// Byte offset of (row, K block kb) in the scale atoms [KT][RT][512].
__device__ __forceinline__ size_t atom_off(int64_t row, int kb, int RT) {
  const int kt = kb >> 2, j = kb & 3;
  const int64_t rt = row >> 7;
  const int rr = (int)(row & 127);
  return ((size_t)kt * RT + rt) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + j;
}

struct Out {
  uint16_t* codes;   // bf16 [R, C]
  uint16_t* scale;   // bf16 [R, C / 32]
  uint8_t* packed;   // E4M3 [RT * 128, Cp]
  uint8_t* sf;       // UE8M0 atoms [Cp / 128][RT][512]
  int C, Cp, RT;
};

// One lane's 8 values at (row, col) of an [R, C] operand: codes, scale (by
// the first lane of the block), E4M3 bytes and the atom byte.
__device__ __forceinline__ void store8(const Out& o, int64_t row, int col, const uint32_t (&v)[4],
                                       int fl2q, uint32_t nan_bits, int lane4) {
  uint32_t codes[4], bytes[2];
  const uint32_t sbits = mx8_quant8(v, fl2q, nan_bits, codes, bytes);
  *reinterpret_cast<uint4*>(o.codes + row * o.C + col) =
      make_uint4(codes[0], codes[1], codes[2], codes[3]);
  *reinterpret_cast<uint2*>(o.packed + row * o.Cp + col) = make_uint2(bytes[0], bytes[1]);
  if (lane4 == 0) {
    o.scale[row * (o.C / 32) + col / 32] = (uint16_t)sbits;
    o.sf[atom_off(row, col / 32, o.RT)] = (uint8_t)((sbits >> 7) & 0xFFu);
  }
}

// The columns [C, Cp) of a packed operand: zero codes, scale 2^0.
__device__ __forceinline__ void pad_row(const Out& o, int64_t row, int lane, int nl) {
  for (int c = o.C + lane * 8; c < o.Cp; c += nl * 8) {
    *reinterpret_cast<uint2*>(o.packed + row * o.Cp + c) = make_uint2(0u, 0u);
    if ((c & 31) == 0) o.sf[atom_off(row, c / 32, o.RT)] = 127;
  }
}

// ---------------------------------------------------------------------------
struct RmsArgs {
  const uint16_t* x;  // bf16 [R, C]
  const uint16_t* w;  // bf16 [C]
  Out o;
  int R;
  float eps;
  int fl2q;
  uint32_t nan_bits;
};

// One warp per row: sum of squares, then the normalised row quantized.
__global__ void __launch_bounds__(256, 6) k_rms_qmx(const __grid_constant__ RmsArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= a.R) return;
  const int C = a.o.C;
  const uint16_t* xr = a.x + row * C;
  float acc = 0.f;
  for (int c = lane * 8; c < C; c += 256) {
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
  for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(FULL, acc, o);
  const float r = rsqrtf(__fdiv_rn(acc, (float)C) + a.eps);
  for (int c = lane * 8; c < C; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 g = *reinterpret_cast<const uint4*>(a.w + c);
    const uint32_t xw[4] = {u.x, u.y, u.z, u.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t y = pack_rn(lo_f(xw[k]) * r, hi_f(xw[k]) * r);
      v[k] = pack_rn(lo_f(gw[k]) * lo_f(y), hi_f(gw[k]) * hi_f(y));
    }
    store8(a.o, row, c, v, a.fl2q, a.nan_bits, lane & 3);
  }
  pad_row(a.o, row, lane, 32);
}

// ---------------------------------------------------------------------------
struct RopeArgs {
  const uint16_t* qkv;  // bf16 [B*S, ld]: q heads at q_off, k heads at k_off
  int64_t ld;
  int q_off, k_off;
  const uint16_t* cos;  // bf16 [S, 128]
  const uint16_t* sin;
  Out q, k;             // [B*H*S, 128] each (head-major rows)
  int B, S, H;
  int fl2q;
  uint32_t nan_bits;
};

// 16 lanes per (token, head) row of 128: lane j holds dims 8j..8j+7; the
// rotate-half partner is lane j ^ 8.
__global__ void __launch_bounds__(256) k_rope_qmx(const __grid_constant__ RopeArgs a) {
  // rows < 2^27 (checked by the host): 32-bit index arithmetic
  const uint32_t gid = blockIdx.x * 256u + threadIdx.x;
  const uint32_t rows = (uint32_t)a.B * a.S * a.H;
  const uint32_t row = gid >> 4;  // token-major: (b, s, h)
  const int j = (int)(gid & 15);
  if (row >= rows) return;  // whole 16-lane groups leave together
  const int h = (int)(row % (uint32_t)a.H);
  const uint32_t t = row / (uint32_t)a.H;  // b * S + s
  const int s = (int)(t % (uint32_t)a.S), b = (int)(t / (uint32_t)a.S);
  const int d0 = j * 8;
  const uint4 cu = *reinterpret_cast<const uint4*>(a.cos + (int64_t)s * 128 + d0);
  const uint4 su = *reinterpret_cast<const uint4*>(a.sin + (int64_t)s * 128 + d0);
  const uint32_t cw[4] = {cu.x, cu.y, cu.z, cu.w}, sw[4] = {su.x, su.y, su.z, su.w};
  const int64_t orow = ((int64_t)b * a.H + h) * a.S + s;
  const unsigned gmask = 0xFFFFu << ((threadIdx.x & 31) & 16);  // this row's 16 lanes
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const uint16_t* src = a.qkv + t * a.ld + (which ? a.k_off : a.q_off) + h * 128 + d0;
    const uint4 xu = *reinterpret_cast<const uint4*>(src);
    uint32_t x[4] = {xu.x, xu.y, xu.z, xu.w}, p[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = __shfl_xor_sync(gmask, x[k], 8);
    uint32_t v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // rot = cat(-x[64:], x[:64]): lanes 0-7 take the negated upper half
      const uint32_t rot = j < 8 ? (p[k] ^ 0x80008000u) : p[k];
      const uint32_t t1 = pack_rn(lo_f(x[k]) * lo_f(cw[k]), hi_f(x[k]) * hi_f(cw[k]));
      const uint32_t t2 = pack_rn(lo_f(rot) * lo_f(sw[k]), hi_f(rot) * hi_f(sw[k]));
      v[k] = pack_rn(lo_f(t1) + lo_f(t2), hi_f(t1) + hi_f(t2));
    }
    store8(which ? a.k : a.q, orow, d0, v, a.fl2q, a.nan_bits, j & 3);
  }
}

// ---------------------------------------------------------------------------
struct VtArgs {
  const uint16_t* qkv;  // bf16 [B*S, ld]: v heads at v_off
  int64_t ld;
  int v_off;
  Out o;                // rows (b, h, d): [B*H*128, S]
  int B, S, H;
  int fl2q;
  uint32_t nan_bits;
};

// One thread per (b, h, block of 32 tokens, pair of dims): the 32 x 2
// values, a scale per dim, codes written along the tokens.
__global__ void __launch_bounds__(256, 3) k_vt_qmx(const __grid_constant__ VtArgs a) {
  // total < 2^31 (checked by the host): 32-bit index arithmetic
  const uint32_t gid = blockIdx.x * 256u + threadIdx.x;
  const uint32_t nsb = (uint32_t)a.S / 32;
  const uint32_t total = (uint32_t)a.B * a.H * nsb * 64;
  if (gid >= total) return;
  const int dp = (int)(gid & 63);          // dims 2dp, 2dp + 1
  const uint32_t r = gid >> 6;
  const int h = (int)(r % (uint32_t)a.H);
  const uint32_t r2 = r / (uint32_t)a.H;
  const int sb = (int)(r2 % nsb), b = (int)(r2 / nsb);
  const uint16_t* src = a.qkv + ((int64_t)b * a.S + sb * 32) * a.ld + a.v_off + h * 128 + 2 * dp;
  uint32_t w[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) w[i] = *reinterpret_cast<const uint32_t*>(src + i * a.ld);
  // magnitudes of both dims at once: lo half = dim 2dp, hi half = 2dp + 1
  uint32_t mx2 = 0, mn2 = 0xFFFFFFFFu;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    mx2 = __vmaxu2(mx2, w[i] & 0x7FFF7FFFu);
    mn2 = __vminu2(mn2, w[i] & 0x7FFF7FFFu);
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t m = half ? mx2 >> 16 : mx2 & 0xFFFFu;
    const uint32_t mn = half ? mn2 >> 16 : mn2 & 0xFFFFu;
    const uint32_t sbits = pow2_scale_bf16(m, a.fl2q);
    const uint32_t E = (sbits >> 7) & 0xFFu;
    const float inv = __uint_as_float((254u - E) << 23);
    uint32_t codes[16], bytes[8];
    if (plain_quotients(E, inv, mn, m)) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t b[2];
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          const uint32_t e0 = half ? (w[4 * i + 2 * x] >> 16) : (w[4 * i + 2 * x] & 0xFFFFu);
          const uint32_t e1 = half ? (w[4 * i + 2 * x + 1] >> 16) : (w[4 * i + 2 * x + 1] & 0xFFFFu);
          b[x] = e4m3_pair(pack_rn(bf2f(e0) * inv, bf2f(e1) * inv), codes[2 * i + x]);
        }
        bytes[i] = b[0] | (b[1] << 16);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t e0 = half ? (w[2 * i] >> 16) : (w[2 * i] & 0xFFFFu);
        const uint32_t e1 = half ? (w[2 * i + 1] >> 16) : (w[2 * i + 1] & 0xFFFFu);
        const float q0 = div_pow2(bf2f(e0), sbits), q1 = div_pow2(bf2f(e1), sbits);
        codes[i] = hw_pair<K_HW_E4M3>(pair_index<K_HW_E4M3>(q0, q1), a.nan_bits);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        bytes[i] = e4m3_bytes(codes[2 * i]) | (e4m3_bytes(codes[2 * i + 1]) << 16);
    }
    const int64_t row = ((int64_t)b * a.H + h) * 128 + 2 * dp + half;
    uint4* dc = reinterpret_cast<uint4*>(a.o.codes + row * a.o.C + sb * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      dc[i] = make_uint4(codes[4 * i], codes[4 * i + 1], codes[4 * i + 2], codes[4 * i + 3]);
    uint4* dp8 = reinterpret_cast<uint4*>(a.o.packed + row * a.o.Cp + sb * 32);
    dp8[0] = make_uint4(bytes[0], bytes[1], bytes[2], bytes[3]);
    dp8[1] = make_uint4(bytes[4], bytes[5], bytes[6], bytes[7]);
    a.o.scale[row * nsb + sb] = (uint16_t)sbits;
    a.o.sf[atom_off(row, sb, a.o.RT)] = (uint8_t)((sbits >> 7) & 0xFFu);
  }
}

// ---------------------------------------------------------------------------
struct SwigluArgs {
  const uint16_t* gu;  // bf16 [R, ld]: gate at columns [0, C), up at [up_off, up_off + C)
  int64_t ld;
  int64_t up_off;
  Out o;
  int64_t R;
  int fl2q;
  uint32_t nan_bits;
};

// One thread per 8 outputs; a row's padding columns by the threads of its
// last 32-column group.
__global__ void __launch_bounds__(256, 8) k_swiglu_qmx(const __grid_constant__ SwigluArgs a) {
  const int64_t gid = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int per_row = a.o.C / 8;
  if (gid >= a.R * per_row) return;  // per_row % 4 == 0: blocks stay whole
  int64_t row;
  int c;
  if (a.R * per_row <= 0xFFFFFFFFll) {  // 32-bit division where it suffices
    const uint32_t g32 = (uint32_t)gid;
    row = g32 / (uint32_t)per_row;
    c = (int)(g32 - (uint32_t)row * (uint32_t)per_row) * 8;
  } else {
    row = gid / per_row;
    c = (int)(gid % per_row) * 8;
  }
  const uint4 gu4 = *reinterpret_cast<const uint4*>(a.gu + row * a.ld + c);
  const uint4 uu4 = *reinterpret_cast<const uint4*>(a.gu + row * a.ld + a.up_off + c);
  const uint32_t g[4] = {gu4.x, gu4.y, gu4.z, gu4.w}, u[4] = {uu4.x, uu4.y, uu4.z, uu4.w};
  uint32_t v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float g0 = lo_f(g[k]), g1 = hi_f(g[k]);
    const uint32_t s = pack_rn(g0 / (1.0f + expf(-g0)), g1 / (1.0f + expf(-g1)));
    v[k] = pack_rn(lo_f(s) * lo_f(u[k]), hi_f(s) * hi_f(u[k]));
  }
  store8(a.o, row, c, v, a.fl2q, a.nan_bits, (int)(gid & 3));
  if (c + 8 == a.o.C) pad_row(a.o, row, 0, 1);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_out(const Out& o) {
  if (!o.codes || !o.scale || !o.packed || !o.sf) return VQ_ERR_NULL;
  if (!aligned16(o.codes) || !aligned16(o.packed) || !aligned16(o.sf)) return VQ_ERR_ALIGNMENT;
  return VQ_OK;
}

int e4m3_rounder(const vq_rounder* r) {
  if (!r) return VQ_ERR_NULL;
  if (r->kind != VQ_R_MINIFLOAT || r->hw != VQ_HW_E4M3) return VQ_ERR_UNSUPPORTED;
  return VQ_OK;
}

}  // namespace fused
}  // namespace vq

using namespace vq::fused;

extern "C" {

int vq_rmsnorm_quantize_mx(const void* x, const void* weight, int64_t rows, int64_t cols, float eps,
                           const vq_rounder* qmap, int32_t floor_log2_qmax, void* codes,
                           void* scale, void* packed, void* packed_sf, void* stream) {
  int st = e4m3_rounder(qmap);
  if (st) return st;
  if (!x || !weight) return VQ_ERR_NULL;
  if (rows <= 0 || cols <= 0 || cols % 32 || rows >= (1ll << 31)) return VQ_ERR_INVALID;
  Out o{(uint16_t*)codes, (uint16_t*)scale, (uint8_t*)packed, (uint8_t*)packed_sf, (int)cols,
        (int)((cols + 127) / 128 * 128), (int)((rows + 127) / 128)};
  if ((st = check_out(o))) return st;
  if (!aligned16(x) || !aligned16(weight)) return VQ_ERR_ALIGNMENT;
  RmsArgs a{(const uint16_t*)x, (const uint16_t*)weight, o, (int)rows, eps, floor_log2_qmax,
            qmap->nan_bits};
  k_rms_qmx<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_rope_quantize_qk(const void* qkv, int64_t ld, int64_t q_off, int64_t k_off,
                        const void* cos, const void* sin, int64_t batch, int64_t seq,
                        int64_t heads, const vq_rounder* qmap, int32_t floor_log2_qmax,
                        void* q_codes, void* q_scale, void* q_packed, void* q_sf, void* k_codes,
                        void* k_scale, void* k_packed, void* k_sf, void* stream) {
  int st = e4m3_rounder(qmap);
  if (st) return st;
  if (!qkv || !cos || !sin) return VQ_ERR_NULL;
  if (batch <= 0 || seq <= 0 || heads <= 0) return VQ_ERR_INVALID;
  const int64_t rows = batch * seq * heads;
  if (rows >= (1ll << 31) / 16 || ld % 8 || q_off % 8 || k_off % 8 || q_off < 0 || k_off < 0 ||
      q_off + heads * 128 > ld || k_off + heads * 128 > ld)
    return VQ_ERR_UNSUPPORTED;
  const int RT = (int)((rows + 127) / 128);
  Out oq{(uint16_t*)q_codes, (uint16_t*)q_scale, (uint8_t*)q_packed, (uint8_t*)q_sf, 128, 128, RT};
  Out ok{(uint16_t*)k_codes, (uint16_t*)k_scale, (uint8_t*)k_packed, (uint8_t*)k_sf, 128, 128, RT};
  if ((st = check_out(oq)) || (st = check_out(ok))) return st;
  if (!aligned16(qkv) || !aligned16(cos) || !aligned16(sin)) return VQ_ERR_ALIGNMENT;
  RopeArgs a{(const uint16_t*)qkv, ld, (int)q_off, (int)k_off, (const uint16_t*)cos,
             (const uint16_t*)sin, oq, ok, (int)batch, (int)seq, (int)heads, floor_log2_qmax,
             qmap->nan_bits};
  k_rope_qmx<<<(unsigned)((rows * 16 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_quantize_vt(const void* qkv, int64_t ld, int64_t v_off, int64_t batch, int64_t seq,
                   int64_t heads, const vq_rounder* qmap, int32_t floor_log2_qmax, void* codes,
                   void* scale, void* packed, void* packed_sf, void* stream) {
  int st = e4m3_rounder(qmap);
  if (st) return st;
  if (!qkv) return VQ_ERR_NULL;
  if (batch <= 0 || seq <= 0 || heads <= 0) return VQ_ERR_INVALID;
  if (seq % 128 || ld % 8 || v_off % 8 || v_off < 0 || v_off + heads * 128 > ld)
    return VQ_ERR_UNSUPPORTED;
  const int64_t rows = batch * heads * 128;
  if (rows * (seq / 32) >= (1ll << 31) / 64) return VQ_ERR_UNSUPPORTED;
  Out o{(uint16_t*)codes, (uint16_t*)scale, (uint8_t*)packed, (uint8_t*)packed_sf, (int)seq,
        (int)seq, (int)((rows + 127) / 128)};
  if ((st = check_out(o))) return st;
  if (!aligned16(qkv)) return VQ_ERR_ALIGNMENT;
  VtArgs a{(const uint16_t*)qkv, ld, (int)v_off, o, (int)batch, (int)seq, (int)heads,
           floor_log2_qmax, qmap->nan_bits};
  const int64_t total = batch * heads * (seq / 32) * 64;
  k_vt_qmx<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

int vq_swiglu_quantize_mx(const void* gate_up, int64_t ld, int64_t up_off, int64_t rows,
                          int64_t cols, const vq_rounder* qmap, int32_t floor_log2_qmax,
                          void* codes, void* scale, void* packed, void* packed_sf, void* stream) {
  int st = e4m3_rounder(qmap);
  if (st) return st;
  if (!gate_up) return VQ_ERR_NULL;
  if (rows <= 0 || cols <= 0 || cols % 32) return VQ_ERR_INVALID;
  if (ld % 8 || up_off % 8 || up_off < cols || up_off + cols > ld ||
      rows * (cols / 8) >= (1ll << 40))
    return VQ_ERR_UNSUPPORTED;
  Out o{(uint16_t*)codes, (uint16_t*)scale, (uint8_t*)packed, (uint8_t*)packed_sf, (int)cols,
        (int)((cols + 127) / 128 * 128), (int)((rows + 127) / 128)};
  if ((st = check_out(o))) return st;
  if (!aligned16(gate_up)) return VQ_ERR_ALIGNMENT;
  SwigluArgs a{(const uint16_t*)gate_up, ld, up_off, o, rows, floor_log2_qmax, qmap->nan_bits};
  const int64_t total = rows * (cols / 8);
  k_swiglu_qmx<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? VQ_OK : VQ_ERR_CUDA;
}

}  // extern "C"
