// Hardware minifloat rounders (cvt.rn.satfinite.{e4m3,e5m2,e2m1}x2.f32):
// the element rounding of a MINIFLOAT table whose values the conversion
// reproduces exactly (vq_rounder.hw, checked on the device by
// vq_rounder_check_hw).  Shared by the quantize kernels and the fused
// decoder kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "vq_numerics.cuh"

namespace vq {

// Element kinds beyond vq_rounder_kind: a MINIFLOAT rounder that the
// hardware conversions reproduce (vq_rounder.hw, verified on the device).
constexpr int K_HW_E4M3 = 10, K_HW_E5M2 = 11, K_HW_E2M1 = 12;

// Two bf16 indices (lo | hi << 16) through a hardware minifloat conversion
// (round-to-nearest-even, saturating) and back: every value of these formats
// is exactly a bf16, so the result is the table entry except for the two
// cases the table treats specially: a -0 index gives +0, a NaN index gives
// nan_bits.
template <int K>
__device__ __forceinline__ uint32_t hw_pair(uint32_t idx2, uint32_t nan_bits) {
  const float lo = __uint_as_float(idx2 << 16);
  const float hi = __uint_as_float(idx2 & 0xFFFF0000u);
  uint32_t h2;
  if (K == K_HW_E4M3) {
    asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(h2) : "f"(hi), "f"(lo));
  } else if (K == K_HW_E5M2) {
    asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e5m2x2.f32 t, %1, %2;\n\t"
        "cvt.rn.f16x2.e5m2x2 %0, t;\n\t}" : "=r"(h2) : "f"(hi), "f"(lo));
  } else {
    asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h2) : "f"(hi), "f"(lo));
  }
  const float flo = __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu)));
  const float fhi = __half2float(__ushort_as_half((unsigned short)(h2 >> 16)));
  uint32_t out = (__float_as_uint(flo) >> 16) | (__float_as_uint(fhi) & 0xFFFF0000u);
  const uint32_t mag = idx2 & 0x7FFF7FFFu;
  out &= __vcmpne2(mag, 0u) | 0x7FFF7FFFu;          // -0 -> +0
  const uint32_t nan = __vcmpgtu2(mag, 0x7F807F80u);  // NaN -> nan_bits
  return (out & ~nan) | ((nan_bits * 0x10001u) & nan);
}

// bf16 indices of two quotients, packed: the exact patterns for a table
// (NaN -> 0xFFFF), the hardware pair conversion otherwise.
template <int K>
__device__ __forceinline__ uint32_t pair_index(float q0, float q1) {
  if (K == VQ_R_TABLE) return f2bf(q0) | (f2bf(q1) << 16);
  __nv_bfloat162 b = __floats2bfloat162_rn(q0, q1);
  return *reinterpret_cast<uint32_t*>(&b);
}

// E4M3 of a pair of bf16 quotients idx2 (lo | hi << 16) by the saturating
// round-to-nearest conversion: returns the two E4M3 bytes (lo byte = lo
// element) and sets code2 to their values as bf16 (every E4M3 value is a
// bf16).  This is hw_pair<K_HW_E4M3>'s result wherever neither quotient
// index is -0 or NaN (its two special cases), which callers establish first
// (plain_quotients).
__device__ __forceinline__ uint32_t e4m3_pair(uint32_t idx2, uint32_t& code2) {
  uint32_t b, h2;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %2, %3;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, t;\n\tcvt.u32.u16 %0, t;\n\t}"
      : "=r"(b), "=r"(h2)
      : "f"(__uint_as_float(idx2 & 0xFFFF0000u)), "f"(__uint_as_float(idx2 << 16)));
  __nv_bfloat162 c = __floats2bfloat162_rn(
      __half2float(__ushort_as_half((unsigned short)(h2 & 0xFFFFu))),
      __half2float(__ushort_as_half((unsigned short)(h2 >> 16))));
  code2 = *reinterpret_cast<uint32_t*>(&c);
  return b;
}

// Whether the quotients x * inv of a group of bf16 values (smallest
// magnitude mn, largest mx, as bf16 magnitude bits) avoid hw_pair's special
// cases: the power-of-two scale has exponent field E in [1, 253] (inv =
// 2^(127 - E) is exact and every quotient is the product), no value is NaN
// or zero, and no quotient is small enough to round to a bf16 zero
// (|q| <= 2^-134), so no quotient index is -0 or NaN.
__device__ __forceinline__ bool plain_quotients(uint32_t E, float inv, uint32_t mn, uint32_t mx) {
  return E >= 1u && E <= 253u && mx <= 0x7F80u && mn != 0u &&
         __uint_as_float(mn << 16) * inv > 0x1p-134f;
}

}  // namespace vq
