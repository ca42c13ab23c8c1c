// Element numerics shared by the CUDA kernels and the host-side classifier.
//
// Every function here is __host__ __device__ and uses only correctly rounded
// IEEE operations (explicit _rn intrinsics on the device, no contraction on
// the host), integer bit manipulation and exact power-of-two scaling, so the
// host build and the device build compute the same bits.  That is what lets
// vq_rounder_from_table() prove a rounder equal to a 65,536-entry table on
// the host and the kernels rely on it.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#include "voyager_b200.h"

#if defined(__CUDACC__)
#define VQ_HD __host__ __device__ __forceinline__
#else
#define VQ_HD inline
#endif

namespace vq {

// ---------------------------------------------------------------------------
// bit casts and correctly rounded float32 arithmetic
// ---------------------------------------------------------------------------
VQ_HD uint32_t f2u(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}
VQ_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}
VQ_HD float fmul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  volatile float r = a * b;
  return r;
#endif
}
VQ_HD float fadd_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  volatile float r = a + b;
  return r;
#endif
}
VQ_HD float fsub_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  volatile float r = a - b;
  return r;
#endif
}
VQ_HD float fdiv_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  volatile float r = a / b;
  return r;
#endif
}
// 1 / b rounded to nearest (the IEEE reciprocal: the same float as 1.0f / b).
VQ_HD float frcp_rn(float b) {
#if defined(__CUDA_ARCH__)
  return __frcp_rn(b);
#else
  volatile float r = 1.0f / b;
  return r;
#endif
}
VQ_HD bool is_nan_f(float f) { return (f2u(f) & 0x7FFFFFFFu) > 0x7F800000u; }
// 1 / q when q is a power of two whose reciprocal is a normal float (then
// x * (1 / q) is exactly the IEEE quotient x / q, both being the rounding
// of the same real number), else 0.
VQ_HD float pow2_inverse(float q) {
  const uint32_t b = f2u(q), e = (b >> 23) & 0xFFu;
  if ((b & 0x807FFFFFu) != 0 || e < 2u || e > 252u) return 0.0f;
  return u2f((254u - e) << 23);
}

// bf16 <-> float32.  float32 -> bf16 rounds to nearest even; every NaN becomes
// 0xFFFF, the pattern torch's vectorised CPU cast writes.
VQ_HD float bf2f(uint32_t b) { return u2f((b & 0xFFFFu) << 16); }
VQ_HD uint32_t f2bf(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0xFFFFu;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}
// Round a float32 to bf16 and widen it back.
VQ_HD float round_bf(float f) { return bf2f(f2bf(f)); }

// 2^k as a float32 for k in [-126, 127] (exact).
VQ_HD float pow2i(int k) { return u2f((uint32_t)(k + 127) << 23); }

VQ_HD int clz32(uint32_t x) {
#if defined(__CUDA_ARCH__)
  return __clz((int)x);
#else
  return x ? __builtin_clz(x) : 32;
#endif
}

VQ_HD float rint_f(float x) {
#if defined(__CUDA_ARCH__)
  return rintf(x);
#else
  return __builtin_rintf(x);
#endif
}

// ---------------------------------------------------------------------------
// Rounders: bf16 pattern -> table entry (bf16 pattern)
// ---------------------------------------------------------------------------

// Minifloat round-half-even with saturation, as the reference builds its fp
// tables: clamp to +-max_norm (abs first when unsigned), scale by the private
// exponent max(floor(log2|x|), min_exp), round the mantissa half-to-even,
// scale back (dtypes/fp8.py:69-133 via fake_quantize.py:70-83).
//
// Worked on the bf16 pattern: the magnitude is clamped as an integer
// (non-negative bf16 patterns order like their values), the rounding is one
// multiply by an exact power of two, rint, and the inverse multiply; the
// result has at most mbits+1 <= 8 significant bits, so it is exactly a bf16
// and its pattern is the top half of the float32.  A -0 input gives +0 and a
// negative input that rounds to zero gives -0, as the table has it.
VQ_HD uint32_t round_minifloat(const vq_rounder& r, uint32_t b) {
  uint32_t mag = b & 0x7FFFu;
  if (mag > 0x7F80u) return r.nan_bits;
  const uint32_t sign = r.is_signed ? (b & 0x8000u) : 0u;
  const uint32_t maxb = f2u(r.max_norm) >> 16;
  if (mag > maxb) mag = maxb;
  int E = (int)(mag >> 7);                 // biased exponent of |x|
  const int Emin = r.min_exp + 127;
  if (E < Emin) E = Emin;
  // |x| * 2^(mbits - e) with e = E - 127, rounded to an integer, scaled back
  const float up = u2f((uint32_t)(254 + r.mbits - E) << 23);
  const float dn = u2f((uint32_t)(E - r.mbits) << 23);
  const float v = rint_f(fmul_rn(u2f(mag << 16), up));
  const uint32_t y = f2u(fmul_rn(v, dn)) >> 16;
  return y | ((mag != 0) ? sign : 0u);
}

// clamp(round_half_even(x), qmin, qmax); a -0 result survives the clamp.
// Integers of magnitude <= 256 are exactly bf16 values, so for the usual
// ranges the result's pattern is the top half of the float32; wider ranges
// (int16 and up) round the clamp bound to bf16 as the table does.
VQ_HD uint32_t round_int(const vq_rounder& r, uint32_t b) {
  if ((b & 0x7FFFu) > 0x7F80u) return r.nan_bits;
  float y = rint_f(bf2f(b));  // exact in bf16: |x| < 256 rounds to <= 8 bits
  if (y < r.qmin) y = r.qmin;
  if (y > r.qmax) y = r.qmax;
  if (r.qmax <= 256.0f && r.qmin >= -256.0f) return f2u(y) >> 16;
  return f2bf(y);
}

// Posit<nbits, es> rounding of the float32 pattern (regime / exponent /
// fraction with last-guard-sticky rounding, values below the smallest posit
// round to zero, +-inf and NaN give NaN), restating dtypes/posit.py:8-73 with
// round_to_even=True.  Regime-dominated inputs (|scale| > max_scale) clamp to
// the extreme posit without rounding, as there.
VQ_HD uint32_t round_posit(const vq_rounder& r, uint32_t b) {
  float x = bf2f(b);
  uint32_t ux = f2u(x);
  if ((ux & 0x7FFFFFFFu) >= 0x7F800000u) return r.nan_bits;  // inf, NaN
  if ((ux & 0x7FFFFFFFu) == 0) return 0;                      // +-0 -> +0
  const int nbits = r.nbits, es = r.es;
  int64_t scale = (int64_t)((ux >> 23) & 0xFF) - 127;
  int64_t fraction = ux & 0x7FFFFF;
  const bool rpos = scale >= 0;
  const int64_t max_scale = (int64_t)(nbits - 2) * (1 << es);
  const bool dominated = rpos ? (scale > max_scale) : (scale < -max_scale);
  // floor division / modulo by 2^es of a possibly negative scale
  const int64_t sdiv = (scale >= 0) ? (scale >> es) : -((-scale + (1 << es) - 1) >> es);
  const int64_t run = rpos ? 1 + sdiv : -sdiv;
  const int64_t exponent = scale - sdiv * (1 << es);
  const int64_t len = 2 + run + es + 23;
  bool rb = false;
  if (!dominated) {
    const int64_t regime = (rpos ? (((int64_t)1 << (run + 1)) - 1) : 0) ^ 1;
    const int64_t pt = (regime << (23 + es)) | (exponent << 23) | fraction;
    int64_t sh = len - nbits;
    if (sh < 0) sh = 0;
    const int64_t lb_mask = (int64_t)1 << sh;
    const int64_t gb_mask = lb_mask >> 1;
    const int64_t sb_mask = gb_mask - 1;
    const bool lb = (pt & lb_mask) != 0, gb = (pt & gb_mask) != 0;
    const bool sb = (pt & sb_mask) != 0;
    rb = (lb && gb) || (gb && sb);
  }
  int64_t ne = 2 + run + es - nbits;
  if (ne < 0) ne = 0;
  if (ne > es) ne = es;
  scale -= scale & (((int64_t)1 << ne) - 1);  // clear the low ne bits
  if (scale < -max_scale) scale = -max_scale;
  if (scale > max_scale) scale = max_scale;
  int64_t nf = len - nbits;
  if (nf < 0) nf = 0;
  if (nf > 23) nf = 23;
  fraction -= fraction & (((int64_t)1 << nf) - 1);
  int64_t out = ((scale + 127) << 23) | fraction;
  if (rb) out += (int64_t)1 << (nf + ne);
  float y = u2f((uint32_t)(out & 0xFFFFFFFF));
  // Below 2^floor(-(nbits-1)*2^es + 2^(es-1)) the result is zero.
  const float ax = u2f(ux & 0x7FFFFFFFu);
  int tk = -(nbits - 1) * (1 << es);
  if (es >= 1) tk += 1 << (es - 1);  // es == 0: floor(tk + 0.5) == tk
  bool tiny;
  if (tk >= -126) {
    tiny = ax < pow2i(tk);
  } else {
    tiny = (tk >= -149) ? (f2u(ax) < (1u << (tk + 149))) : false;
  }
  if (tiny) return 0;
  if (ux >> 31) y = -y;
  return f2bf(y);
}

// Sortable 16-bit key: bf16 patterns in ascending numeric order (negative
// NaNs first, positive NaNs last).
VQ_HD uint32_t sort_key(uint32_t b) {
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

// Step function over the sortable key (binary search, <= 64 breakpoints).
VQ_HD uint32_t round_step_arrays(const uint16_t* keys, const uint16_t* vals, int n,
                                 uint32_t b) {
  uint32_t key = sort_key(b);
  int lo = 0;
#pragma unroll
  for (int step = 64; step >= 1; step >>= 1) {
    if (lo + step <= n && keys[lo + step - 1] <= key) lo += step;
  }
  return vals[lo];
}

// Any rounder, dispatching on its kind at run time (used once per block for
// scales, and by the host classifier).  TABLE reads `tbl` (device or host).
VQ_HD uint32_t round_any(const vq_rounder& r, uint32_t b, const uint16_t* tbl) {
  switch (r.kind) {
    case VQ_R_IDENTITY: return b & 0xFFFFu;
    case VQ_R_MINIFLOAT: return round_minifloat(r, b);
    case VQ_R_INT: return round_int(r, b);
    case VQ_R_POSIT: return round_posit(r, b);
    case VQ_R_STEP: return round_step_arrays(r.step_keys, r.step_vals, r.nsteps, b);
    default: return tbl[b & 0xFFFFu];
  }
}

// ---------------------------------------------------------------------------
// Division whose result is rounded to bfloat16 next
// ---------------------------------------------------------------------------
// quantize's index is bf16(fl32(x / s)).  With r = fl32(1/s) a normal number,
// q = fl32(x * r) lies within 3 float32 patterns of fl32(x / s) (relative
// error <= 2^-23 + 2^-48 in the normal range, <= 1 subnormal ulp below it),
// so both round to the same bf16 unless q's low 16 bits sit within 4 of the
// round-to-nearest-even tie at 0x8000.  Those few quotients take the IEEE
// division.  Overflow of x * r only happens where bf16(x / s) is infinite
// anyway.  The result is NOT fl32(x / s) in general: callers round it to bf16
// (or take its bf16 pattern) immediately.
struct Divisor {
  float s, r;
  int fast;
};

VQ_HD Divisor make_divisor(float s) {
  Divisor d;
  d.s = s;
  const uint32_t e = (f2u(s) >> 23) & 0xFF;  // |s| in [2^-126, 2^126)
  d.fast = (e >= 1u && e <= 252u) ? 1 : 0;    // 1/s then normal too
  d.r = d.fast ? frcp_rn(s) : 0.0f;
  return d;
}

// The IEEE division, kept out of line on the device so the rare slow path is
// a real branch rather than predicated into every element.
#if defined(__CUDACC__)
__host__ __device__ __noinline__ float div_slow(float x, float s);
#else
inline float div_slow(float x, float s) { return fdiv_rn(x, s); }
#endif

VQ_HD float div_to_bf16_domain(float x, const Divisor& d) {
  if (d.fast) {
    const float q = fmul_rn(x, d.r);
    if (((f2u(q) & 0xFFFFu) - 0x7FFCu) > 8u) return q;
  }
  return div_slow(x, d.s);
}

// ---------------------------------------------------------------------------
// Microscaling block scales (calculate_mx_qparam, quantized.py:787-851)
// ---------------------------------------------------------------------------

// floor(bf16(log2(a))) for a bf16 amax, a > 0 finite (mx_utils.py:48-53 with
// the log2 rounded to bfloat16 before the floor).  log2(a) = e + log2(1.m);
// it rounds up to e + 1 exactly when the 7-bit mantissa reaches a threshold
// that depends only on k = floor(log2 of the integer it rounds towards):
// ceil((2^(1 - 2^(k-8)) - 1) * 128) for k = 0..7, i.e.
// {128 (never), 127, 126, 123, 118, 107, 88, 54}.  Checked against the
// reference on all 65,536 bf16 inputs.
VQ_HD int floor_log2_bf16(uint32_t a_bits) {
  uint32_t E = (a_bits >> 7) & 0xFF;
  uint32_t M = a_bits & 0x7F;
  int e;
  uint32_t m;
  if (E == 0) {  // subnormal: a = M * 2^-133, M in [1, 127]
    int lz = 31 - clz32(M);  // floor(log2 M)
    e = lz - 133;
    m = (M << (7 - lz)) & 0x7F;
  } else {
    e = (int)E - 127;
    m = M;
  }
  int t = e >= 0 ? e : -(e + 1);  // integer |v| rounds towards
  // k = floor(log2 t); t == 0 never rounds up.
  uint32_t thr = 128;
  if (t > 0) {
    int k = 31 - clz32((uint32_t)t);
    const uint64_t pack = 0x36586B767B7E7F80ull;  // bytes k=0..7
    thr = (uint32_t)((pack >> (8 * k)) & 0xFF);
  }
  return e + (m >= thr ? 1 : 0);
}

// Power-of-two block scale of a bf16 block amax: 2^(floor(bf16(log2 amax'))
// - floor_log2_qmax) in bf16, where amax' = 2^-126 for a zero block, and
// where(scale > 0, scale, 1) (quantized.py:823-840,850).  Returns bf16 bits.
VQ_HD uint32_t pow2_scale_bf16(uint32_t amax_bits, int fl2q) {
  uint32_t a = amax_bits & 0x7FFFu;
  if (a > 0x7F80u) return 0x3F80u;   // NaN amax -> NaN scale -> 1.0
  if (a == 0x7F80u) return 0x7F80u;  // inf amax -> inf scale
  int f = (a == 0 ? -126 : floor_log2_bf16(a)) - fl2q;
  if (f > 127) return 0x7F80u;
  if (f >= -126) return (uint32_t)(f + 127) << 7;
  if (f >= -133) return 1u << (f + 133);  // bf16 subnormal
  return 0x3F80u;                          // underflows to 0 -> 1.0
}

// Same for a float32 block amax: the log2 is rounded to float32 before the
// floor.  log2 is evaluated in double precision and rounded once to float32
// (the correctly rounded value the reference's float32 log2 returns on the
// inputs where the floor is decided).  Returns float32 bits.
VQ_HD uint32_t pow2_scale_f32(uint32_t amax_bits, int fl2q) {
  uint32_t a = amax_bits & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return 0x3F800000u;
  if (a == 0x7F800000u) return 0x7F800000u;
  int fl;
  if (a == 0) {
    fl = -126;
  } else {
    double lg = log2((double)u2f(a));
    float lgf = (float)lg;
    fl = (int)floorf(lgf);
  }
  int f = fl - fl2q;
  if (f > 127) return 0x7F800000u;
  if (f >= -126) return (uint32_t)(f + 127) << 23;
  if (f >= -149) return 1u << (f + 149);
  return 0x3F800000u;
}

// Block scale from a block amax by division (quantized.py:842-848,850):
// amax / quant_max in the input dtype, optionally through scale_qmap, then
// where(scale > 0, scale, 1).  `is_bf16` selects the dtype; returns the
// scale as a float32 value (exact in the dtype).
VQ_HD float div_scale(float amax, float qmax, bool is_bf16, const vq_rounder* sq,
                      const uint16_t* sq_table) {
  float s = fdiv_rn(amax, qmax);
  if (is_bf16) s = round_bf(s);
  if (sq != nullptr) s = bf2f(round_any(*sq, f2bf(s), sq_table));
  return (s > 0.0f) ? s : 1.0f;
}

}  // namespace vq
