// Host-side pieces of the C ABI: status strings and the table classifier.
//
// vq_rounder_from_table() replaces the reference's per-element gather
// `qmap[bits & 0xFFFF]` (src/voyager_compiler/ops/quantized.py:174-203) by
// the cheapest rounder that reproduces the table on ALL 65,536 inputs.  Each
// candidate is verified entry by entry with the same __host__ __device__
// functions the kernels run (vq_numerics.cuh), so a rounder it returns is
// exact by construction; a table no candidate matches stays a table.
#include <math.h>
#include <string.h>

#include "vq_numerics.cuh"

using namespace vq;

namespace {

bool matches(const vq_rounder& r, const uint16_t* t) {
  // Cheap probes first, then every entry.
  static const uint16_t probes[] = {0x0000, 0x8000, 0x3F80, 0xBF80, 0x3F00, 0x4000,
                                    0x40C0, 0x43E0, 0x7F80, 0xFF80, 0x7FC0, 0xFFFF,
                                    0x3E80, 0x3FA0, 0x0001, 0x4780, 0x4F80};
  for (uint16_t p : probes)
    if (round_any(r, p, t) != t[p]) return false;
  for (uint32_t i = 0; i < 65536; ++i)
    if (round_any(r, i, t) != t[i]) return false;
  return true;
}

vq_rounder blank() {
  vq_rounder r;
  memset(&r, 0, sizeof(r));
  return r;
}

bool try_minifloat(const uint16_t* t, vq_rounder* out) {
  for (int ebits = 1; ebits <= 7; ++ebits) {
    for (int mbits = 0; mbits <= 7; ++mbits) {
      const int emax = ebits > 4 ? (1 << (ebits - 1)) - 1 : (1 << (ebits - 1));
      const double m1 = ldexp(2.0 - ldexp(1.0, -mbits), emax);
      const double m2 = ldexp(1.75, emax);  // the fp8_e4m3 (float8_e4m3fn) rule
      for (int variant = 0; variant < 2; ++variant) {
        const double mx = variant == 0 ? m1 : m2;
        if (variant == 1 && !(ebits == 4 && mbits == 3)) continue;
        for (int sgn = 1; sgn >= 0; --sgn) {
          vq_rounder r = blank();
          r.kind = VQ_R_MINIFLOAT;
          r.ebits = ebits;
          r.mbits = mbits;
          r.is_signed = sgn;
          r.min_exp = -(1 << (ebits - 1)) + 2;
          r.max_norm = (float)mx;
          r.nan_bits = t[0xFFFF];
          if ((double)r.max_norm != mx) continue;
          if (matches(r, t)) {
            // formats the tensor cores' conversion instructions produce
            // (round-to-nearest-even, saturating to the largest finite)
            if (sgn && ebits == 4 && mbits == 3 && mx == 448.0) r.hw = VQ_HW_E4M3;
            if (sgn && ebits == 5 && mbits == 2 && mx == 57344.0) r.hw = VQ_HW_E5M2;
            if (sgn && ebits == 2 && mbits == 1 && mx == 6.0) r.hw = VQ_HW_E2M1;
            *out = r;
            return true;
          }
        }
      }
    }
  }
  return false;
}

bool try_int(const uint16_t* t, vq_rounder* out) {
  for (int bits = 1; bits <= 16; ++bits) {
    for (int uns = 0; uns <= 1; ++uns) {
      vq_rounder r = blank();
      r.kind = VQ_R_INT;
      if (uns) {
        r.qmin = 0.0f;
        r.qmax = (float)((1 << bits) - 1);
      } else {
        r.qmin = -(float)(1 << (bits - 1));
        r.qmax = (float)((1 << (bits - 1)) - 1);
      }
      r.nan_bits = t[0xFFFF];
      if (matches(r, t)) {
        *out = r;
        return true;
      }
    }
  }
  return false;
}

bool try_posit(const uint16_t* t, vq_rounder* out) {
  for (int nbits = 3; nbits <= 16; ++nbits) {
    for (int es = 0; es <= 3; ++es) {
      vq_rounder r = blank();
      r.kind = VQ_R_POSIT;
      r.nbits = nbits;
      r.es = es;
      r.nan_bits = t[0xFFFF];
      if (matches(r, t)) {
        *out = r;
        return true;
      }
    }
  }
  return false;
}

uint32_t key_to_bits(uint32_t k) { return (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu); }

bool try_step(const uint16_t* t, vq_rounder* out) {
  vq_rounder r = blank();
  r.kind = VQ_R_STEP;
  int n = 0;
  uint16_t cur = t[key_to_bits(0)];
  r.step_vals[0] = cur;
  for (uint32_t k = 1; k < 65536; ++k) {
    uint16_t v = t[key_to_bits(k)];
    if (v != cur) {
      if (n == VQ_STEP_MAX) return false;
      r.step_keys[n] = (uint16_t)k;
      ++n;
      r.step_vals[n] = v;
      cur = v;
    }
  }
  r.nsteps = n;
  if (!matches(r, t)) return false;
  *out = r;
  return true;
}

}  // namespace

extern "C" {

const char* vq_status_string(int status) {
  switch (status) {
    case VQ_OK: return "ok";
    case VQ_ERR_INVALID: return "invalid argument";
    case VQ_ERR_UNSUPPORTED: return "unsupported dtype or layout";
    case VQ_ERR_ALIGNMENT: return "alignment requirement not met";
    case VQ_ERR_CUDA: return "CUDA runtime error";
    case VQ_ERR_SHAPE: return "shapes do not broadcast";
    case VQ_ERR_NULL: return "required pointer is NULL";
    case VQ_ERR_TIMEOUT: return "bounded device wait timed out";
    case VQ_ERR_TOO_LARGE: return "problem exceeds the fixed scratch area";
    default: return "unknown status";
  }
}

const char* vq_version(void) { return "voyager_b200 0.1 (sm_100a)"; }

int vq_rounder_from_table(const uint16_t* t, vq_rounder* out) {
  if (t == nullptr || out == nullptr) return VQ_ERR_NULL;
  bool ident = true;
  for (uint32_t i = 0; i < 65536 && ident; ++i) ident = t[i] == i;
  if (ident) {
    *out = blank();
    out->kind = VQ_R_IDENTITY;
    return VQ_OK;
  }
  if (try_minifloat(t, out)) return VQ_OK;
  if (try_int(t, out)) return VQ_OK;
  if (try_step(t, out)) return VQ_OK;
  if (try_posit(t, out)) return VQ_OK;
  *out = blank();
  out->kind = VQ_R_TABLE;
  return VQ_OK;
}

uint16_t vq_rounder_eval_host(const vq_rounder* r, uint16_t bits) {
  return (uint16_t)round_any(*r, bits, r->table);
}

uint32_t vq_pow2_scale_host(uint32_t amax_bits, int32_t dtype, int32_t fl2q) {
  if (dtype == VQ_BF16) return pow2_scale_bf16(amax_bits, fl2q);
  return pow2_scale_f32(amax_bits, fl2q);
}

}  // extern "C"
