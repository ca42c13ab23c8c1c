"""The premise of the NVFP4 quantize fast path (``k_qmx_nvfp4``), checked on
the host over every case it covers.

quantize_mx rounds each element's quotient x / s to bfloat16 before the
E2M1 table lookup (``quantized.py:854-881`` through ``quantize``: ``input /
scale`` in float32, rounded to the input's bf16).  The kernel multiplies by
the reciprocal instead: bf16(f32(x * f32(1 / s))).  For a bf16 x and an E4M3
scale s the two agree whenever the quotient is a normal float: the exact
quotient is M_x / M_s * 2^E with M_x < 256 and M_s < 16, so it is never a
bf16 rounding midpoint and stays at least 2^-8 / 15 (relative to its binade)
away from one, while both float32 results are within 2^-23 of it.  This test
checks that claim for all 65,536 bf16 patterns times all 126 positive finite
E4M3 scales."""

import numpy as np


def _e4m3_positive():
    vals = []
    for e in range(16):
        for m in range(8):
            if e == 15 and m == 7:
                continue  # NaN
            v = (m / 8.0) * 2.0**-6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
            if v > 0:
                vals.append(v)
    return np.array(vals, dtype=np.float32)


def _bf16_rn_bits(f):
    u = f.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32)


def test_reciprocal_quotient_rounds_like_division():
    scales = _e4m3_positive()
    assert len(scales) == 126
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    x = x[np.isfinite(x) & (x != 0)]
    checked = 0
    with np.errstate(over="ignore"):
        for s in scales:
            r = np.float32(np.float32(1.0) / s)
            q_mul = (x * r).astype(np.float32)
            q_div = (x / s).astype(np.float32)
            tiny = np.float32(2.0**-126)
            normal = (np.isfinite(q_mul) & np.isfinite(q_div) & (np.abs(q_mul) >= tiny)
                      & (np.abs(q_div) >= tiny))
            a, b = _bf16_rn_bits(q_mul[normal]), _bf16_rn_bits(q_div[normal])
            assert np.array_equal(a, b), f"scale {s}: {int((a != b).sum())} quotients differ"
            checked += int(normal.sum())
    assert checked > 8_000_000
