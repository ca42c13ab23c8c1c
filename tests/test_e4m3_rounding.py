"""The E4M3 element rounding the CUDA kernels take from the hardware
conversion (cvt.rn.satfinite.e4m3x2.f32 of the bf16 quotient, then back to
bf16) against the oracle's E4M3 value table, exhaustively over the 65,536
bf16 index patterns.  An independent round-to-nearest-even onto the finite
E4M3 values, saturating at +-448, gives the table's entry for every index
except the two the kernels keep away from the conversion: -0 (the table
gives +0) and NaN (the table's NaN pattern).  The kernels' fast paths
(e4m3_pair where plain_quotients holds) rest on this; on the GPU
vq_rounder_check_hw checks the conversion itself against the table."""

import numpy as np

from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits, quantization_map


def _e4m3_magnitudes() -> np.ndarray:
    """The 127 finite non-negative E4M3 values in code order (code = index):
    exponent field e, mantissa m; e = 0 subnormal; S.1111.111 is NaN."""
    out = []
    for e in range(16):
        for m in range(8):
            if e == 15 and m == 7:
                continue
            out.append((m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7))
    return np.array(out, dtype=np.float64)


def _rne_saturating(x: np.ndarray) -> np.ndarray:
    """Round finite or infinite x to the nearest E4M3 value, ties to the even
    code, magnitudes above 448 to 448; the sign is kept (tiny negatives give
    -0)."""
    mags = _e4m3_magnitudes()
    a = np.minimum(np.abs(x), mags[-1])
    hi = np.clip(np.searchsorted(mags, a), 0, len(mags) - 1)
    lo = np.clip(hi - 1, 0, len(mags) - 1)
    dlo, dhi = a - mags[lo], mags[hi] - a
    pick = np.where(dlo < dhi, lo, np.where(dhi < dlo, hi, np.where(lo % 2 == 0, lo, hi)))
    pick = np.where(a == mags[hi], hi, pick)
    return np.copysign(mags[pick], x)


def test_e4m3_table_is_the_saturating_conversion():
    table = quantization_map("fp8_e4m3")
    idx = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = bf16_bits_to_f32(idx).astype(np.float64)
    mag = idx & 0x7FFF
    regular = (mag <= 0x7F80) & (idx != 0x8000)
    conv = f32_to_bf16_bits(_rne_saturating(x[regular]).astype(np.float32))
    assert np.array_equal(conv, table[regular])
    # the two special indices
    assert table[0x8000] == 0x0000
    nan_bits = table[0x7FC0]
    assert np.all(table[mag > 0x7F80] == nan_bits)


def test_plain_quotient_bound():
    """A quotient above 2^-134 has a nonzero bf16 index (the smallest bf16
    magnitude is 2^-133; 2^-134 ties to even, i.e. to zero), so with no zero
    or NaN input the fast path never meets a -0 or NaN index."""
    q = np.array([2.0 ** -134, np.nextafter(np.float32(2.0 ** -134), np.float32(1)),
                  2.0 ** -133], dtype=np.float32)
    bits = f32_to_bf16_bits(q)
    assert bits[0] == 0 and bits[1] != 0 and bits[2] == 1
