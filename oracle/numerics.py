"""bfloat16 arithmetic and value-table builders, restated in numpy.

Test infrastructure only (see ``oracle/__init__.py``).

The reference rounds every element through a 65,536-entry table indexed by
the bfloat16 bit pattern (``get_quantization_map``,
``src/voyager_compiler/quantization/fake_quantize.py:40-94``).  This module
rebuilds those tables from the same arithmetic:

* integers: ``clamp(round_half_even(v), qmin, qmax)`` (``fake_quantize.py:67-68``);
* minifloats: ``quantize_to_minifloat`` (``dtypes/fp8.py:69-133``) in float32
  after clamping to the format's largest normal (``fake_quantize.py:70-83``);
* posits: ``quantize_to_posit`` (``dtypes/posit.py:8-73``);
* lookup tables: NormalFloat levels (``dtypes/normal_float.py:4-62``),
  optionally snapped to an entry dtype's grid (``fake_quantize.py:88-92,97-113``).
"""

import math
import re
from typing import NamedTuple, Optional, Tuple

import numpy as np

BF16 = "bf16"
F32 = "fp32"

QMAP_SIZE = 1 << 16


# ---------------------------------------------------------------------------
# bfloat16 <-> float32
# ---------------------------------------------------------------------------
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bfloat16 bit patterns to float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(
        np.float32
    )


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16, nearest-even, as torch's CPU cast does.

    NaN becomes ``0xFFFF``: torch's vectorised float->bfloat16 conversion
    writes that pattern for every NaN (probed against
    ``vc/ops/quantized.py:183-184``'s ``input.to(torch.bfloat16)``).
    """
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0xFFFF), r).astype(np.uint16)


def round_to(x_f32: np.ndarray, dtype: str) -> np.ndarray:
    """Round a float32 intermediate to ``dtype``'s storage."""
    if dtype == BF16:
        return f32_to_bf16_bits(x_f32)
    return np.asarray(x_f32, dtype=np.float32)


def to_f32(a: np.ndarray) -> np.ndarray:
    """Widen a bf16-bits or float32 array to float32."""
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return bf16_bits_to_f32(a)
    return a.astype(np.float32, copy=False)


def dtype_of(a: np.ndarray) -> str:
    return BF16 if np.asarray(a).dtype == np.uint16 else F32


def all_bf16() -> np.ndarray:
    """All 65,536 bfloat16 bit patterns, in index order."""
    return np.arange(QMAP_SIZE, dtype=np.uint32).astype(np.uint16)


# ---------------------------------------------------------------------------
# Spec vocabulary (``src/voyager_compiler/quantization/qspec.py:70-206``)
# ---------------------------------------------------------------------------
class FloatFormat(NamedTuple):
    bits: int
    ebits: int
    mbits: int
    max_norm: float

    @property
    def signed(self) -> bool:
        return self.bits == self.ebits + self.mbits + 1


def int_range(dtype: str) -> Optional[Tuple[int, int]]:
    """``qspec.py:70-85``."""
    m = re.fullmatch(r"(u?)int(\d+)", dtype, re.IGNORECASE)
    if m is None:
        return None
    bits = int(m.group(2))
    if m.group(1):
        return 0, 2**bits - 1
    return -(2 ** (bits - 1)), 2 ** (bits - 1) - 1


def float_format(dtype: str) -> Optional[FloatFormat]:
    """``qspec.py:103-135``: fp8_e4m3 keeps its top exponent for finite
    values except the all-ones mantissa; wider exponents reserve it."""
    m = re.fullmatch(r"fp(\d+)_e(\d+)m(\d+)", dtype, re.IGNORECASE)
    if m is None:
        return None
    bits, ebits, mbits = map(int, m.groups())
    if bits not in (ebits + mbits, ebits + mbits + 1):
        raise ValueError(f"{dtype}: bad bit split")
    emax = 2 ** (ebits - 1) - 1 if ebits > 4 else 2 ** (ebits - 1)
    if dtype.lower() == "fp8_e4m3":
        max_norm = 2**emax * 1.75
    else:
        max_norm = 2**emax * (2 - 2.0**-mbits)
    return FloatFormat(bits, ebits, mbits, max_norm)


def posit_format(dtype: str) -> Optional[Tuple[int, int]]:
    """``qspec.py:138-150``."""
    m = re.fullmatch(r"posit(\d+)_(\d+)", dtype, re.IGNORECASE)
    if m is None:
        return None
    return int(m.group(1)), int(m.group(2))


def parse_codebook_dtype(dtype: str):
    """``qspec.py:175-206``: ``lut<I>[_to_<E>]``."""
    m = re.fullmatch(r"lut(\d+)(?:_to_(\w+))?", dtype)
    if m is None:
        return None
    index_bits, entry = m.groups()
    return int(index_bits), entry


def quant_min_max(dtype: str) -> Tuple[float, float]:
    """``qspec.py:153-172``."""
    if (b := int_range(dtype)) is not None:
        return b
    if (f := float_format(dtype)) is not None:
        return -f.max_norm, f.max_norm
    if (p := posit_format(dtype)) is not None:
        bits, es = p
        mx = (2 ** (2**es)) ** (bits - 2)
        return -mx, mx
    if (c := parse_codebook_dtype(dtype)) is not None:
        mx = 1 if c[1] is None else quant_min_max(c[1])[1]
        return -mx, mx
    raise ValueError(f"Unsupported dtype: {dtype}")


# ---------------------------------------------------------------------------
# Table builders
# ---------------------------------------------------------------------------
def _minifloat_f32(a: np.ndarray, bits: int, exp_bits: int, max_norm: float):
    """``dtypes/fp8.py:69-133`` with round="even", saturate_normals=True,
    allow_denorm=True, evaluated in float32."""
    a = a.astype(np.float32)
    with np.errstate(all="ignore"):
        if exp_bits != 0:
            pe = np.floor(
                np.log2(np.abs(a) + (a == 0).astype(np.float32))
            ).astype(np.float32)
            min_exp = -(2 ** (exp_bits - 1)) + 2
            pe = np.maximum(pe, np.float32(min_exp))  # NaN propagates
            p2 = np.power(np.float32(2), pe).astype(np.float32)
            out = a / p2 * np.float32(2 ** (bits - 2))
        else:
            p2 = None
            out = a * np.float32(2 ** (bits - 2))
        # _round_mantissa(..., "even"), fp8.py:45-49
        absA = np.abs(out)
        mask = (np.fmod(absA - np.float32(0.5), np.float32(2)) == 0).astype(
            np.float32
        )
        out = np.sign(out) * (np.floor(absA + np.float32(0.5)) - mask)
        out = out.astype(np.float32)
        if p2 is None:
            out = out / np.float32(2 ** (bits - 2))
        else:
            out = out / np.float32(2 ** (bits - 2)) * p2
        out = np.clip(out, -max_norm, max_norm).astype(np.float32)
        out = np.where(a == np.inf, np.float32(np.inf), out)
        out = np.where(a == -np.inf, np.float32(-np.inf), out)
    return out.astype(np.float32)


def _posit_bf16(bits16: np.ndarray, nbits: int, es: int) -> np.ndarray:
    """``dtypes/posit.py:8-73`` (round_to_even=True) on bfloat16 inputs."""
    x = bf16_bits_to_f32(bits16)
    raw = x.view(np.int32).astype(np.int64)
    scale = ((raw & 0x7F800000) >> 23) - 127
    fraction = raw & 0x7FFFFF
    r = scale >= 0
    max_scale = (nbits - 2) * (1 << es)
    regime_dominated = np.where(r, scale > max_scale, scale < -max_scale)
    run = np.where(r, 1 + (scale >> es), -(scale >> es))
    # The reference evaluates both branches in int32; only the taken one
    # matters, and the shift is bounded for it.
    safe_run = np.where(r, np.minimum(run, 60), 0)
    regime = np.where(r, (np.int64(1) << (safe_run + 1)) - 1, 0) ^ 1
    exponent = np.mod(scale, 1 << es)
    pt_bits = (regime << (23 + es)) | (exponent << 23) | fraction
    length = 2 + run + es + 23
    sh = np.clip(length - nbits, 0, 62)
    lb_mask = np.int64(1) << sh
    gb_mask = lb_mask >> 1
    sb_mask = gb_mask - 1
    lb = (pt_bits & lb_mask) != 0
    gb = (pt_bits & gb_mask) != 0
    sb = (pt_bits & sb_mask) != 0
    rb = ((lb & gb) | (gb & sb)) & ~regime_dominated
    ne_mask = np.clip(2 + run + es - nbits, 0, es)
    scale = scale & (np.int64(-1) << ne_mask)
    scale = np.clip(scale, -max_scale, max_scale)
    nf_mask = np.clip(length - nbits, 0, 23)
    fraction = fraction & (np.int64(-1) << nf_mask)
    out = ((scale + 127) << 23) | fraction
    out = np.where(rb, out + (np.int64(1) << (nf_mask + ne_mask)), out)
    out = (out & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    sign_in = np.sign(x)  # sign of the bf16 input (exact in f32)
    with np.errstate(all="ignore"):
        out = (out * sign_in).astype(np.float32)
        threshold = math.pow(2, math.floor(-(nbits - 1) * (1 << es) + 2 ** (es - 1)))
        out = np.where(np.abs(x) < threshold, np.float32(0), out)
        out = np.where(x == 0, np.float32(0), out)
        out = np.where(np.isfinite(x), out, np.float32(np.nan))
    # ``output.to(input.dtype)``: the float32 result rounds to bfloat16
    # (NaN -> 0xFFFF, like every float->bfloat16 cast here).
    return f32_to_bf16_bits(out)


def _torch_linspace_f32(start: float, end: float, steps: int) -> np.ndarray:
    """torch.linspace in float32: the first half counts up from ``start``,
    the second half down from ``end``."""
    step = np.float32((np.float32(end) - np.float32(start)) / np.float32(steps - 1))
    half = steps // 2
    out = np.empty(steps, dtype=np.float32)
    for i in range(steps):
        if i < half:
            out[i] = np.float32(start) + step * np.float32(i)
        else:
            out[i] = np.float32(end) - step * np.float32(steps - i - 1)
    return out


def create_normal_map(offset=0.9677083, use_extra_value=True, k=4) -> np.ndarray:
    """``dtypes/normal_float.py:4-29`` -> float32 levels, ascending."""
    from scipy.stats import norm

    n = 2 ** (k - 1)
    if use_extra_value:
        v1 = norm.ppf(_torch_linspace_f32(offset, 0.5, n + 1)[:-1]).tolist()
        v2 = [0]
        v3 = (-norm.ppf(_torch_linspace_f32(offset, 0.5, n)[:-1])).tolist()
    else:
        v1 = norm.ppf(_torch_linspace_f32(offset, 0.5, n)[:-1]).tolist()
        v2 = [0] * 2
        v3 = (-norm.ppf(_torch_linspace_f32(offset, 0.5, n)[:-1])).tolist()
    v = np.array(v1 + v2 + v3, dtype=np.float32)
    v = np.sort(v)
    v = (v / v.max()).astype(np.float32)
    return v


def _nf_levels_bf16(index_bits: int, entry: Optional[str]) -> np.ndarray:
    """Levels of ``lut<I>[_to_<E>]`` as bf16 bits (``normal_float.py:32-62``)."""
    values = create_normal_map(k=index_bits)
    if entry is not None:
        grid = entry_levels(entry)
        values = (values * grid.max()).astype(np.float32)
        values = grid[np.argmin(np.abs(values[:, None] - grid[None, :]), axis=-1)]
    return f32_to_bf16_bits(values.astype(np.float32))


def _nf_table(index_bits: int, entry: Optional[str]) -> np.ndarray:
    """``quantize_to_nf`` on every bf16 pattern, then ``levels[indices]``.

    The distances are bfloat16 arithmetic (``values - input`` rounds to
    bfloat16) and ties go to the first level.
    """
    levels = _nf_levels_bf16(index_bits, entry)
    lv = bf16_bits_to_f32(levels)
    x = bf16_bits_to_f32(all_bf16())
    with np.errstate(all="ignore"):
        xc = np.clip(x, lv.min(), lv.max())  # NaN stays NaN
        d = bf16_bits_to_f32(f32_to_bf16_bits(lv[None, :] - xc[:, None]))
        d = np.abs(d)
    idx = np.argmin(d, axis=-1)  # NaN rows pick the first NaN: index 0
    return levels[idx]


def entry_levels(dtype: str) -> np.ndarray:
    """``fake_quantize.py:97-113``: distinct finite values, symmetric, +0."""
    t = bf16_bits_to_f32(quantization_map(dtype))
    lv = np.unique(t[np.isfinite(t)])
    lv = lv[lv >= -lv.max()] + np.float32(0.0)
    return lv.astype(np.float32)


_TABLE_CACHE = {}


def quantization_map(dtype: Optional[str]) -> np.ndarray:
    """``get_quantization_map`` (``fake_quantize.py:40-94``) -> bf16 bits."""
    if dtype in _TABLE_CACHE:
        return _TABLE_CACHE[dtype]
    v16 = all_bf16()
    if dtype is None:
        out = v16.copy()
    elif (b := int_range(dtype)) is not None:
        x = bf16_bits_to_f32(v16)
        # torch.round on bfloat16 rounds half-to-even; the result is already
        # a bfloat16 value, and so is the clamp.
        r = f32_to_bf16_bits(np.round(x).astype(np.float32))
        r = bf16_bits_to_f32(r)
        with np.errstate(invalid="ignore"):
            r = np.clip(r, b[0], b[1]).astype(np.float32)
        out = f32_to_bf16_bits(r)
    elif (f := float_format(dtype)) is not None:
        x = bf16_bits_to_f32(v16)
        if not f.signed:
            x = np.abs(x)
        # clamp on bfloat16, then round in float32 (fake_quantize.py:73-83)
        x = bf16_bits_to_f32(
            f32_to_bf16_bits(np.clip(x, -f.max_norm, f.max_norm).astype(np.float32))
        )
        out = f32_to_bf16_bits(_minifloat_f32(x, f.mbits + 2, f.ebits, f.max_norm))
    elif (p := posit_format(dtype)) is not None:
        out = _posit_bf16(v16, *p)
    elif (c := parse_codebook_dtype(dtype)) is not None:
        out = _nf_table(*c)
    else:
        raise ValueError(f"Unsupported dtype: {dtype}")
    out = np.ascontiguousarray(out, dtype=np.uint16)
    _TABLE_CACHE[dtype] = out
    return out


def index_table(value_table_bits: np.ndarray) -> np.ndarray:
    """The int64 index table ``convert_pt2e`` swaps in for a codebook
    (``quantize_pt2e.py:697-716``): ``searchsorted(unique(table), table)``."""
    v = bf16_bits_to_f32(value_table_bits)
    u = np.unique(v)  # NaN sorts last, one copy per NaN in numpy >= 1.21
    return np.searchsorted(u, v).astype(np.int64)
