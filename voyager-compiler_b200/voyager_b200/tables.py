"""Value tables and their rounders.

The reference quantizes through a 65,536-entry table indexed by the bfloat16
bit pattern (``get_quantization_map``,
``src/voyager_compiler/quantization/fake_quantize.py:40-94``).  On the GPU
the kernels evaluate a ``vq_rounder`` instead: the C library classifies a
table (once, on the host) into the analytic form that reproduces all of its
65,536 entries, or keeps it as a table staged in shared memory.

``rounder_for(qmap)`` returns that rounder for a table tensor, cached per
tensor object and version.  The first sight of a table on the GPU copies it
to the host once (a synchronisation); tables are constants shared by every
node that uses them, so warm-up covers this before any CUDA-graph capture.

``get_quantization_map(dtype, device)`` builds the tables for the spec
dtypes (``int<N>``, ``uint<N>``, ``fp<B>_e<X>m<Y>``, ``posit<N>_<es>``,
``lut<I>[_to_<E>]``) for callers that do not have the reference installed.
"""

import ctypes
import functools
import math
import re
import threading
from typing import NamedTuple, Optional, Tuple

import numpy as np
import torch

from voyager_b200 import _lib
from voyager_b200._cache import TensorCache

QMAP_SIZE = 1 << 16

# ---------------------------------------------------------------------------
# spec vocabulary (src/voyager_compiler/quantization/qspec.py:70-206)
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
    m = re.fullmatch(r"(u?)int(\d+)", dtype, re.IGNORECASE)
    if m is None:
        return None
    b = int(m.group(2))
    return (0, 2**b - 1) if m.group(1) else (-(2 ** (b - 1)), 2 ** (b - 1) - 1)


def float_format(dtype: str) -> Optional[FloatFormat]:
    m = re.fullmatch(r"fp(\d+)_e(\d+)m(\d+)", dtype, re.IGNORECASE)
    if m is None:
        return None
    bits, ebits, mbits = map(int, m.groups())
    if bits not in (ebits + mbits, ebits + mbits + 1):
        raise ValueError(f"{dtype}: {bits} bits is neither {ebits}+{mbits} nor that plus a sign bit")
    emax = 2 ** (ebits - 1) - 1 if ebits > 4 else 2 ** (ebits - 1)
    mx = 2**emax * 1.75 if dtype.lower() == "fp8_e4m3" else 2**emax * (2 - 2.0**-mbits)
    return FloatFormat(bits, ebits, mbits, mx)


def posit_format(dtype: str) -> Optional[Tuple[int, int]]:
    m = re.fullmatch(r"posit(\d+)_(\d+)", dtype, re.IGNORECASE)
    return None if m is None else (int(m.group(1)), int(m.group(2)))


def parse_codebook_dtype(dtype: str):
    m = re.fullmatch(r"lut(\d+)(?:_to_(\w+))?", dtype)
    if m is None:
        return None
    return int(m.group(1)), m.group(2)


def quant_min_max(dtype: str) -> Tuple[float, float]:
    """``qspec.py:153-172``."""
    if (b := int_range(dtype)) is not None:
        return float(b[0]), float(b[1])
    if (f := float_format(dtype)) is not None:
        return -f.max_norm, f.max_norm
    if (p := posit_format(dtype)) is not None:
        mx = (2 ** (2 ** p[1])) ** (p[0] - 2)
        return -float(mx), float(mx)
    if (c := parse_codebook_dtype(dtype)) is not None:
        mx = 1.0 if c[1] is None else quant_min_max(c[1])[1]
        return -mx, mx
    raise ValueError(f"Unsupported dtype: {dtype}")


# ---------------------------------------------------------------------------
# bf16 helpers (numpy)
# ---------------------------------------------------------------------------
def _f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0xFFFF), r).astype(np.uint16)


def _bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def table_to_bf16_bits(q: torch.Tensor) -> np.ndarray:
    """A table tensor's entries as bfloat16 patterns on the host, cast the
    way the reference's ``vmap`` assigns them into a bfloat16 tensor
    (``quantized.py:199-201``)."""
    q = q.detach()
    if q.dtype == torch.bfloat16:
        return q.contiguous().cpu().view(torch.int16).numpy().view(np.uint16).copy()
    if q.dtype in (torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8):
        return _f32_to_bf16_bits(q.cpu().numpy().astype(np.float64).astype(np.float32))
    return _f32_to_bf16_bits(q.cpu().float().numpy())


# ---------------------------------------------------------------------------
# rounder cache
# ---------------------------------------------------------------------------
class Rounder:
    """A classified table: the C struct plus the device table it may read."""

    __slots__ = ("c", "device_table", "host_table", "coded", "__weakref__")

    def __init__(self, c: "_lib.VqRounder", device_table: Optional[torch.Tensor], host_table,
                 coded=None):
        self.c = c
        self.device_table = device_table
        self.host_table = host_table
        self.coded = coded  # (byte codes, palette) on the device, or None

    @property
    def kind(self) -> str:
        return _lib.KIND_NAMES[self.c.kind]

    def ref(self):
        return ctypes.byref(self.c)


_lock = threading.Lock()
_cache = TensorCache()
_content_cache = {}


def classify_host_table(bits: np.ndarray) -> "_lib.VqRounder":
    lib = _lib.load()
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    assert bits.size == QMAP_SIZE
    r = _lib.VqRounder()
    _lib.check(lib.vq_rounder_from_table(bits.ctypes.data, ctypes.byref(r)), "classify table")
    return r


def _verify_hw(c: "_lib.VqRounder", device) -> None:
    """Keep the hardware-conversion form of a minifloat rounder only if it
    reproduces all 65,536 table entries on this device (one launch, one
    synchronisation, once per table)."""
    mism = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    st = _lib.load().vq_rounder_check_hw(ctypes.byref(c), mism.data_ptr(), stream)
    if st != 0 or int(mism.item()) != 0:
        c.hw = 0


def _byte_coded(c: "_lib.VqRounder", bits: np.ndarray, device):
    """For a rounder the kernels evaluate as a table (TABLE, POSIT, STEP)
    whose entries take at most 256 distinct patterns: byte codes into a
    palette, on the device (64.5 KB of shared memory instead of 128 KB)."""
    if c.kind not in (_lib.VQ_R_TABLE, _lib.VQ_R_POSIT, _lib.VQ_R_STEP):
        return None
    if torch.device(device).type != "cuda":
        return None
    uniq, inv = np.unique(bits, return_inverse=True)
    if uniq.size > 256:
        return None
    pal = np.zeros(256, dtype=np.uint16)
    pal[: uniq.size] = uniq
    t8 = torch.from_numpy(inv.astype(np.uint8).reshape(-1)).to(device)
    p16 = torch.from_numpy(pal.view(np.int16).copy()).to(device)
    c.table8 = t8.data_ptr()
    c.palette = p16.data_ptr()
    return t8, p16


def rounder_for(qmap: torch.Tensor, device: torch.device) -> Rounder:
    """The rounder of a 65,536-entry table, with its bf16 device copy on
    ``device``.  Cached per tensor object (and its version counter) and per
    table content."""
    if qmap.numel() != QMAP_SIZE or qmap.dim() != 1:
        raise ValueError("a lookup table has 65,536 entries, one per bfloat16 pattern")
    key = (qmap._version, str(device))
    hit = _cache.get(qmap, key)
    if hit is not None:
        return hit
    if qmap.is_cuda and torch.cuda.is_current_stream_capturing():
        raise RuntimeError(
            "quantized_ops: a lookup table seen for the first time during CUDA-graph "
            "capture; run the graph once before capturing so its tables are classified")
    bits = table_to_bf16_bits(qmap)
    ck = (bits.tobytes(), str(device))
    with _lock:
        rd = _content_cache.get(ck)
    if rd is None:
        c = classify_host_table(bits)
        dev = torch.from_numpy(bits.view(np.int16).copy()).to(device).view(torch.bfloat16)
        c.table = dev.data_ptr()
        if c.hw and torch.device(device).type == "cuda":
            _verify_hw(c, device)
        coded = _byte_coded(c, bits, device)
        rd = Rounder(c, dev, bits, coded)
        with _lock:
            _content_cache[ck] = rd
    return _cache.put(qmap, key, rd)


# ---------------------------------------------------------------------------
# table builders (get_quantization_map for callers without the reference)
# ---------------------------------------------------------------------------
def _analytic_table(r: "_lib.VqRounder") -> np.ndarray:
    lib = _lib.load()
    ev = lib.vq_rounder_eval_host
    out = np.empty(QMAP_SIZE, dtype=np.uint16)
    ref = ctypes.byref(r)
    for i in range(QMAP_SIZE):
        out[i] = ev(ref, i)
    return out


def _torch_linspace_f32(start, end, steps):
    step = np.float32((np.float32(end) - np.float32(start)) / np.float32(steps - 1))
    half = steps // 2
    return np.array([np.float32(start) + step * np.float32(i) if i < half
                     else np.float32(end) - step * np.float32(steps - i - 1)
                     for i in range(steps)], dtype=np.float32)


def _normal_levels(k: int) -> np.ndarray:
    """NormalFloat levels (``dtypes/normal_float.py:4-29``), float32."""
    from scipy.stats import norm

    n = 2 ** (k - 1)
    off = 0.9677083
    v1 = norm.ppf(_torch_linspace_f32(off, 0.5, n + 1)[:-1]).tolist()
    v3 = (-norm.ppf(_torch_linspace_f32(off, 0.5, n)[:-1])).tolist()
    v = np.sort(np.array(v1 + [0] + v3, dtype=np.float32))
    return (v / v.max()).astype(np.float32)


def _entry_levels(dtype: str) -> np.ndarray:
    t = _bf16_bits_to_f32(_table_bits(dtype))
    lv = np.unique(t[np.isfinite(t)])
    return (lv[lv >= -lv.max()] + np.float32(0)).astype(np.float32)


@functools.lru_cache(maxsize=None)
def _table_bits(dtype: Optional[str]) -> np.ndarray:
    if dtype is None:
        return np.arange(QMAP_SIZE, dtype=np.uint32).astype(np.uint16)
    r = _lib.VqRounder()
    if (b := int_range(dtype)) is not None:
        r.kind, r.qmin, r.qmax, r.nan_bits = _lib.VQ_R_INT, b[0], b[1], 0xFFFF
        return _analytic_table(r)
    if (f := float_format(dtype)) is not None:
        r.kind = _lib.VQ_R_MINIFLOAT
        r.ebits, r.mbits, r.is_signed = f.ebits, f.mbits, int(f.signed)
        r.min_exp = -(2 ** (f.ebits - 1)) + 2
        r.max_norm, r.nan_bits = f.max_norm, 0xFFFF
        if f.ebits > 7:
            raise ValueError(f"{dtype}: exponent field wider than 7 bits is not provided")
        return _analytic_table(r)
    if (p := posit_format(dtype)) is not None:
        r.kind, r.nbits, r.es, r.nan_bits = _lib.VQ_R_POSIT, p[0], p[1], 0xFFFF
        return _analytic_table(r)
    if (c := parse_codebook_dtype(dtype)) is not None:
        k, entry = c
        lv = _normal_levels(k)
        if entry is not None:
            grid = _entry_levels(entry)
            lv = (lv * grid.max()).astype(np.float32)
            lv = grid[np.argmin(np.abs(lv[:, None] - grid[None, :]), axis=-1)]
        lvb = _f32_to_bf16_bits(lv)
        lvf = _bf16_bits_to_f32(lvb)
        x = _bf16_bits_to_f32(np.arange(QMAP_SIZE, dtype=np.uint32).astype(np.uint16))
        with np.errstate(invalid="ignore"):
            xc = np.clip(x, lvf.min(), lvf.max())
            d = np.abs(_bf16_bits_to_f32(_f32_to_bf16_bits(lvf[None, :] - xc[:, None])))
        return lvb[np.argmin(d, axis=-1)]
    raise ValueError(f"Unsupported dtype: {dtype}")


@functools.lru_cache(maxsize=None)
def get_quantization_map(dtype: Optional[str], device=None) -> torch.Tensor:
    """A 65,536-entry bfloat16 table (``fake_quantize.py:40-94``); shared,
    must not be modified in place."""
    bits = _table_bits(dtype)
    t = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    return t.to(device) if device is not None else t


def index_table(values_table: torch.Tensor) -> torch.Tensor:
    """The int64 index table ``convert_pt2e`` swaps in for a codebook
    (``quantize_pt2e.py:697-716``)."""
    return torch.searchsorted(torch.unique(values_table), values_table).to(torch.int64)


def floor_log2(quant_max: float) -> int:
    """``math.floor(math.log2(quant_max))`` as ``calculate_mx_qparam`` takes it
    (``quantized.py:825``)."""
    return math.floor(math.log2(quant_max))
