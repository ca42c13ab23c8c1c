"""Codebook (small ``qmap``) quantization as bfloat16-indexed tables.

The reference's ``encode`` (``src/voyager_compiler/ops/quantized.py:251-309``)
rounds its input to bfloat16 and searches the midpoints of an ascending
codebook; ``decode`` (``:312-337``) gathers ``codebook[index]``.  Both are
functions of the input's bfloat16 pattern, so each becomes a 65,536-entry
table built once per codebook on the host.  A 1-D codebook's table is
evaluated inside the quantize kernel like every other table.  A codebook
``[*counts, k]`` holds one table per region of the tensor (``_region_view``,
``:211-248``: ``counts[i]`` equal regions along axis ``i``); its tables are
kept in the output dtype and ``vq_codebook_lookup`` gathers each element
through its region's table -- after the quantize kernel has produced the
bfloat16-rounded quotient with the identity table.

The midpoints are computed in the codebook's dtype, as the reference's
``(codebook[..., :-1] + codebook[..., 1:]) / 2`` is: a bfloat16 codebook
rounds the sum to bfloat16.
"""

import ctypes
from typing import Optional

import numpy as np
import torch

from voyager_b200 import _lib
from voyager_b200._cache import TensorCache
from voyager_b200.tables import QMAP_SIZE, _bf16_bits_to_f32, _f32_to_bf16_bits

_enc = TensorCache()
_dec = TensorCache()
_ALL_BF16 = None


def _all_bf16() -> np.ndarray:
    global _ALL_BF16
    if _ALL_BF16 is None:
        _ALL_BF16 = _bf16_bits_to_f32(np.arange(QMAP_SIZE, dtype=np.uint32).astype(np.uint16))
    return _ALL_BF16


def _as_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy().astype(np.float32)


def _edges(codebook: torch.Tensor) -> np.ndarray:
    """Midpoints between consecutive entries, in the codebook's dtype."""
    cb = _as_f32(codebook)
    s = (cb[..., :-1] + cb[..., 1:]).astype(np.float32)
    if codebook.dtype == torch.bfloat16:
        s = _bf16_bits_to_f32(_f32_to_bf16_bits(s))
        return _bf16_bits_to_f32(_f32_to_bf16_bits((s / np.float32(2)).astype(np.float32)))
    return (s / np.float32(2)).astype(np.float32)


def _bf16_exact(cb: np.ndarray) -> bool:
    return bool(np.array_equal(_bf16_bits_to_f32(_f32_to_bf16_bits(cb)), cb))


def is_region_grid(codebook: torch.Tensor) -> bool:
    return codebook.dim() > 1


def region_counts(codebook: torch.Tensor, shape) -> list:
    """The region counts of ``codebook`` for a tensor of ``shape``, checked
    as ``_region_view`` checks them (a 1-D codebook: one region)."""
    if codebook.dim() == 1:
        return [1] * len(shape)
    counts = list(codebook.shape[:-1])
    if len(counts) != len(shape):
        raise ValueError(
            f"a {counts} region codebook tiles {len(counts)} axes, "
            f"but the tensor reaching it has {len(shape)}")
    if any(e % c for e, c in zip(shape, counts)):
        raise ValueError(
            f"a {counts} region codebook does not divide the {list(shape)} tensor reaching it")
    return counts


def encode_table(codebook: torch.Tensor, bounds, out_dtype: torch.dtype, device) -> torch.Tensor:
    """1-D codebook: table T with T[p] = encode(bf16 value p), the entry
    (or its index when ``bounds`` are given) of the interval the value falls
    in, as bf16.  Raises NotImplementedError where bf16 cannot hold the
    result (float32 output of entries that are not bf16 values): the caller
    then takes the per-region path, whose tables are float32."""
    if codebook.dim() != 1:
        raise NotImplementedError("a region-grid codebook has one table per region")
    key = (codebook._version, None if bounds is None else id(bounds), out_dtype, str(device))
    hit = _enc.get(codebook, key)
    if hit is not None:
        return hit
    cb = _as_f32(codebook)
    edges = _edges(codebook) if bounds is None else _as_f32(bounds)
    idx = np.searchsorted(edges, _all_bf16(), side="left")
    picked = idx.astype(np.float32) if bounds is not None else cb[idx]
    if out_dtype == torch.float32 and bounds is None and not _bf16_exact(cb):
        raise NotImplementedError("float32 codes of entries that are not bfloat16 values")
    table = torch.from_numpy(_f32_to_bf16_bits(picked).view(np.int16).copy()).view(
        torch.bfloat16).to(device)
    return _enc.put(codebook, key, table)


def decode_table(codebook: torch.Tensor, in_dtype: torch.dtype, device) -> torch.Tensor:
    """1-D codebook: table T with T[p] = codebook[int(p)] for the bf16
    patterns of the integers 0..k-1 (``decode``, ``quantized.py:312-337``)."""
    if codebook.dim() != 1:
        raise NotImplementedError("a region-grid codebook has one table per region")
    key = (codebook._version, in_dtype, str(device))
    hit = _dec.get(codebook, key)
    if hit is not None:
        return hit
    cb = _as_f32(codebook)
    if in_dtype == torch.float32 and not _bf16_exact(cb):
        raise NotImplementedError("float32 decode of entries that are not bfloat16 values")
    if cb.size > 256:
        raise NotImplementedError("codebooks of more than 256 entries")
    bits = np.zeros(QMAP_SIZE, dtype=np.uint16)
    ints = _f32_to_bf16_bits(np.arange(cb.size, dtype=np.float32))
    bits[ints] = _f32_to_bf16_bits(cb)
    table = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return _dec.put(codebook, key, table)


def _in_dtype(values: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    """float32 values as a tensor of ``dtype`` (bf16: round to nearest even)."""
    if dtype == torch.bfloat16:
        return torch.from_numpy(_f32_to_bf16_bits(values).view(np.int16).copy()).view(torch.bfloat16)
    if dtype == torch.float32:
        return torch.from_numpy(np.ascontiguousarray(values, dtype=np.float32))
    raise NotImplementedError(f"codebook outputs of dtype {dtype}")


def encode_tables(codebook: torch.Tensor, bounds: Optional[torch.Tensor],
                  out_dtype: torch.dtype, device) -> torch.Tensor:
    """[regions, 65536] tables of ``out_dtype``: per region, encode() of
    every bf16 value -- the entry, or its index when ``bounds`` are given."""
    key = ("regions", codebook._version, None if bounds is None else (id(bounds), bounds._version),
           out_dtype, str(device))
    hit = _enc.get(codebook, key)
    if hit is not None:
        return hit
    k = codebook.shape[-1]
    cb = _as_f32(codebook).reshape(-1, k)
    edges = (_edges(codebook) if bounds is None else _as_f32(bounds)).reshape(cb.shape[0], -1)
    x = _all_bf16()
    out = np.empty((cb.shape[0], QMAP_SIZE), dtype=np.float32)
    for r in range(cb.shape[0]):
        idx = np.searchsorted(edges[r], x, side="left")
        out[r] = idx.astype(np.float32) if bounds is not None else cb[r][idx]
    table = _in_dtype(out, out_dtype).to(device)
    return _enc.put(codebook, key, table)


def decode_tables(codebook: torch.Tensor, dtype: torch.dtype, device) -> torch.Tensor:
    """[regions, 65536] tables of ``dtype``: per region, the entry of each
    index 0..k-1 at that integer's bf16 pattern (0 elsewhere)."""
    key = ("regions", codebook._version, dtype, str(device))
    hit = _dec.get(codebook, key)
    if hit is not None:
        return hit
    k = codebook.shape[-1]
    if k > 256:
        raise NotImplementedError("codebooks of more than 256 entries")
    cb = _as_f32(codebook).reshape(-1, k)
    out = np.zeros((cb.shape[0], QMAP_SIZE), dtype=np.float32)
    ints = _f32_to_bf16_bits(np.arange(k, dtype=np.float32)).astype(np.int64)
    out[:, ints] = cb
    table = _in_dtype(out, dtype).to(device)
    return _dec.put(codebook, key, table)


def lookup(x: torch.Tensor, counts, tables: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """out[i] = tables[region(i)][bf16 pattern of x[i]] (``vq_codebook_lookup``)."""
    from voyager_b200 import ops as _ops

    x = x.contiguous()
    out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    if x.dim() == 0:
        x, o, cnt = x.reshape(1), out.reshape(1), [1]
    else:
        o, cnt = out, list(counts)
    c = (ctypes.c_int64 * len(cnt))(*cnt)
    st = _ops.lib().vq_codebook_lookup(_ops._ref(_ops._vt(x)), c, len(cnt), tables.data_ptr(),
                                       tables.shape[0], _ops._ref(_ops._vt(o)),
                                       _ops._stream(x.device))
    _lib.check(st, "codebook lookup")
    return out


def decode(x: torch.Tensor, codebook: torch.Tensor) -> torch.Tensor:
    """``decode`` (``quantized.py:312-337``): each index read back as its
    entry, in x's dtype (one table per region of a ``[*counts, k]``
    codebook)."""
    counts = region_counts(codebook, x.shape)
    return lookup(x, counts, decode_tables(codebook, x.dtype, x.device), x.dtype)
