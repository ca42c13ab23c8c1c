"""Codebook (small ``qmap``) quantization as a bfloat16-indexed table.

The reference's ``encode`` (``src/voyager_compiler/ops/quantized.py:212-309``)
rounds its input to bfloat16 and searches the midpoints of an ascending 1-D
codebook; ``decode`` (``:312-337``) gathers ``codebook[index]``.  Both are
functions of the input's bfloat16 pattern only, so each becomes a 65,536-entry
table built once per codebook on the host and evaluated by the same kernels
as every other table.  Region-grid codebooks (``[*counts, k]``) are not
provided yet and raise.
"""

import numpy as np
import torch

from voyager_b200._cache import TensorCache
from voyager_b200.tables import QMAP_SIZE, _bf16_bits_to_f32, _f32_to_bf16_bits

_enc = TensorCache()
_dec = TensorCache()


def _as_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy().astype(np.float32)


def _check_1d(codebook: torch.Tensor):
    if codebook.dim() != 1:
        raise NotImplementedError(
            "quantized_ops on CUDA: region-grid codebooks ([*counts, k]) are not provided yet")


def encode_table(codebook: torch.Tensor, bounds, out_dtype: torch.dtype, device) -> torch.Tensor:
    """Table T with T[p] = encode(bf16 value p): the codebook entry (or its
    index when ``bounds`` are given) of the interval the value falls in."""
    _check_1d(codebook)
    key = (codebook._version, None if bounds is None else id(bounds), out_dtype, str(device))
    hit = _enc.get(codebook, key)
    if hit is not None:
        return hit
    cb = _as_f32(codebook)
    edges = ((cb[:-1] + cb[1:]) / np.float32(2)).astype(np.float32) if bounds is None \
        else _as_f32(bounds)
    x = _bf16_bits_to_f32(np.arange(QMAP_SIZE, dtype=np.uint32).astype(np.uint16))
    idx = np.searchsorted(edges, x, side="left")
    picked = idx.astype(np.float32) if bounds is not None else cb[idx]
    if out_dtype == torch.float32 and bounds is None:
        exact = _bf16_bits_to_f32(_f32_to_bf16_bits(cb))
        if not np.array_equal(exact, cb):
            raise NotImplementedError(
                "quantized_ops on CUDA: float32 codes from a codebook whose entries are not "
                "bfloat16 values are not provided yet")
    table = torch.from_numpy(_f32_to_bf16_bits(picked).view(np.int16).copy()).view(
        torch.bfloat16).to(device)
    return _enc.put(codebook, key, table)


def decode_table(codebook: torch.Tensor, in_dtype: torch.dtype, device) -> torch.Tensor:
    """Table T with T[p] = codebook[int(p)] for the bf16 patterns of the
    integers 0..k-1 (``decode``, ``quantized.py:312-337``)."""
    _check_1d(codebook)
    key = (codebook._version, in_dtype, str(device))
    hit = _dec.get(codebook, key)
    if hit is not None:
        return hit
    cb = _as_f32(codebook)
    if in_dtype == torch.float32:
        exact = _bf16_bits_to_f32(_f32_to_bf16_bits(cb))
        if not np.array_equal(exact, cb):
            raise NotImplementedError(
                "quantized_ops on CUDA: decoding float32 codes through a codebook whose "
                "entries are not bfloat16 values is not provided yet")
    if cb.size > 256:
        raise NotImplementedError("codebooks of more than 256 entries")
    bits = np.zeros(QMAP_SIZE, dtype=np.uint16)
    ints = _f32_to_bf16_bits(np.arange(cb.size, dtype=np.float32))
    bits[ints] = _f32_to_bf16_bits(cb)
    table = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return _dec.put(codebook, key, table)
