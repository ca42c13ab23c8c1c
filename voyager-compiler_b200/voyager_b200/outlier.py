"""The outlier CSR side-stream on CUDA (``src/voyager_compiler/ops/quantized.py:958-1327``).

``filter_outlier`` splits a tensor into its inliers and a CSR of the
elements with ``|x| > threshold``; ``quantize_mx_outlier`` quantizes the
inliers with ``quantize_mx``; ``spmm_csr`` multiplies such a CSR with a
(decoded, scaled) dense operand; ``slice_csr_tensor`` cuts a CSR by rows or
by a column window.  ``linear_mx`` / ``matmul_mx`` add ``spmm_csr`` of their
``A_data`` / ``A_indices`` / ``A_indptr`` to the dense product
(``voyager_b200.gemm``).

Kernels (``csrc/vq_sparse.cu``): the filter counts outliers per tile, scans
the counts and scatters the CSR in row-major order (three launches, no waits
between CTAs); ``quantize_mx_outlier`` along the
last dim masks the outliers inside ``quantize_mx``'s kernel instead of
writing and re-reading the inliers; ``spmm_csr`` is a gather of B rows
accumulated with float32 fused multiply-adds in CSR order (what the CPU
sparse mm computes), so its products match the reference bit for bit.
"""

import math
from typing import Optional

import torch

from voyager_b200 import _lib
from voyager_b200 import ops as _ops
from voyager_b200._cache import TensorCache
from voyager_b200.tables import QMAP_SIZE, floor_log2, rounder_for

_tcache = TensorCache()
_I32 = (-(1 << 31), (1 << 31) - 1)


def _max_nnz(mat_shape, max_pct: float) -> int:
    """``int(math.prod(mat_shape) * max_pct)``, as the reference sizes the
    stream (quantized.py:1016)."""
    return int(math.prod(mat_shape) * max_pct)


def _filter(input: torch.Tensor, threshold, max_pct: float, offset: int, want_inliers: bool):
    _ops._check_cuda(input, "filter_outlier")
    if threshold is None:
        raise TypeError("'>' not supported between instances of 'Tensor' and 'NoneType'")
    if input.dim() < 2:
        raise RuntimeError("filter_outlier: the input must have at least 2 dims (a CSR matrix)")
    if not _I32[0] <= int(offset) <= _I32[1]:
        raise ValueError(f"indptr_offset {offset} does not fit the int32 row pointers")
    x = input.contiguous()
    dev = x.device
    batch = tuple(x.shape[:-2])
    R, C = x.shape[-2], x.shape[-1]
    max_nnz = _max_nnz(x.shape[-2:], max_pct)
    if max_nnz < 0:
        raise ValueError(f"max_pct {max_pct} gives a negative stream size")
    if math.prod(batch) == 0:
        raise RuntimeError("stack expects a non-empty TensorList")
    data = torch.empty((*batch, max_nnz), dtype=x.dtype, device=dev)
    indices = torch.empty((*batch, max_nnz), dtype=torch.int32, device=dev)
    indptr = torch.empty((*batch, R + 1), dtype=torch.int32, device=dev)
    inliers = torch.empty_like(x) if want_inliers else None
    L = _ops.lib()
    vt = _ops._vt(x)
    nbytes = int(L.vq_filter_outlier_workspace_bytes(_ops._ref(vt)))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    st = L.vq_filter_outlier(_ops._ref(vt), float(threshold), max_nnz, int(offset),
                             data.data_ptr() if data.numel() else None,
                             indices.data_ptr() if indices.numel() else None, indptr.data_ptr(),
                             inliers.data_ptr() if inliers is not None and inliers.numel() else None,
                             ws.data_ptr(), ws.numel(), None, _ops._stream(dev))
    _lib.check(st, "quantized_ops::filter_outlier")
    return data, indices, indptr, inliers


def filter_outlier(input: torch.Tensor, threshold: float, max_pct: float = 0.01):
    """``quantized.py:995-1045`` -> ``(data, indices, indptr, inliers)``."""
    return _filter(input, threshold, max_pct, 0, True)


def _masked_quantize_mx(x, qmap, ax, block_size, quant_max, pow2, scale_qmap, threshold):
    """quantize_mx of ``x`` with its outliers quantized as +0, in one pass;
    None when the fused kernel does not take this layout."""
    if not (qmap.numel() == QMAP_SIZE and qmap.dim() == 1) or ax != [x.dim() - 1]:
        return None
    if x.numel() == 0:
        return None
    dev = x.device
    scale = torch.empty(_ops._blocked_shape(x.shape, ax, block_size), dtype=x.dtype, device=dev)
    codes = torch.empty_like(x)
    rd = rounder_for(qmap, dev)
    sq = rounder_for(scale_qmap, dev) if scale_qmap is not None else None
    fl2q = floor_log2(quant_max) if pow2 else 0
    C = x.shape[-1]
    mxfp8 = (block_size == 32 and pow2 and scale_qmap is None and x.dtype == torch.bfloat16
             and rd.c.kind == _lib.VQ_R_MINIFLOAT and rd.c.hw == 1)
    packed = packed_sf = None
    if mxfp8 and C % 128 == 0:
        R = x.numel() // C
        rt = (R + 127) // 128
        packed = torch.empty(rt * 128 * C, dtype=torch.uint8, device=dev)
        packed_sf = torch.empty((C // 128) * rt * 512, dtype=torch.uint8, device=dev)
    st = _ops.lib().vq_quantize_mx_masked(
        _ops._ref(_ops._vt(x)), rd.ref(), int(block_size), float(quant_max), int(bool(pow2)),
        fl2q, sq.ref() if sq else None, float(threshold), _ops._ref(_ops._vt(scale)),
        _ops._ref(_ops._vt(codes)), None if packed is None else packed.data_ptr(),
        None if packed_sf is None else packed_sf.data_ptr(), _ops._stream(dev))
    if st == 2:  # VQ_ERR_UNSUPPORTED
        return None
    _lib.check(st, "quantized_ops::quantize_mx_outlier")
    if mxfp8:
        from voyager_b200 import mxgemm

        mxgemm.vouch(codes, scale, None if packed is None else (packed, packed_sf))
    return scale, codes


def quantize_mx_outlier(input: torch.Tensor, qmap: torch.Tensor, axes, block_size: int,
                        quant_max: float, force_scale_power_of_two: bool = False,
                        scale_qmap: Optional[torch.Tensor] = None,
                        output_code: Optional[torch.Tensor] = None,
                        threshold: Optional[float] = None, max_pct: float = 0.01,
                        indptr_offset: int = 0):
    """``quantized.py:1078-1130`` -> ``(data, indices, indptr, scale, inliers)``
    where ``inliers`` are quantize_mx's codes of the inliers."""
    assert block_size > 0
    _ops._check_cuda(input, "quantize_mx_outlier")
    if threshold is None:
        raise TypeError("'>' not supported between instances of 'Tensor' and 'NoneType'")
    x = input.contiguous()
    ax = _ops._norm_axes(axes, x.dim())
    fused = None
    if x.dim() >= 2:
        fused = _masked_quantize_mx(x, qmap, ax, block_size, quant_max,
                                    force_scale_power_of_two, scale_qmap, threshold)
    if fused is not None:
        data, indices, indptr, _ = _filter(x, threshold, max_pct, indptr_offset, False)
        scale, codes = fused
        return data, indices, indptr, scale, codes
    data, indices, indptr, inliers = _filter(x, threshold, max_pct, indptr_offset, True)
    scale, codes = _ops.quantize_mx(inliers, qmap, axes, block_size, quant_max,
                                    force_scale_power_of_two, scale_qmap, output_code)
    return data, indices, indptr, scale, codes


def _transposed(b: torch.Tensor) -> torch.Tensor:
    """[..., R, C] -> contiguous [..., C, R] by this library's kernel."""
    out = torch.empty((*b.shape[:-2], b.shape[-1], b.shape[-2]), dtype=b.dtype, device=b.device)
    st = _ops.lib().vq_transpose(_ops._ref(_ops._vt(b)), _ops._ref(_ops._vt(out)),
                                 _ops._stream(b.device))
    _lib.check(st, "transpose")
    return out


def _operand(B, B_scale, B_code, block_size, weight_layout, cache: bool):
    """B decoded and scaled (``_dequantize_mx``), laid out [.., K, N]."""
    from voyager_b200.gemm import _weight_dequant, dequantize_mx

    if not cache:
        b = dequantize_mx(B, B_scale, B_code, block_size)
        b = b.contiguous()
        return _transposed(b) if weight_layout == "kc" else b
    key = ("spmm", weight_layout, B._version,
           None if B_scale is None else (id(B_scale), B_scale._version),
           None if B_code is None else (id(B_code), B_code._version), block_size)
    hit = _tcache.get(B, key)
    if hit is not None:
        return hit
    b = _weight_dequant(B, B_scale, B_code, block_size).contiguous()
    b = _transposed(b) if weight_layout == "kc" else b
    return _tcache.put(B, key, b)


def spmm_csr(data: torch.Tensor, indices: torch.Tensor, indptr: torch.Tensor, B: torch.Tensor,
             B_scale: Optional[torch.Tensor] = None, B_code: Optional[torch.Tensor] = None,
             block_size: Optional[int] = None, weight_layout: str = "kc",
             _cache_operand: Optional[bool] = None) -> torch.Tensor:
    """``quantized.py:1245-1311``: the CSR (batched over indptr's leading
    dims) times B, B decoded through ``B_code`` and scaled by ``B_scale``
    first; a KC-stored B ([out, contraction]) is transposed."""
    assert weight_layout in ("kc", "ck"), weight_layout
    _ops._check_cuda(B, "spmm_csr")
    dev = B.device
    # a KC-stored 2-D B is a linear weight: its decoded, transposed copy is
    # kept (until B is freed or changed); other operands convert per call
    cache = (_cache_operand if _cache_operand is not None
             else (B.dim() == 2 and weight_layout == "kc"))
    b = _operand(B, B_scale, B_code, block_size, weight_layout, cache)
    batch = tuple(indptr.shape[:-1])
    nb = math.prod(batch)
    X = indptr.shape[-1] - 1
    if nb == 0:
        raise RuntimeError("stack expects a non-empty TensorList")
    ip = _ops._on(indptr, dev).reshape(-1, X + 1)
    ix = _ops._on(indices, dev).reshape(-1, indices.shape[-1])
    dt = _ops._on(data, dev).reshape(-1, data.shape[-1])
    if ip.dtype != torch.int32:
        ip = ip.to(torch.int32)
    if ix.dtype != torch.int32:
        ix = ix.to(torch.int32)
    if b.dim() > 2:
        b = b.reshape(nb, b.shape[-2], b.shape[-1])
    N = b.shape[-1]
    out = torch.empty((nb, X, N), dtype=b.dtype, device=dev)
    ws = torch.empty(nb * (X + 1), dtype=torch.int32, device=dev)
    st = _ops.lib().vq_spmm_csr(_ops._ref(_ops._vt(dt)), ix.data_ptr() if ix.numel() else None,
                                ip.data_ptr(), X, _ops._ref(_ops._vt(b)),
                                _ops._ref(_ops._vt(out)), ws.data_ptr(), _ops._stream(dev))
    _lib.check(st, "quantized_ops::spmm_csr")
    return out.reshape(*batch, X, N)


def slice_csr_tensor(data: torch.Tensor, indices: torch.Tensor, indptr: torch.Tensor,
                     dim: int = 0, start: Optional[int] = None, end: Optional[int] = None,
                     size_factor: float = 1.0):
    """``quantized.py:1173-1216`` -> ``(data, indices, indptr)`` of the rows
    ``[start, end)`` (dim 0) or the columns ``[start, end)`` (dim 1, shifted
    to start at 0), in ``int(data.shape[0] * size_factor)`` slots."""
    dim = dim + 2 if dim < 0 else dim
    if dim not in [0, 1]:
        raise ValueError(f"Cannot slice sparse CSR matrix along dim {dim}")
    _ops._check_cuda(data, "slice_csr_tensor")
    if start is None or end is None:
        raise ValueError("slice_csr_tensor on CUDA needs both start and end")
    dev = data.device
    rows = indptr.shape[0] - 1
    start, end = int(start), int(end)
    if dim == 0 and not 0 <= start <= end <= rows:
        raise ValueError(f"row slice [{start}, {end}) outside the {rows} rows")
    if dim == 1 and start < 0:
        raise ValueError(f"column slice start {start} is negative")
    max_out = int(data.shape[0] * size_factor)
    d = data.contiguous()
    ix = _ops._on(indices, dev)
    ip = _ops._on(indptr, dev)
    if ix.dtype != torch.int32:
        ix = ix.to(torch.int32)
    if ip.dtype != torch.int32:
        ip = ip.to(torch.int32)
    new_data = torch.empty(max_out, dtype=d.dtype, device=dev)
    new_indices = torch.empty(max_out, dtype=torch.int32, device=dev)
    n_ptr = end - start + 1 if dim == 0 else rows + 1
    new_indptr = torch.empty(n_ptr, dtype=torch.int32, device=dev)
    ws = torch.empty(2 * rows + 1, dtype=torch.int32, device=dev) if dim == 1 else None
    st = _ops.lib().vq_slice_csr(_ops._ref(_ops._vt(d)), ix.data_ptr() if ix.numel() else None,
                                 ip.data_ptr(), rows, dim, start, end, max_out,
                                 new_data.data_ptr() if max_out else None,
                                 new_indices.data_ptr() if max_out else None,
                                 new_indptr.data_ptr(), None if ws is None else ws.data_ptr(),
                                 _ops._stream(dev))
    _lib.check(st, "quantized_ops::slice_csr_tensor")
    return new_data, new_indices, new_indptr
