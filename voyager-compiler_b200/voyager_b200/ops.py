"""CUDA kernels for the reference's ``quantized_ops`` torch.library ops.

The reference defines the namespace in
``src/voyager_compiler/ops/quantized.py:88`` (``Library("quantized_ops",
"DEF")``) with ``CompositeExplicitAutograd`` bodies, and registers
``torch.compile``d copies of four of them on the CUDA key
(``quantized.py:951-955``).  Importing this module registers the B200
kernels on the CUDA key of the same ops instead, so exported and converted
graphs dispatch here unchanged.  If the reference is not imported, the
namespace is defined here with the reference's schemas, verbatim, plus Meta
kernels for shape propagation; CPU tensors then have no kernel (there is no
CPU fallback in this package).  Import the reference (``voyager_compiler.ops``)
before this module when both are used.

Every function mirrors the reference op of the same name: same arguments,
same result dtypes and shapes, same assertion / ValueError behaviour.
"""

import ctypes
import math
from typing import List, Optional, Sequence

import torch

from voyager_b200 import _lib
from voyager_b200.tables import QMAP_SIZE, Rounder, floor_log2, rounder_for

_L = None


def lib():
    global _L
    if _L is None:
        _L = _lib.load()
    return _L


_DTYPES = {torch.bfloat16: _lib.VQ_BF16, torch.float32: _lib.VQ_F32}


def _vq_dtype(dt: torch.dtype) -> int:
    if dt not in _DTYPES:
        raise NotImplementedError(
            f"quantized_ops on CUDA: dtype {dt} is not provided by the B200 kernels "
            "(bfloat16 and float32 are)")
    return _DTYPES[dt]


def _vt(t: Optional[torch.Tensor]):
    if t is None:
        return None
    v = _lib.VqTensor()
    v.data = t.data_ptr() if t.numel() else None
    v.dtype = _vq_dtype(t.dtype)
    v.ndim = t.dim()
    if t.dim() > _lib.VQ_MAX_DIMS:
        raise NotImplementedError(f"tensors of more than {_lib.VQ_MAX_DIMS} dims")
    for i, s in enumerate(t.shape):
        v.shape[i] = s
    return v


def _ref(v):
    return None if v is None else ctypes.byref(v)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _on(t: Optional[torch.Tensor], dev: torch.device) -> Optional[torch.Tensor]:
    """Operand on the kernel's device, dense.  A CPU 0-d scalar (which torch
    lets a CUDA op take) is copied over."""
    if t is None:
        return None
    if t.device != dev:
        t = t.to(dev, non_blocking=True)
    return t.contiguous()


def _promote(da: torch.dtype, na: int, db: torch.dtype, nb: int) -> torch.dtype:
    """torch's result dtype for float operands: a 0-d operand does not
    promote a dimensioned one."""
    if nb == 0 and na > 0:
        return da
    if na == 0 and nb > 0:
        return db
    return torch.promote_types(da, db)


def _norm_axes(axes, ndim) -> List[int]:
    axes = [axes] if isinstance(axes, int) else list(axes)
    return sorted({a + ndim if a < 0 else a for a in axes})


def _blocked_shape(shape: Sequence[int], axes: List[int], bs: int) -> List[int]:
    return [(-(-s // bs) if d in axes else s) for d, s in enumerate(shape)]


def _check_cuda(x: torch.Tensor, op: str):
    if not x.is_cuda:
        raise NotImplementedError(f"quantized_ops::{op}: the B200 kernels take CUDA tensors")


# ---------------------------------------------------------------------------
# ops
# ---------------------------------------------------------------------------
def quantize(input: torch.Tensor, scale: torch.Tensor, zero_point=None, axes=None,
             block_size=None, qmap=None, output_code=None) -> torch.Tensor:
    """``quantized.py:340-397``."""
    assert qmap is not None, "qmap must be provided for quantization"
    _check_cuda(input, "quantize")
    dev = input.device
    x = input.contiguous()
    s, z = _on(scale, dev), _on(zero_point, dev)
    r1 = _promote(x.dtype, x.dim(), s.dtype, s.dim())
    r2 = r1 if z is None else _promote(r1, x.dim(), z.dtype, z.dim())
    if not (qmap.numel() == QMAP_SIZE and qmap.dim() == 1):
        # a codebook: encode() is a function of the bf16 pattern, i.e. a table
        from voyager_b200 import codebook as cbm

        table = None
        if qmap.dim() == 1:
            try:
                table = cbm.encode_table(qmap, output_code, r2, dev)
            except NotImplementedError:
                table = None
        if table is None:
            # one table per region (or float32 entries bf16 cannot hold):
            # the bf16-rounded quotients through the identity table, then
            # each element through its region's table
            counts = cbm.region_counts(qmap, x.shape)
            t = quantize(x, s, z, axes, block_size, _identity(dev))
            tabs = cbm.encode_tables(qmap, _on(output_code, dev) if output_code is not None
                                     else None, r2, dev)
            return cbm.lookup(t, counts, tabs, r2)
        qmap = table
    out = torch.empty(x.shape, dtype=r2, device=dev)
    rd = rounder_for(qmap, dev)
    st = lib().vq_quantize(_ref(_vt(x)), _ref(_vt(s)), _ref(_vt(z)),
                           int(block_size or 0), rd.ref(), _ref(_vt(out)), _stream(dev))
    _lib.check(st, "quantized_ops::quantize")
    return out


def dequantize(input: torch.Tensor, scale: torch.Tensor, zero_point=None, axes=None,
               block_size=None, input_qmap=None, output_qmap=None) -> torch.Tensor:
    """``quantized.py:400-452``."""
    _check_cuda(input, "dequantize")
    dev = input.device
    x = input.contiguous()
    s, z = _on(scale, dev), _on(zero_point, dev)
    r1 = x.dtype if z is None else _promote(x.dtype, x.dim(), z.dtype, z.dim())
    r2 = _promote(r1, x.dim(), s.dtype, s.dim())
    out = torch.empty(x.shape, dtype=r2, device=dev)
    iq = rounder_for(input_qmap, dev) if input_qmap is not None else None
    oq = rounder_for(output_qmap, dev) if output_qmap is not None else None
    st = lib().vq_dequantize(_ref(_vt(x)), _ref(_vt(s)), _ref(_vt(z)), int(block_size or 0),
                             iq.ref() if iq else None, oq.ref() if oq else None,
                             _ref(_vt(out)), _stream(dev))
    _lib.check(st, "quantized_ops::dequantize")
    return out


_ONES = {}
_IDENT = {}


def _identity(dev):
    """The identity table (entry = its bf16 pattern) on ``dev``."""
    t = _IDENT.get(str(dev))
    if t is None:
        t = torch.arange(QMAP_SIZE, dtype=torch.int32).to(torch.int16).view(
            torch.bfloat16).to(dev)
        _IDENT[str(dev)] = t
    return t


def _one(dev, dtype):
    k = (str(dev), dtype)
    t = _ONES.get(k)
    if t is None:
        t = torch.ones((), dtype=dtype, device=dev)
        _ONES[k] = t
    return t


def vmap(input: torch.Tensor, qmap: torch.Tensor) -> torch.Tensor:
    """``quantized.py:174-203``: the table entry of each element's bfloat16
    pattern, in the input's dtype."""
    _check_cuda(input, "vmap")
    return dequantize(input, _one(input.device, input.dtype), input_qmap=qmap)


def calculate_mx_qparam(input: torch.Tensor, axes, block_size: int, quant_max: float,
                        force_scale_power_of_two: bool = False,
                        scale_qmap: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``quantized.py:787-851``."""
    assert block_size > 0
    _check_cuda(input, "calculate_mx_qparam")
    dev = input.device
    x = input.contiguous()
    ax = _norm_axes(axes, x.dim())
    out = torch.empty(_blocked_shape(x.shape, ax, block_size), dtype=x.dtype, device=dev)
    sq = rounder_for(scale_qmap, dev) if scale_qmap is not None else None
    axes_c = (ctypes.c_int64 * len(ax))(*ax)
    fl2q = floor_log2(quant_max) if force_scale_power_of_two else 0
    st = lib().vq_calculate_mx_qparam(_ref(_vt(x)), axes_c, len(ax), int(block_size),
                                      float(quant_max), int(bool(force_scale_power_of_two)),
                                      fl2q, sq.ref() if sq else None, _ref(_vt(out)),
                                      _stream(dev))
    _lib.check(st, "quantized_ops::calculate_mx_qparam")
    return out


def quantize_mx(input: torch.Tensor, qmap: torch.Tensor, axes, block_size: int,
                quant_max: float, force_scale_power_of_two: bool = False,
                scale_qmap: Optional[torch.Tensor] = None,
                output_code: Optional[torch.Tensor] = None):
    """``quantized.py:854-881`` -> ``(scale, codes)``; one fused pass when
    the blocks run along the last dim."""
    assert block_size > 0
    _check_cuda(input, "quantize_mx")
    if not (qmap.numel() == QMAP_SIZE and qmap.dim() == 1):
        scale = calculate_mx_qparam(input, axes, block_size, quant_max,
                                    force_scale_power_of_two, scale_qmap)
        return scale, quantize(input, scale, None, axes, block_size, qmap, output_code)
    dev = input.device
    x = input.contiguous()
    ax = _norm_axes(axes, x.dim())
    scale = torch.empty(_blocked_shape(x.shape, ax, block_size), dtype=x.dtype, device=dev)
    codes = torch.empty_like(x)
    rd = rounder_for(qmap, dev)
    sq = rounder_for(scale_qmap, dev) if scale_qmap is not None else None
    fl2q = floor_log2(quant_max) if force_scale_power_of_two else 0
    mxfp8 = (block_size == 32 and ax == [x.dim() - 1] and force_scale_power_of_two
             and scale_qmap is None and x.dtype == torch.bfloat16 and x.dim() >= 1
             and rd.c.kind == _lib.VQ_R_MINIFLOAT and rd.c.hw == 1)
    if mxfp8 and x.shape[-1] % 128 == 0 and x.numel() > 0:
        # MXFP8 activations: also write the tcgen05 GEMM operand in this pass
        from voyager_b200 import mxgemm

        C = x.shape[-1]
        R = x.numel() // C
        rt = (R + 127) // 128
        packed = torch.empty(rt * 128 * C, dtype=torch.uint8, device=dev)
        packed_sf = torch.empty((C // 128) * rt * 512, dtype=torch.uint8, device=dev)
        st = lib().vq_quantize_mx_packed(_ref(_vt(x.view(R, C))), rd.ref(), fl2q,
                                         _ref(_vt(scale.view(R, C // 32))),
                                         _ref(_vt(codes.view(R, C))), packed.data_ptr(),
                                         packed_sf.data_ptr(), _stream(dev))
        _lib.check(st, "quantized_ops::quantize_mx")
        mxgemm.vouch(codes, scale, (packed, packed_sf))
        return scale, codes
    axes_c = (ctypes.c_int64 * len(ax))(*ax)
    st = lib().vq_quantize_mx(_ref(_vt(x)), rd.ref(), axes_c, len(ax), int(block_size),
                              float(quant_max), int(bool(force_scale_power_of_two)), fl2q,
                              sq.ref() if sq else None, _ref(_vt(scale)), _ref(_vt(codes)),
                              _stream(dev))
    _lib.check(st, "quantized_ops::quantize_mx")
    if mxfp8:
        # E4M3 codes with power-of-two scales: the MXFP8 GEMM may take them
        # without re-checking
        from voyager_b200 import mxgemm

        mxgemm.vouch(codes, scale)
    elif (block_size == 32 and x.dim() >= 2 and ax == [x.dim() - 2] and force_scale_power_of_two
          and scale_qmap is None and x.dtype == torch.bfloat16
          and rd.c.kind == _lib.VQ_R_MINIFLOAT and rd.c.hw == 1):
        # blocks along dim -2: the right operand of a matmul_mx stored [.., K, N]
        from voyager_b200 import mxgemm

        mxgemm.vouch(codes, scale, axis=-2)
    return scale, codes


def quantize_affine(input: torch.Tensor, qmap: torch.Tensor, axes, block_size: int,
                    quant_min: float, quant_max: float,
                    scale_qmap: Optional[torch.Tensor] = None):
    """``quantized.py:884-948`` -> ``(scale, zero_point, codes)``: per-block
    parameters from each block's min / max, then an affine quantize."""
    assert block_size > 0
    _check_cuda(input, "quantize_affine")
    (axis,) = axes
    dev = input.device
    x = input.contiguous()
    ax = [axis % x.dim()]
    shape = _blocked_shape(x.shape, ax, block_size)
    scale = torch.empty(shape, dtype=x.dtype, device=dev)
    zp = torch.empty(shape, dtype=x.dtype, device=dev)
    sq = rounder_for(scale_qmap, dev) if scale_qmap is not None else None
    axes_c = (ctypes.c_int64 * 1)(ax[0])
    st = lib().vq_quantize_affine_qparams(_ref(_vt(x)), axes_c, 1, int(block_size),
                                          float(quant_min), float(quant_max),
                                          sq.ref() if sq else None, _ref(_vt(scale)),
                                          _ref(_vt(zp)), _stream(dev))
    _lib.check(st, "quantized_ops::quantize_affine")
    return scale, zp, quantize(x, scale, zp, ax, block_size, qmap)


def linear_mx(input, weight, bias=None, *, input_scale=None, weight_scale=None,
              block_size=None, input_code=None, weight_code=None, A_data=None,
              A_indices=None, A_indptr=None, weight_layout="kc"):
    """``quantized.py:522-586``."""
    from voyager_b200.gemm import linear_mx as impl

    return impl(input, weight, bias, input_scale=input_scale, weight_scale=weight_scale,
                block_size=block_size, input_code=input_code, weight_code=weight_code,
                A_data=A_data, A_indices=A_indices, A_indptr=A_indptr,
                weight_layout=weight_layout)


def matmul_mx(self, other, *, input_scale=None, weight_scale=None, block_size=None,
              input_code=None, weight_code=None, A_data=None, A_indices=None, A_indptr=None,
              weight_layout="ck"):
    """``quantized.py:589-648``."""
    from voyager_b200.gemm import matmul_mx as impl

    return impl(self, other, input_scale=input_scale, weight_scale=weight_scale,
                block_size=block_size, input_code=input_code, weight_code=weight_code,
                A_data=A_data, A_indices=A_indices, A_indptr=A_indptr,
                weight_layout=weight_layout)


def sdpa_mx(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False,
            query_residual=None, key_residual=None, value_residual=None, residual_mask=None,
            *, scale=None, enable_gqa=False, query_scale=None, key_scale=None, value_scale=None,
            block_size=None, input_code=None, weight_code=None, probs_qmap=None,
            probs_quant_max=None, probs_scale_qmap=None, probs_code=None,
            force_scale_power_of_two=False):
    """``quantized.py:651-784``."""
    from voyager_b200.attention import sdpa_mx as impl

    return impl(query, key, value, attn_mask, dropout_p, is_causal, query_residual,
                key_residual, value_residual, residual_mask, scale=scale, enable_gqa=enable_gqa,
                query_scale=query_scale, key_scale=key_scale, value_scale=value_scale,
                block_size=block_size, input_code=input_code, weight_code=weight_code,
                probs_qmap=probs_qmap, probs_quant_max=probs_quant_max,
                probs_scale_qmap=probs_scale_qmap, probs_code=probs_code,
                force_scale_power_of_two=force_scale_power_of_two)


def filter_outlier(input, threshold, max_pct=0.01):
    """``quantized.py:995-1045``."""
    from voyager_b200.outlier import filter_outlier as impl

    return impl(input, threshold, max_pct)


def quantize_mx_outlier(input, qmap, axes, block_size, quant_max,
                        force_scale_power_of_two=False, scale_qmap=None, output_code=None,
                        threshold=None, max_pct=0.01, indptr_offset=0):
    """``quantized.py:1078-1130``."""
    from voyager_b200.outlier import quantize_mx_outlier as impl

    return impl(input, qmap, axes, block_size, quant_max, force_scale_power_of_two,
                scale_qmap, output_code, threshold, max_pct, indptr_offset)


def slice_csr_tensor(data, indices, indptr, dim=0, start=None, end=None, size_factor=1.0):
    """``quantized.py:1173-1216``."""
    from voyager_b200.outlier import slice_csr_tensor as impl

    return impl(data, indices, indptr, dim, start, end, size_factor)


def spmm_csr(data, indices, indptr, B, B_scale=None, B_code=None, block_size=None,
             weight_layout="kc"):
    """``quantized.py:1245-1311``."""
    from voyager_b200.outlier import spmm_csr as impl

    return impl(data, indices, indptr, B, B_scale, B_code, block_size, weight_layout)


# ---------------------------------------------------------------------------
# registration
# ---------------------------------------------------------------------------
SCHEMAS = {
    "vmap": "vmap(Tensor self, Tensor other) -> Tensor",
    "quantize": (
        "quantize(Tensor input, Tensor scale, Tensor? zero_point=None, "
        "SymInt[]? axes=None, int? block_size=None, Tensor? qmap=None, "
        "Tensor? output_code=None) -> Tensor"),
    "dequantize": (
        "dequantize(Tensor input, Tensor scale, Tensor? zero_point=None, "
        "SymInt[]? axes=None, int? block_size=None, Tensor? input_qmap=None, "
        "Tensor? output_qmap=None) -> Tensor"),
    "linear_mx": (
        "linear_mx(Tensor input, Tensor weight, Tensor? bias=None, *, "
        "Tensor? input_scale=None, Tensor? weight_scale=None, "
        "int? block_size=None, Tensor? input_code=None, Tensor? weight_code=None, "
        "Tensor? A_data=None, Tensor? A_indices=None, Tensor? A_indptr=None, "
        'str weight_layout="kc") -> Tensor'),
    "matmul_mx": (
        "matmul_mx(Tensor self, Tensor other, *, Tensor? input_scale=None, "
        "Tensor? weight_scale=None, int? block_size=None, Tensor? input_code=None, "
        "Tensor? weight_code=None, Tensor? A_data=None, Tensor? A_indices=None, "
        'Tensor? A_indptr=None, str weight_layout="ck") -> Tensor'),
    "sdpa_mx": (
        "sdpa_mx(Tensor query, Tensor key, Tensor value, Tensor? attn_mask=None, "
        "float dropout_p=0., bool is_causal=False, Tensor? query_residual=None, "
        "Tensor? key_residual=None, Tensor? value_residual=None, "
        "Tensor? residual_mask=None, *, float? scale=None, "
        "bool enable_gqa=False, Tensor? query_scale=None, Tensor? key_scale=None, "
        "Tensor? value_scale=None, int? block_size=None, Tensor? input_code=None, "
        "Tensor? weight_code=None, Tensor? probs_qmap=None, "
        "float? probs_quant_max=None, Tensor? probs_scale_qmap=None, "
        "Tensor? probs_code=None, bool force_scale_power_of_two=False) -> Tensor"),
    "calculate_mx_qparam": (
        "calculate_mx_qparam(Tensor self, SymInt[] axes, int block_size, "
        "float quant_max, bool force_scale_power_of_two=False, "
        "Tensor scale_qmap=None) -> Tensor"),
    "quantize_mx": (
        "quantize_mx(Tensor self, Tensor qmap, SymInt[] axes, int block_size, "
        "float quant_max, bool force_scale_power_of_two=False, "
        "Tensor scale_qmap=None, Tensor output_code=None) -> (Tensor, Tensor)"),
    "quantize_affine": (
        "quantize_affine(Tensor self, Tensor qmap, SymInt[] axes, int block_size, "
        "float quant_min, float quant_max, Tensor scale_qmap=None) "
        "-> (Tensor, Tensor, Tensor)"),
    "filter_outlier": (
        "filter_outlier(Tensor input, float threshold, float max_pct=0.01) "
        "-> (Tensor, Tensor, Tensor, Tensor)"),
    "quantize_mx_outlier": (
        "quantize_mx_outlier(Tensor self, Tensor qmap, SymInt[] axes, "
        "int block_size, float quant_max, bool force_scale_power_of_two=False, "
        "Tensor scale_qmap=None, Tensor output_code=None, float? threshold=None, "
        "float max_pct=0.01, SymInt indptr_offset=0) "
        "-> (Tensor, Tensor, Tensor, Tensor, Tensor)"),
    "slice_csr_tensor": (
        "slice_csr_tensor(Tensor data, Tensor indices, Tensor indptr, int dim=0, "
        "SymInt? start=None, SymInt? end=None, float size_factor=1.0) "
        "-> (Tensor, Tensor, Tensor)"),
    "spmm_csr": (
        "spmm_csr(Tensor data, Tensor indices, Tensor indptr, Tensor B, "
        "Tensor? B_scale=None, Tensor? B_code=None, int? block_size=None, "
        'str weight_layout="kc") -> Tensor'),
}

CUDA_IMPLS = {
    "vmap": vmap,
    "quantize": quantize,
    "dequantize": dequantize,
    "calculate_mx_qparam": calculate_mx_qparam,
    "quantize_mx": quantize_mx,
    "quantize_affine": quantize_affine,
    "linear_mx": linear_mx,
    "matmul_mx": matmul_mx,
    "sdpa_mx": sdpa_mx,
    "filter_outlier": filter_outlier,
    "quantize_mx_outlier": quantize_mx_outlier,
    "slice_csr_tensor": slice_csr_tensor,
    "spmm_csr": spmm_csr,
}


def _meta_impls():
    """Shape / dtype propagation for the namespace defined here."""

    def q(input, scale, zero_point=None, axes=None, block_size=None, qmap=None, output_code=None):
        r = _promote(input.dtype, input.dim(), scale.dtype, scale.dim())
        if zero_point is not None:
            r = _promote(r, input.dim(), zero_point.dtype, zero_point.dim())
        return input.new_empty(input.shape, dtype=r)

    def dq(input, scale, zero_point=None, axes=None, block_size=None, input_qmap=None,
           output_qmap=None):
        r = input.dtype
        if zero_point is not None:
            r = _promote(r, input.dim(), zero_point.dtype, zero_point.dim())
        r = _promote(r, input.dim(), scale.dtype, scale.dim())
        return input.new_empty(input.shape, dtype=r)

    def vm(input, qmap):
        return input.new_empty(input.shape)

    def mxq(input, axes, block_size, quant_max, force_scale_power_of_two=False,
            scale_qmap=None):
        return input.new_empty(_blocked_shape(input.shape, _norm_axes(axes, input.dim()),
                                              block_size))

    def qmx(input, qmap, axes, block_size, quant_max, force_scale_power_of_two=False,
            scale_qmap=None, output_code=None):
        return mxq(input, axes, block_size, quant_max), input.new_empty(input.shape)

    def qaff(input, qmap, axes, block_size, quant_min, quant_max, scale_qmap=None):
        s = mxq(input, axes, block_size, quant_max)
        return s, s.new_empty(s.shape), input.new_empty(input.shape)

    def lin(input, weight, bias=None, **kw):
        n = weight.shape[-1] if kw.get("weight_layout", "kc") == "ck" else weight.shape[0]
        return input.new_empty(list(input.shape[:-1]) + [n])

    def mm(self, other, **kw):
        if kw.get("weight_layout", "ck") == "kc":
            other = other.transpose(-1, -2)
        return torch.matmul(self, other)

    def sdpa(query, key, value, *a, **kw):
        return query.new_empty(list(query.shape[:-1]) + [value.shape[-1]])

    def csr_fake(input, max_pct):
        batch, mat = list(input.shape[:-2]), list(input.shape[-2:])
        nnz = int(math.prod(mat) * max_pct)
        return (input.new_empty(batch + [nnz]),
                input.new_empty(batch + [nnz], dtype=torch.int32),
                input.new_empty(batch + [mat[0] + 1], dtype=torch.int32))

    def fo(input, threshold, max_pct=0.01):
        return (*csr_fake(input, max_pct), torch.empty_like(input))

    def qmxo(input, qmap, axes, block_size, quant_max, force_scale_power_of_two=False,
             scale_qmap=None, output_code=None, threshold=None, max_pct=0.01, indptr_offset=0):
        return (*csr_fake(input, max_pct), mxq(input, axes, block_size, quant_max),
                torch.empty_like(input, memory_format=torch.contiguous_format))

    def slc(data, indices, indptr, dim=0, start=None, end=None, size_factor=1.0):
        p = indptr.new_empty(indptr.shape)
        if dim in (0, -2):
            p = p[start:end + 1]
        return torch.empty_like(data), torch.empty_like(indices), p

    def spmm(data, indices, indptr, B, B_scale=None, B_code=None, block_size=None,
             weight_layout="kc"):
        n = B.shape[-1] if weight_layout == "ck" else B.shape[-2]
        return data.new_empty(list(indptr.shape[:-1]) + [indptr.shape[-1] - 1, n])

    return {"quantize": q, "dequantize": dq, "vmap": vm, "calculate_mx_qparam": mxq,
            "quantize_mx": qmx, "quantize_affine": qaff, "linear_mx": lin, "matmul_mx": mm,
            "sdpa_mx": sdpa, "filter_outlier": fo, "quantize_mx_outlier": qmxo,
            "slice_csr_tensor": slc, "spmm_csr": spmm}


_LIBS = []
_REGISTERED = {"defined_here": False, "ops": []}


def _op_exists(name: str) -> bool:
    try:
        getattr(torch.ops.quantized_ops, name)
        return True
    except (AttributeError, RuntimeError):
        return False


def register() -> dict:
    """Register the CUDA kernels (idempotent).  Returns what was done."""
    if _REGISTERED["ops"]:
        return _REGISTERED
    import warnings

    if not _op_exists("quantize"):
        d = torch.library.Library("quantized_ops", "DEF")
        _LIBS.append(d)
        for name, schema in SCHEMAS.items():
            d.define(schema)
        metas = _meta_impls()
        for name in SCHEMAS:
            d.impl(name, metas[name], "Meta")
        _REGISTERED["defined_here"] = True
    impl = torch.library.Library("quantized_ops", "IMPL")
    _LIBS.append(impl)
    with warnings.catch_warnings():
        # the reference registers torch.compile'd CUDA kernels for some ops;
        # replacing them is the point of this package
        warnings.simplefilter("ignore")
        for name, fn in CUDA_IMPLS.items():
            if _op_exists(name):
                impl.impl(name, fn, "CUDA")
                _REGISTERED["ops"].append(name)
    return _REGISTERED
