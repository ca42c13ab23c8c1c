"""``linear_mx`` / ``matmul_mx`` on CUDA (``src/voyager_compiler/ops/quantized.py:522-648``).

Both operands are read back through their codebook and block scale
(``_dequantize_mx``, ``quantized.py:455-472``) and multiplied with float32
accumulation, the result in the operands' dtype.

Paths, chosen per call:
  * MXFP8 x MXFP8 (E4M3 codes, power-of-two block-32 scales along K on both
    operands, bf16): the tcgen05 block-scaled GEMM in ``libvoyager_b200``
    (``voyager_b200.mxgemm``), weights packed once and cached;
  * NVFP4 x NVFP4 (E2M1 codes, E4M3 scales per 16 along K on both): the
    tcgen05 ``kind::mxf4nvf4`` block-scaled GEMM (``mxgemm.nvf4_linear``);
  * every other bf16 operand pair: the tcgen05 bf16 GEMM
    (``voyager_b200.dqgemm``), the weight read back from palette indices in
    shared memory (or, when it does not fit that form, by this library's
    dequantize kernels), the activations by the dequantize kernels;
  * float32 / float16 operands: dequantized by this library's kernels and
    multiplied by torch (the tcgen05 kernels multiply bf16 and FP8).
With the outlier CSR side-stream (``A_data`` / ``A_indices`` / ``A_indptr``)
the result is the dense product plus ``spmm_csr`` of the CSR with the
decoded weight (``quantized.py:560-574``, ``:625-637``); on the MXFP8 path
the addition is the GEMM epilogue's residual add (one bf16 rounding of the
dense product, then the bf16 sum, as the reference's two bf16 tensors add).
"""

from typing import Optional

import torch
import torch.nn.functional as F

from voyager_b200 import ops as _ops
from voyager_b200._cache import TensorCache

_wcache = TensorCache()


def dequantize_mx(x: torch.Tensor, scale: Optional[torch.Tensor], code: Optional[torch.Tensor],
                  block_size: Optional[int]) -> torch.Tensor:
    """``_dequantize_mx``: decode through ``code``, then scale by the
    expand()ed block ``scale``; either may be absent."""
    if code is None and scale is None:
        return x
    if code is not None:
        from voyager_b200 import codebook as cbm

        try:
            x = _ops.vmap(x, cbm.decode_table(code, x.dtype, x.device))
        except NotImplementedError:
            # one table per region, or float32 entries bf16 cannot hold
            x = cbm.decode(x, code.to(x.device))
    if scale is not None:
        x = _ops.dequantize(x, scale, None, None, block_size)
    return x


def _weight_dequant(w, scale, code, bs):
    """Dequantized weights, cached per (tensor, version) of codes and scale."""
    key = (w._version, None if scale is None else (id(scale), scale._version),
           None if code is None else (id(code), code._version), bs)
    hit = _wcache.get(w, key)
    if hit is not None:
        return hit
    return _wcache.put(w, key, dequantize_mx(w, scale, code, bs))


def _outliers(A_data, A_indices, A_indptr, weight, weight_scale, weight_code, block_size,
              weight_layout):
    """spmm_csr of the CSR side-stream with the weight, or None."""
    if A_data is None:
        return None
    from voyager_b200.outlier import spmm_csr

    return spmm_csr(A_data, A_indices, A_indptr, weight, weight_scale, weight_code, block_size,
                    weight_layout)


def linear_mx(input, weight, bias=None, *, input_scale=None, weight_scale=None,
              block_size=None, input_code=None, weight_code=None, A_data=None,
              A_indices=None, A_indptr=None, weight_layout="kc"):
    assert weight_layout in ("kc", "ck"), weight_layout
    from voyager_b200 import mxgemm

    sp = _outliers(A_data, A_indices, A_indptr, weight, weight_scale, weight_code, block_size,
                   weight_layout)
    if mxgemm.applies(input, weight, input_scale, weight_scale, block_size, input_code,
                      weight_code, weight_layout, "linear"):
        res = None
        if sp is not None and sp.dtype == torch.bfloat16 and sp.shape[-1] == weight.shape[0] \
                and sp.numel() == input.numel() // input.shape[-1] * weight.shape[0]:
            res = sp.contiguous()
        if sp is None or res is not None:
            out = mxgemm.linear(input, weight, bias, input_scale, weight_scale, residual=res)
            if out is not None:
                return out
    if sp is None and mxgemm.nvf4_applies(input, weight, input_scale, weight_scale, block_size,
                                          input_code, weight_code, weight_layout, "linear"):
        out = mxgemm.nvf4_linear(input, weight, bias, input_scale, weight_scale)
        if out is not None:
            return out
    from voyager_b200 import dqgemm

    out = dqgemm.linear(input, weight, bias, input_scale, weight_scale, block_size, input_code,
                        weight_code, weight_layout)
    if out is not None:
        return out if sp is None else out + sp
    a = dequantize_mx(input, input_scale, input_code, block_size)
    w = _weight_dequant(weight, weight_scale, weight_code, block_size)
    if weight_layout == "ck":
        w = w.transpose(-1, -2)
    out = F.linear(a, w, bias)
    return out if sp is None else out + sp


def matmul_mx(self, other, *, input_scale=None, weight_scale=None, block_size=None,
              input_code=None, weight_code=None, A_data=None, A_indices=None, A_indptr=None,
              weight_layout="ck"):
    assert weight_layout in ("kc", "ck"), weight_layout
    from voyager_b200 import mxgemm

    sp = _outliers(A_data, A_indices, A_indptr, other, weight_scale, weight_code, block_size,
                   weight_layout)
    if mxgemm.matmul_applies(self, other, input_scale, weight_scale, block_size, input_code,
                             weight_code, weight_layout):
        out = mxgemm.matmul(self, other, input_scale, weight_scale, weight_layout)
        if out is not None:
            return out if sp is None else out + sp
    from voyager_b200 import dqgemm

    out = dqgemm.matmul(self, other, input_scale, weight_scale, block_size, input_code,
                        weight_code, weight_layout)
    if out is not None:
        return out if sp is None else out + sp
    a = dequantize_mx(self, input_scale, input_code, block_size)
    b = dequantize_mx(other, weight_scale, weight_code, block_size)
    if weight_layout == "kc":
        b = b.transpose(-1, -2)
    out = torch.matmul(a, b)
    return out if sp is None else out + sp
