"""``sdpa_mx`` on CUDA (``src/voyager_compiler/ops/quantized.py:651-784``).

Fused path (``vq_attn_mxf8``, one tcgen05 kernel): MXFP8 operands -- E4M3
codes with power-of-two block-32 scales, query / key blocked along
head_dim, value along the keys -- probabilities quantized to E4M3 with
power-of-two block-32 scales, no codebooks, no residual, no explicit mask,
head_dim 128, sequence lengths multiples of 128, bf16.  The scores and
probabilities never leave the chip.

Everything else runs the reference's composition on the GPU: operands
dequantized by this library's kernels, the two products on this library's
tcgen05 bf16 GEMM (torch's matmul only for shapes it does not take), the
mask and the float32 softmax with torch's elementwise ops, the
probabilities through this library's ``quantize_mx``.

The fused output is returned as a [B, H, Sq, D] view of a [B, Sq, H, D]
buffer, the layout the following o_proj reads, so a caller's
``transpose(1, 2).reshape(B, Sq, H * D)`` costs nothing.
"""

import math
import os
from typing import Optional

import torch

from voyager_b200 import _lib

CHECK_ERRORS = os.environ.get("VQ_CHECK_ERRORS", "0") == "1"


def _packed_operand(codes: torch.Tensor, scale: torch.Tensor):
    """(E4M3 bytes, scale atoms) of a contiguous [.., C] operand blocked
    along its last dim: the buffers quantize_mx wrote in the same pass when
    it did, else packed now (with the exactness check); None if inexact."""
    from voyager_b200 import mxgemm

    entry = mxgemm._vouched_entry(codes, scale)
    if entry is not None and entry[1] is not None:
        return entry[1]
    C = codes.shape[-1]
    pc, ps, ok = mxgemm._pack(codes.reshape(-1, C), scale.reshape(-1, scale.shape[-1]), 128,
                              entry is None)
    return (pc, ps) if ok else None


def _value_transposed(value: torch.Tensor, value_scale: torch.Tensor):
    """value [.., S, D] with scales [.., S/32, D] -> the packed V^T operand
    [.., D, S].  A value passed as the transposed view of a contiguous
    quantize_mx output (blocks along its last dim) is used as it is."""
    vb, sb = value._base, value_scale._base
    if (vb is not None and sb is not None and vb.is_contiguous() and sb.is_contiguous()
            and vb.dim() == value.dim() and tuple(vb.shape) == tuple(value.transpose(-1, -2).shape)
            and value.data_ptr() == vb.data_ptr()
            and value.stride() == vb.transpose(-1, -2).stride()
            and tuple(sb.shape) == tuple(value_scale.transpose(-1, -2).shape)
            and value_scale.data_ptr() == sb.data_ptr()
            and value_scale.stride() == sb.transpose(-1, -2).stride()):
        return _packed_operand(vb, sb)
    return _packed_operand(value.transpose(-1, -2).contiguous(),
                           value_scale.transpose(-1, -2).contiguous())


def _fused_applies(query, key, value, attn_mask, residual, enable_gqa, query_scale, key_scale,
                   value_scale, block_size, input_code, weight_code, probs_qmap,
                   probs_scale_qmap, probs_code, force_scale_power_of_two) -> bool:
    if residual or attn_mask is not None or block_size != 32 or not force_scale_power_of_two:
        return False
    if any(t is not None for t in (input_code, weight_code, probs_code, probs_scale_qmap)):
        return False
    if probs_qmap is None or query_scale is None or key_scale is None or value_scale is None:
        return False
    ts = (query, key, value, query_scale, key_scale, value_scale)
    if any(t.dtype != torch.bfloat16 or not t.is_cuda or t.dim() != 4 for t in ts):
        return False
    B, H, Sq, D = query.shape
    Bk, Hkv, Skv, Dk = key.shape
    if D != 128 or Dk != 128 or tuple(value.shape) != (Bk, Hkv, Skv, 128) or Bk != B:
        return False
    if Sq % 128 or Skv % 128 or H % Hkv or (Hkv != H and not enable_gqa):
        return False
    if (tuple(query_scale.shape) != (B, H, Sq, 4) or tuple(key_scale.shape) != (B, Hkv, Skv, 4)
            or tuple(value_scale.shape) != (B, Hkv, Skv // 32, 128)):
        return False
    if not (query.is_contiguous() and key.is_contiguous()):
        return False
    from voyager_b200.tables import rounder_for

    rd = rounder_for(probs_qmap, query.device)
    return rd.c.kind == _lib.VQ_R_MINIFLOAT and rd.c.hw == 1


def _fused(query, key, value, is_causal, scale, query_scale, key_scale, value_scale,
           probs_quant_max):
    from voyager_b200.ops import _stream, floor_log2

    B, H, Sq, D = query.shape
    Hkv, Skv = key.shape[1], key.shape[2]
    pq = _packed_operand(query, query_scale)
    pk = _packed_operand(key, key_scale)
    pv = _value_transposed(value, value_scale)
    if pq is None or pk is None or pv is None:
        return None
    dev = query.device
    buf = torch.empty((B, Sq, H, D), dtype=torch.bfloat16, device=dev)
    err = torch.empty(1, dtype=torch.int32, device=dev)
    st = _lib.load().vq_attn_mxf8(
        pq[0].data_ptr(), pq[1].data_ptr(), pk[0].data_ptr(), pk[1].data_ptr(),
        pv[0].data_ptr(), pv[1].data_ptr(), B, H, Hkv, Sq, Skv, D, float(scale),
        int(bool(is_causal)), floor_log2(probs_quant_max), buf.data_ptr(), Sq * H * D, D, H * D,
        err.data_ptr(), _stream(dev))
    _lib.check(st, "quantized_ops::sdpa_mx (tcgen05 MXFP8 attention)")
    if CHECK_ERRORS and int(err.item()) != 0:
        raise _lib.VqError(f"sdpa_mx: device wait timed out (code {int(err.item())})")
    return buf.permute(0, 2, 1, 3)


def _masked(scores, mask):
    """``quantized.py:772-780``."""
    if mask is None:
        return scores
    if mask.dtype == torch.bool:
        return scores.masked_fill(~mask, float("-inf"))
    return scores + mask


def _composite(query, key, value, attn_mask, is_causal, query_residual, key_residual,
               value_residual, residual_mask, scale, enable_gqa, query_scale, key_scale,
               value_scale, block_size, input_code, weight_code, probs_qmap, probs_quant_max,
               probs_scale_qmap, probs_code, force_scale_power_of_two):
    """The reference's composition (``quantized.py:716-769``) on the GPU: the
    two products on this library's tcgen05 bf16 GEMM where they fit it
    (bf16, K and N multiples of 8), torch's matmul otherwise; the mask and
    the float32 softmax with torch's elementwise ops."""
    from voyager_b200.dqgemm import bmm_nt, transpose_last2
    from voyager_b200.gemm import dequantize_mx
    from voyager_b200.ops import quantize_mx

    def qk(a, b):  # a @ b^T
        out = bmm_nt(a, b)
        return out if out is not None else torch.matmul(a, b.transpose(-1, -2))

    def pv(p, v):  # p @ v
        if p.dtype == torch.bfloat16 and v.dtype == torch.bfloat16 and p.shape[-1] % 8 == 0:
            out = bmm_nt(p, transpose_last2(v.contiguous()))
            if out is not None:
                return out
        return torch.matmul(p, v)

    query = dequantize_mx(query, query_scale, input_code, block_size)
    key = dequantize_mx(key, key_scale, weight_code, block_size)
    value = dequantize_mx(value, value_scale, weight_code, block_size)
    residual = key_residual is not None
    if enable_gqa:
        group = query.shape[-3] // key.shape[-3]
        key = key.repeat_interleave(group, dim=-3)
        value = value.repeat_interleave(group, dim=-3)
        if residual:
            key_residual = key_residual.repeat_interleave(group, dim=-3)
            value_residual = value_residual.repeat_interleave(group, dim=-3)
    scores = qk(query, key) * scale
    if is_causal:
        attn_mask = torch.ones(scores.shape[-2:], dtype=torch.bool, device=scores.device).tril()
    scores = _masked(scores, attn_mask)
    keys = scores.shape[-1]
    if residual:
        rs = qk(query_residual, key_residual)
        scores = torch.cat([scores, _masked(rs * scale, residual_mask)], dim=-1)
    probs = torch.softmax(scores, dim=-1)
    probs, residual_probs = probs[..., :keys], probs[..., keys:]
    if probs_qmap is not None:
        ps, probs = quantize_mx(probs, probs_qmap, [-1], block_size, probs_quant_max,
                                force_scale_power_of_two, probs_scale_qmap, probs_code)
        probs = dequantize_mx(probs, ps, input_code, block_size)
    out = pv(probs, value)
    if residual:
        out = out + pv(residual_probs, value_residual)
    return out


def sdpa_mx(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False,
            query_residual=None, key_residual=None, value_residual=None, residual_mask=None,
            *, scale: Optional[float] = None, enable_gqa=False, query_scale=None, key_scale=None,
            value_scale=None, block_size=None, input_code=None, weight_code=None,
            probs_qmap=None, probs_quant_max=None, probs_scale_qmap=None, probs_code=None,
            force_scale_power_of_two=False):
    """``quantized.py:663-769``; ``dropout_p`` is ignored, as there."""
    if is_causal and attn_mask is not None:
        raise ValueError("is_causal excludes an explicit attn_mask")
    for t in (query, key, value):
        if not t.is_cuda:
            raise NotImplementedError("quantized_ops::sdpa_mx: the CUDA kernel needs CUDA tensors")
    if scale is None:
        scale = 1.0 / math.sqrt(query.shape[-1])
    residual = key_residual is not None
    if _fused_applies(query, key, value, attn_mask, residual, enable_gqa, query_scale, key_scale,
                      value_scale, block_size, input_code, weight_code, probs_qmap,
                      probs_scale_qmap, probs_code, force_scale_power_of_two):
        out = _fused(query, key, value, is_causal, scale, query_scale, key_scale, value_scale,
                     probs_quant_max)
        if out is not None:
            return out
    return _composite(query, key, value, attn_mask, is_causal, query_residual, key_residual,
                      value_residual, residual_mask, scale, enable_gqa, query_scale, key_scale,
                      value_scale, block_size, input_code, weight_code, probs_qmap,
                      probs_quant_max, probs_scale_qmap, probs_code, force_scale_power_of_two)
