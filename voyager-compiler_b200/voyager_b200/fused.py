"""Decoder-graph fusions around MXFP8 ``quantize_mx`` (``vq_fused.cu``).

Each function computes the bf16 ops a converted LLaMA layer runs in front of
one ``quantize_mx(x, E4M3 table, [-1], 32, quant_max, True)`` and quantizes
in the same pass.  It returns what that ``quantize_mx`` returns -- ``(scale,
codes)`` -- with the tcgen05 operand (E4M3 bytes + scale atoms) recorded on
the codes, so the ``linear_mx`` / ``sdpa_mx`` that consume them read the
operand directly.

  rmsnorm_quantize_mx   RMSNorm -> quantize_mx          (both layer norms)
  rope_quantize_qk      RoPE of q and k -> quantize_mx  (blocks along head_dim)
  quantize_vt           v -> quantize_mx of v^T          (blocks along tokens)
  swiglu_quantize_mx    silu(gate) * up -> quantize_mx  (the MLP activation)
"""

import torch

from voyager_b200 import _lib, mxgemm
from voyager_b200.ops import _stream, floor_log2
from voyager_b200.tables import rounder_for


def _e4m3(table, dev):
    rd = rounder_for(table, dev)
    if rd.c.kind != _lib.VQ_R_MINIFLOAT or rd.c.hw != 1:
        raise ValueError("the fused quantizations take an E4M3 table (hardware rounder)")
    return rd


def _outputs(rows: int, cols: int, shape, dev):
    """codes, scale (quantize_mx's outputs, `shape` = the codes' shape) and
    the packed operand of a [rows, cols] view (cols padded to 128)."""
    rt = (rows + 127) // 128
    cp = (cols + 127) // 128 * 128
    codes = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    scale = torch.empty(tuple(shape[:-1]) + (shape[-1] // 32,), dtype=torch.bfloat16, device=dev)
    packed = torch.empty(rt * 128 * cp, dtype=torch.uint8, device=dev)
    packed_sf = torch.empty((cp // 128) * rt * 512, dtype=torch.uint8, device=dev)
    return codes, scale, packed, packed_sf


def _finish(codes, scale, packed, packed_sf):
    mxgemm.vouch(codes, scale, (packed, packed_sf))
    return scale, codes


def rmsnorm_quantize_mx(x: torch.Tensor, weight: torch.Tensor, eps: float, table,
                        quant_max: float = 448.0):
    """quantize_mx(weight * bf16(rms_norm(x)), table, [-1], 32, quant_max, True)."""
    assert x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
    x = x.contiguous()
    C = x.shape[-1]
    R = x.numel() // C
    dev = x.device
    out = _outputs(R, C, x.shape, dev)
    rd = _e4m3(table, dev)
    st = _lib.load().vq_rmsnorm_quantize_mx(
        x.data_ptr(), weight.contiguous().data_ptr(), R, C, float(eps), rd.ref(),
        floor_log2(quant_max), *[t.data_ptr() for t in out], _stream(dev))
    _lib.check(st, "rmsnorm + quantize_mx")
    return _finish(*out)


def rope_quantize_qk(qkv: torch.Tensor, q_off: int, k_off: int, cos: torch.Tensor,
                     sin: torch.Tensor, batch: int, seq: int, heads: int, table,
                     quant_max: float = 448.0):
    """RoPE'd q and k heads of qkv [batch*seq, ld], each through quantize_mx
    along head_dim: ((sq, cq), (sk, ck)), codes [batch, heads, seq, 128]."""
    assert qkv.dtype == torch.bfloat16 and qkv.dim() == 2 and qkv.stride(1) == 1
    dev = qkv.device
    rows = batch * heads * seq
    oq = _outputs(rows, 128, (batch, heads, seq, 128), dev)
    ok = _outputs(rows, 128, (batch, heads, seq, 128), dev)
    rd = _e4m3(table, dev)
    st = _lib.load().vq_rope_quantize_qk(
        qkv.data_ptr(), qkv.stride(0), q_off, k_off, cos.contiguous().data_ptr(),
        sin.contiguous().data_ptr(), batch, seq, heads, rd.ref(), floor_log2(quant_max),
        *[t.data_ptr() for t in oq], *[t.data_ptr() for t in ok], _stream(dev))
    _lib.check(st, "rope + quantize_mx")
    return _finish(*oq), _finish(*ok)


def quantize_vt(qkv: torch.Tensor, v_off: int, batch: int, seq: int, heads: int, table,
                quant_max: float = 448.0):
    """v^T of the v heads of qkv through quantize_mx along the tokens:
    (scale [batch, heads, 128, seq/32], codes [batch, heads, 128, seq])."""
    assert qkv.dtype == torch.bfloat16 and qkv.dim() == 2 and qkv.stride(1) == 1
    dev = qkv.device
    out = _outputs(batch * heads * 128, seq, (batch, heads, 128, seq), dev)
    rd = _e4m3(table, dev)
    st = _lib.load().vq_quantize_vt(qkv.data_ptr(), qkv.stride(0), v_off, batch, seq, heads,
                                    rd.ref(), floor_log2(quant_max),
                                    *[t.data_ptr() for t in out], _stream(dev))
    _lib.check(st, "quantize_mx of v^T")
    return _finish(*out)


def swiglu_quantize_mx(gate_up: torch.Tensor, cols: int, table, quant_max: float = 448.0,
                       up_off: int = None):
    """quantize_mx(bf16(silu(gate)) * up) for gate = gate_up[:, :cols], up =
    gate_up[:, up_off:up_off + cols] (default up_off = cols)."""
    assert gate_up.dtype == torch.bfloat16 and gate_up.dim() == 2 and gate_up.stride(1) == 1
    dev = gate_up.device
    R = gate_up.shape[0]
    up_off = cols if up_off is None else up_off
    out = _outputs(R, cols, (R, cols), dev)
    rd = _e4m3(table, dev)
    st = _lib.load().vq_swiglu_quantize_mx(gate_up.data_ptr(), gate_up.stride(0), up_off, R,
                                           cols, rd.ref(), floor_log2(quant_max),
                                           *[t.data_ptr() for t in out], _stream(dev))
    _lib.check(st, "swiglu + quantize_mx")
    return _finish(*out)
