"""MXFP8 ``linear_mx`` on the tcgen05 block-scaled tensor cores.

Applies when both operands are E4M3 codes (bf16 values) with power-of-two
block-32 scales along K, blocks along the last dim of both ``input`` [.., K]
and ``weight`` [N, K] (``weight_layout="kc"``), no codebooks, bf16 everywhere
(the C3 benchmark configuration: ``fp8_e4m3,qs=microscaling,bs=32`` with
``--force_scale_power_of_two``).  The product equals the reference's
dequantize-then-matmul (``quantized.py:455-586``) up to the float32
summation order: E4M3 x 2^e values are exact in bf16, and the tensor cores
multiply them exactly and accumulate in float32.

Operands are packed to E4M3 bytes + UE8M0 scale atoms (``vq_mx_pack``).
Weights are packed once and cached per (tensor, version).  An operand whose
provenance is unknown is packed with an exactness count that is checked on
the host (one synchronisation); activations produced by this package's
``quantize_mx`` with an E4M3 table and power-of-two scales are vouched for
and skip it.
"""

import ctypes
import os

import torch

from voyager_b200 import _lib
from voyager_b200._cache import TensorCache

# codes tensors produced by quantize_mx with (E4M3 table, pow2 scales, block
# 32, last-dim blocks): (version, scale tensor id)
_vouched = TensorCache()
_wcache = TensorCache()

CHECK_ERRORS = os.environ.get("VQ_CHECK_ERRORS", "0") == "1"


def vouch(codes: torch.Tensor, scale: torch.Tensor, packed=None, axis: int = -1):
    """Record that ``codes`` / ``scale`` are exact MXFP8 (quantize_mx wrote
    them, blocks along ``axis``: -1 or -2); ``packed`` = the (E4M3 bytes,
    scale atoms) written in the same pass, if any."""
    _vouched.put(codes, "mxfp8" if axis == -1 else f"mxfp8{axis}",
                 ((codes._version, id(scale), scale._version), packed))


def _vouched_entry(codes, scale, axis: int = -1):
    v = _vouched.get(codes, "mxfp8" if axis == -1 else f"mxfp8{axis}")
    if v is None or v[0] != (codes._version, id(scale), scale._version):
        return None
    return v


def _is_vouched(codes, scale) -> bool:
    return _vouched_entry(codes, scale) is not None


def applies(input, weight, input_scale, weight_scale, block_size, input_code, weight_code,
            weight_layout, op) -> bool:
    if op != "linear" or weight_layout != "kc" or block_size != 32:
        return False
    if input_code is not None or weight_code is not None:
        return False
    if input_scale is None or weight_scale is None:
        return False
    ts = (input, weight, input_scale, weight_scale)
    if any(t.dtype != torch.bfloat16 or not t.is_cuda for t in ts):
        return False
    if weight.dim() != 2 or input.dim() < 1 or input.shape[-1] != weight.shape[1]:
        return False
    K, N = weight.shape[1], weight.shape[0]
    nkb = (K + 31) // 32
    if tuple(weight_scale.shape) != (N, nkb):
        return False
    if tuple(input_scale.shape) != tuple(input.shape[:-1]) + (nkb,):
        return False
    if N % 8 != 0 or input.numel() == 0:
        return False
    return True


def _pack(codes2d: torch.Tensor, scale2d: torch.Tensor, row_multiple: int, check: bool):
    lib = _lib.load()
    R, K = codes2d.shape
    cb, sb, ld = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    _lib.check(lib.vq_mx_pack_sizes(R, K, row_multiple, ctypes.byref(cb), ctypes.byref(sb),
                                    ctypes.byref(ld)), "mx pack sizes")
    dev = codes2d.device
    pc = torch.empty(cb.value, dtype=torch.uint8, device=dev)
    ps = torch.empty(sb.value, dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev) if check else None
    from voyager_b200.ops import _ref, _stream, _vt

    st = lib.vq_mx_pack(_ref(_vt(codes2d)), _ref(_vt(scale2d)), 32, row_multiple,
                        pc.data_ptr(), ps.data_ptr(), bad.data_ptr() if check else None,
                        _stream(dev))
    _lib.check(st, "quantized_ops::linear_mx (pack)")
    ok = True
    if check:
        ok = int(bad.item()) == 0
    return pc, ps, ok


def packed_weight(weight, weight_scale):
    key = (weight._version, id(weight_scale), weight_scale._version)
    hit = _wcache.get(weight, key)
    if hit is not None:
        return hit
    pc, ps, ok = _pack(weight.contiguous(), weight_scale.contiguous(), 256, True)
    return _wcache.put(weight, key, (pc, ps, ok))


def linear(input, weight, bias, input_scale, weight_scale, residual=None):
    """MXFP8 linear; returns None when an operand turns out not to be exact
    E4M3 / power-of-two (the caller then takes the dequantize path).  With
    ``residual`` ([.., N] bf16) the result is bf16(linear) + residual, the
    graph's residual add done in the GEMM epilogue (the same rounding)."""
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.dim() != 1
                             or bias.shape[0] != weight.shape[0] or not bias.is_cuda):
        return None
    pw, pws, wok = packed_weight(weight, weight_scale)
    if not wok:
        return None
    K, N = weight.shape[1], weight.shape[0]
    M = input.numel() // K
    entry = _vouched_entry(input, input_scale)
    if entry is not None and entry[1] is not None:
        pa, pas = entry[1]  # packed by quantize_mx in the same pass
    else:
        a2 = input.reshape(-1, K).contiguous()
        s2 = input_scale.reshape(-1, input_scale.shape[-1]).contiguous()
        pa, pas, aok = _pack(a2, s2, 128, entry is None)
        if not aok:
            return None
    out = torch.empty((M, N), dtype=torch.bfloat16, device=input.device)
    err = torch.empty(1, dtype=torch.int32, device=input.device)
    b = bias.contiguous() if bias is not None else None
    from voyager_b200.ops import _stream

    r = None
    if residual is not None:
        r = residual.reshape(M, N)
        if r.dtype != torch.bfloat16 or not r.is_contiguous():
            return None
    st = _lib.load().vq_gemm_mxf8_ex(pa.data_ptr(), pas.data_ptr(), pw.data_ptr(),
                                     pws.data_ptr(), M, N, K,
                                     b.data_ptr() if b is not None else None,
                                     r.data_ptr() if r is not None else None, N,
                                     out.data_ptr(), N, 0, err.data_ptr(),
                                     _stream(input.device))
    _lib.check(st, "quantized_ops::linear_mx (tcgen05 MXFP8)")
    if CHECK_ERRORS and int(err.item()) != 0:
        raise _lib.VqError(f"linear_mx: device wait timed out (code {int(err.item())})")
    return out.reshape(tuple(input.shape[:-1]) + (N,))


def last_error(err: torch.Tensor) -> int:
    return int(err.item())


# ---------------------------------------------------------------------------
# matmul_mx: batched MXFP8 products on the same kernels
# ---------------------------------------------------------------------------
def matmul_applies(a, b, input_scale, weight_scale, block_size, input_code, weight_code,
                   weight_layout) -> bool:
    """``matmul_mx(a, b)`` with MXFP8 operands: E4M3 codes, power-of-two
    block-32 scales along K on both (``a`` [.., M, K] blocked along its last
    dim; ``b`` [.., K, N] blocked along dim -2 for ``weight_layout="ck"``, or
    [.., N, K] blocked along its last dim for "kc"), bf16, and the leading
    dims of ``b`` equal to ``a``'s or absent."""
    if block_size != 32 or input_code is not None or weight_code is not None:
        return False
    if input_scale is None or weight_scale is None:
        return False
    ts = (a, b, input_scale, weight_scale)
    if any(t.dtype != torch.bfloat16 or not t.is_cuda for t in ts):
        return False
    if a.dim() < 2 or b.dim() < 2 or a.numel() == 0 or b.numel() == 0:
        return False
    M, K = a.shape[-2], a.shape[-1]
    nkb = (K + 31) // 32
    if weight_layout == "ck":
        if b.shape[-2] != K:
            return False
        N = b.shape[-1]
        want_sb = tuple(b.shape[:-2]) + (nkb, N)
    else:
        if b.shape[-1] != K:
            return False
        N = b.shape[-2]
        want_sb = tuple(b.shape[:-2]) + (N, nkb)
    if tuple(weight_scale.shape) != want_sb:
        return False
    if tuple(input_scale.shape) != tuple(a.shape[:-1]) + (nkb,):
        return False
    if b.dim() > 2 and tuple(b.shape[:-2]) != tuple(a.shape[:-2]):
        return False
    return N % 8 == 0


def _pack_batched(codes3, scale3, row_multiple, k_axis, check):
    lib = _lib.load()
    from voyager_b200.ops import _ref, _stream, _vt

    B = codes3.shape[0]
    R = codes3.shape[1] if k_axis == 2 else codes3.shape[2]
    K = codes3.shape[2] if k_axis == 2 else codes3.shape[1]
    rtb = (R + row_multiple - 1) // row_multiple * (row_multiple // 128)
    kt = (K + 127) // 128
    dev = codes3.device
    pc = torch.empty(B * rtb * 128 * kt * 128, dtype=torch.uint8, device=dev)
    ps = torch.empty(kt * B * rtb * 512, dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev) if check else None
    st = lib.vq_mx_pack_batched(_ref(_vt(codes3)), _ref(_vt(scale3)), 32, row_multiple, k_axis,
                                pc.data_ptr(), ps.data_ptr(), bad.data_ptr() if check else None,
                                _stream(dev))
    _lib.check(st, "quantized_ops::matmul_mx (pack)")
    ok = int(bad.item()) == 0 if check else True
    return pc, ps, rtb * 128, ok


def _shared_b(b, sb, weight_layout):
    """A 2-D right operand packed once per (tensor, version)."""
    if weight_layout == "kc":
        return packed_weight(b, sb)
    key = ("ck", b._version, id(sb), sb._version)
    hit = _wcache.get(b, key)
    if hit is not None:
        return hit
    pc, ps, _, ok = _pack_batched(b.contiguous().unsqueeze(0), sb.contiguous().unsqueeze(0), 256,
                                  1, True)
    return _wcache.put(b, key, (pc, ps, ok))


def matmul(a, b, input_scale, weight_scale, weight_layout):
    """MXFP8 matmul_mx on the tcgen05 kernels; None when an operand turns
    out not to be exact E4M3 / power-of-two (the caller then takes the
    dequantize path)."""
    batch_shape = tuple(a.shape[:-2])
    Bt = 1
    for d in batch_shape:
        Bt *= d
    M, K = a.shape[-2], a.shape[-1]
    N = b.shape[-1] if weight_layout == "ck" else b.shape[-2]
    dev = a.device
    shared = b.dim() == 2
    k_axis_b = 1 if weight_layout == "ck" else 2
    if shared:
        pb, pbs, ok = _shared_b(b, weight_scale, weight_layout)
        if not ok:
            return None
    else:
        b3 = b.reshape((Bt,) + tuple(b.shape[-2:])).contiguous()
        s3 = weight_scale.reshape((Bt,) + tuple(weight_scale.shape[-2:])).contiguous()
        pb, pbs, _, ok = _pack_batched(b3, s3, 256, k_axis_b,
                                       _vouched_entry(b, weight_scale, k_axis_b - 3) is None)
        if not ok:
            return None
    entry = _vouched_entry(a, input_scale)
    a_rows = (M + 127) // 128 * 128
    if entry is not None and entry[1] is not None and M % 128 == 0:
        pa, pas = entry[1]  # quantize_mx's own pack: the same layout when M % 128 == 0
    else:
        a3 = a.reshape(Bt, M, K).contiguous()
        sa3 = input_scale.reshape(Bt, M, input_scale.shape[-1]).contiguous()
        pa, pas, a_rows, ok = _pack_batched(a3, sa3, 128, 2, entry is None)
        if not ok:
            return None
    out = torch.empty(batch_shape + (M, N), dtype=torch.bfloat16, device=dev)
    err = torch.empty(1, dtype=torch.int32, device=dev)
    from voyager_b200.ops import _stream

    st = _lib.load().vq_gemm_mxf8_batched(pa.data_ptr(), pas.data_ptr(), pb.data_ptr(),
                                          pbs.data_ptr(), Bt, a_rows, M, N, K, int(shared), None,
                                          out.data_ptr(), N, M * N, err.data_ptr(), _stream(dev))
    _lib.check(st, "quantized_ops::matmul_mx (tcgen05 MXFP8)")
    if CHECK_ERRORS and int(err.item()) != 0:
        raise _lib.VqError(f"matmul_mx: device wait timed out (code {int(err.item())})")
    return out


# ---------------------------------------------------------------------------
# NVFP4 x NVFP4 linear_mx on tcgen05 kind::mxf4nvf4
# ---------------------------------------------------------------------------
def nvf4_applies(input, weight, input_scale, weight_scale, block_size, input_code, weight_code,
                 weight_layout, op) -> bool:
    """Both operands E2M1 codes with E4M3-valued scales per 16 along K
    (``fp4_e2m1,qs=microscaling,bs=16,ax=-1,scale=fp8_e4m3``), bf16, blocks
    along the last dim of ``input`` [.., K] and ``weight`` [N, K]."""
    if op != "linear" or weight_layout != "kc" or block_size != 16:
        return False
    if input_code is not None or weight_code is not None:
        return False
    if input_scale is None or weight_scale is None:
        return False
    ts = (input, weight, input_scale, weight_scale)
    if any(t.dtype != torch.bfloat16 or not t.is_cuda for t in ts):
        return False
    if weight.dim() != 2 or input.dim() < 1 or input.shape[-1] != weight.shape[1]:
        return False
    K, N = weight.shape[1], weight.shape[0]
    nkb = (K + 15) // 16
    if tuple(weight_scale.shape) != (N, nkb):
        return False
    if tuple(input_scale.shape) != tuple(input.shape[:-1]) + (nkb,):
        return False
    return N % 8 == 0 and input.numel() > 0


def _pack_nvf4(codes2d, scale2d, row_multiple):
    lib = _lib.load()
    from voyager_b200.ops import _ref, _stream, _vt

    R, K = codes2d.shape
    cb, sb = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(lib.vq_nvf4_pack_sizes(R, K, row_multiple, ctypes.byref(cb), ctypes.byref(sb)),
               "nvf4 pack sizes")
    dev = codes2d.device
    pc = torch.empty(cb.value, dtype=torch.uint8, device=dev)
    ps = torch.empty(sb.value, dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.vq_nvf4_pack(_ref(_vt(codes2d)), _ref(_vt(scale2d)), row_multiple,
                                pc.data_ptr(), ps.data_ptr(), bad.data_ptr(), _stream(dev)),
               "quantized_ops::linear_mx (NVFP4 pack)")
    return pc, ps, int(bad.item()) == 0


def nvf4_linear(input, weight, bias, input_scale, weight_scale):
    """NVFP4 linear; None when an operand is not exact E2M1 / E4M3 (the
    caller then takes the dequantize path)."""
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.dim() != 1
                             or bias.shape[0] != weight.shape[0] or not bias.is_cuda):
        return None
    key = ("nvf4", weight._version, id(weight_scale), weight_scale._version)
    hit = _wcache.get(weight, key)
    if hit is None:
        hit = _wcache.put(weight, key, _pack_nvf4(weight.contiguous(),
                                                  weight_scale.contiguous(), 256))
    pw, pws, wok = hit
    if not wok:
        return None
    K, N = weight.shape[1], weight.shape[0]
    M = input.numel() // K
    pa, pas, aok = _pack_nvf4(input.reshape(M, K).contiguous(),
                              input_scale.reshape(M, input_scale.shape[-1]).contiguous(), 128)
    if not aok:
        return None
    out = torch.empty((M, N), dtype=torch.bfloat16, device=input.device)
    err = torch.empty(1, dtype=torch.int32, device=input.device)
    b = bias.contiguous() if bias is not None else None
    from voyager_b200.ops import _stream

    st = _lib.load().vq_gemm_nvf4(pa.data_ptr(), pas.data_ptr(), pw.data_ptr(), pws.data_ptr(),
                                  M, N, K, b.data_ptr() if b is not None else None,
                                  out.data_ptr(), N, err.data_ptr(), _stream(input.device))
    _lib.check(st, "quantized_ops::linear_mx (tcgen05 NVFP4)")
    if CHECK_ERRORS and int(err.item()) != 0:
        raise _lib.VqError(f"linear_mx: device wait timed out (code {int(err.item())})")
    return out.reshape(tuple(input.shape[:-1]) + (N,))
