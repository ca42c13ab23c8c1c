"""``linear_mx`` / ``matmul_mx`` for every format but MXFP8 x MXFP8, on the
tcgen05 bf16 GEMM of this library (``vq_gemm_dq``).

The reference reads each operand back with ``_dequantize_mx``
(``src/voyager_compiler/ops/quantized.py:455-472``: codebook ``decode``, then
``* expand(scale)`` in the operand's dtype) and multiplies with
``aten.linear`` / ``aten.matmul``.  Here:

  * a 2-D weight whose codes take at most 256 distinct bf16 values (every
    posit8 / int8 / NormalFloat / E2M1 / E4M3 / codebook weight) is packed
    once into palette indices -- 4-bit for at most 16 values, 8-bit else --
    with its bf16 block scales, and the GEMM kernel reads it back inside
    shared memory: palette lookup, then the bf16 product with the scale
    (one rounding of the exact product, as the reference's bf16 multiply);
  * any other bf16 operand (more than 256 values, scales of another dtype
    or layout, both operands of an activation matmul) is read back by this
    library's dequantize kernels and multiplied by the same kernel with the
    weight loaded by TMA;
  * the activations are read back by the dequantize kernels (when they have
    a scale or a codebook) and loaded by TMA.

Float32 and float16 operands have no path here (the kernel multiplies bf16);
callers keep the reference composition for them.
"""

import ctypes
import os
from typing import Optional

import numpy as np
import torch

from voyager_b200 import _lib
from voyager_b200._cache import TensorCache

MODE_TMA, MODE_LUT4, MODE_LUT8 = 0, 1, 2
KSTEP = 64
# split the K steps of few-tile GEMMs over more CTA pairs (VQ_DQ_SPLITK=0: never)
SPLIT_K = os.environ.get("VQ_DQ_SPLITK", "1") != "0"
# from this many activation rows on, a packed weight is decoded once per call
# into a bf16 copy (N * K * 2 bytes of scratch) multiplied by the TMA-mode
# kernel: the in-kernel decode repeats for every 256-row tile of the
# activations and is what bounds that kernel at large M (0 or less: never)
DECODE_ONCE_M = int(os.environ.get("VQ_DQ_DECODE_ONCE_M", "4096"))
_wcache = TensorCache()


def _ops():
    from voyager_b200 import ops

    return ops


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


class PackedWeight:
    """A weight [N, K] in the kernel's form: ``mode``; ``w`` (step-major
    palette indices, or the bf16 weight for MODE_TMA); ``scale4`` the
    quarter-step bf16 scales or None; ``palette`` bf16 [16 | 256]."""

    def __init__(self, mode, w, N, K, scale4=None, palette=None):
        self.mode, self.w, self.N, self.K = mode, w, N, K
        self.scale4, self.palette = scale4, palette


def _scale_form(weight_scale, N, K, block_size):
    """(scale [N, nkb] bf16, nkb, block size) as the kernel reads it, or None
    when the scale is not bf16 blocks along K of each row."""
    if weight_scale is None:
        return None, 1, 0
    s = weight_scale
    if s.dtype != torch.bfloat16:
        return None
    if s.dim() == 0 or (s.dim() == 2 and tuple(s.shape) == (1, 1)):
        # one scale for the tensor: the same for every row
        return s.reshape(1, 1).expand(N, 1).contiguous(), 1, 0
    if s.dim() != 2 or s.shape[0] != N:
        return None
    nkb = s.shape[1]
    if nkb == 1:
        if block_size is not None and block_size < K:
            return None  # the reference's expand() would not reach K columns
        return s.contiguous(), 1, 0
    if block_size is None or block_size < 16 or block_size & (block_size - 1):
        return None
    if (K + block_size - 1) // block_size != nkb:
        return None
    return s.contiguous(), nkb, block_size


def _palette_of(codes2d):
    """(keys, key_index, palette): the distinct bf16 bit patterns of
    ``codes2d`` (ascending), each key's palette position, and the palette;
    None when more than 256 values remain.  With 257 patterns, -0 shares
    +0's entry (int8 codes span -128..127 and both zeros): the product is a
    zero either way, so the GEMM's sums do not change."""
    lib = _lib.load()
    ops = _ops()
    dev = codes2d.device
    present = torch.empty(65536, dtype=torch.uint8, device=dev)
    _lib.check(lib.vq_dq_patterns(ops._ref(ops._vt(codes2d)), present.data_ptr(), _stream(dev)),
               "linear_mx (weight patterns)")
    pats = np.nonzero(present.cpu().numpy())[0].astype(np.uint16)  # one-time, per weight
    key_index = np.arange(len(pats))
    palette = pats
    if len(pats) > 256 and 0x8000 in pats and 0 in pats:
        palette = pats[pats != 0x8000]
        key_index = np.searchsorted(palette, pats)
        key_index[pats == 0x8000] = int(np.searchsorted(palette, 0))
    if len(palette) > 256:
        return None
    return pats, key_index.astype(np.uint8), palette


def pack(codes2d: torch.Tensor, weight_scale, weight_code, block_size) -> Optional[PackedWeight]:
    """Pack a bf16 weight [N, K] (codes) for the in-kernel decode; None when
    it does not fit the form (then the caller reads it back in HBM)."""
    lib = _lib.load()
    ops = _ops()
    N, K = codes2d.shape
    dev = codes2d.device
    if K % 8 or N % 8:
        return None
    sf = _scale_form(weight_scale, N, K, block_size)
    if sf is None:
        return None
    scale, nkb, bs = sf
    if weight_code is not None:
        if weight_code.dim() != 1 or weight_code.numel() > 256 or weight_code.numel() == 0:
            return None
        # decode() reads codebook[index] and casts it to the codes' dtype
        entries = weight_code.to(device=dev).to(torch.bfloat16)
        P = entries.numel()
        mode = MODE_LUT4 if P <= 16 else MODE_LUT8
        pal = torch.zeros(16 if mode == MODE_LUT4 else 256, dtype=torch.bfloat16, device=dev)
        pal[:P] = entries
        keys = key_index = None
        index_mode = 1
    else:
        found = _palette_of(codes2d)
        if found is None:
            return None
        pats, kidx, palette = found
        P = len(palette)
        mode = MODE_LUT4 if P <= 16 else MODE_LUT8
        size = 16 if mode == MODE_LUT4 else 256
        pal_np = np.zeros(size, dtype=np.uint16)
        pal_np[:P] = palette
        pal = torch.from_numpy(pal_np.view(np.int16)).to(dev).view(torch.bfloat16)
        keys = torch.from_numpy(pats.view(np.int16)).to(dev)
        key_index = torch.from_numpy(kidx).to(dev)
        P = len(pats)  # keys searched by the pack kernel
        index_mode = 0
    cb, sb = ctypes.c_int64(), ctypes.c_int64()
    _lib.check(lib.vq_dq_pack_sizes(1, N, K, mode, ctypes.byref(cb), ctypes.byref(sb)),
               "linear_mx (pack sizes)")
    wq = torch.empty(cb.value, dtype=torch.uint8, device=dev)
    missing = torch.zeros(1, dtype=torch.int32, device=dev)
    st = lib.vq_dq_pack(ops._ref(ops._vt(codes2d)), 1, mode, index_mode,
                        keys.data_ptr() if keys is not None else None,
                        key_index.data_ptr() if key_index is not None else None, P,
                        wq.data_ptr(), missing.data_ptr(), _stream(dev))
    _lib.check(st, "linear_mx (weight pack)")
    scale4 = None
    if scale is not None:
        scale4 = torch.empty(sb.value // 2, dtype=torch.bfloat16, device=dev)
        _lib.check(lib.vq_dq_pack_scales(scale.data_ptr(), 1, N, K, nkb, bs, scale4.data_ptr(),
                                         _stream(dev)), "linear_mx (scale pack)")
    if int(missing.item()) != 0:  # codes that are not indices of the codebook
        return None
    return PackedWeight(mode, wq, N, K, scale4, pal)


def _kc_weight(weight, weight_scale, weight_layout):
    """The weight's codes and scale as [N, K] / [N, nkb] (a CK-stored weight
    transposed once)."""
    if weight_layout == "kc":
        return weight.contiguous(), weight_scale
    w = transpose_last2(weight.contiguous())
    s = weight_scale
    if s is not None and s.dim() == 2 and s.shape[1] == weight.shape[1] \
            and s.dtype == torch.bfloat16:
        s = transpose_last2(s.contiguous())  # [nkb, N] blocks along K -> [N, nkb]
    return w, s


def packed_weight(weight, weight_scale, weight_code, block_size, weight_layout):
    """The kernel form of a 2-D weight, cached per (tensor, version)."""
    key = ("dq", weight._version, weight_layout, block_size,
           None if weight_scale is None else (id(weight_scale), weight_scale._version),
           None if weight_code is None else (id(weight_code), weight_code._version))
    hit = _wcache.get(weight, key)
    if hit is not None:
        return hit or None  # False: known not to fit either form
    w, s = _kc_weight(weight, weight_scale, weight_layout)
    pw = pack(w, s, weight_code, block_size)
    if pw is None:
        # read back in HBM by the dequantize kernels; the GEMM loads it by TMA
        from voyager_b200.gemm import dequantize_mx

        wd = dequantize_mx(weight, weight_scale, weight_code, block_size)
        if wd.dtype != torch.bfloat16:
            _wcache.put(weight, key, False)
            return None
        if weight_layout == "ck":
            wd = transpose_last2(wd.contiguous())
        pw = PackedWeight(MODE_TMA, wd.contiguous(), wd.shape[0], wd.shape[1])
        if pw.K % 8 or pw.N % 8:
            _wcache.put(weight, key, False)
            return None
    return _wcache.put(weight, key, pw)


def transpose_last2(x: torch.Tensor) -> torch.Tensor:
    """[.., R, C] -> [.., C, R] (bf16) with the library's transpose kernel."""
    if x.dtype != torch.bfloat16:
        raise NotImplementedError("transpose_last2 takes bf16")
    R, C = x.shape[-2], x.shape[-1]
    B = x.numel() // max(1, R * C)
    out = torch.empty(tuple(x.shape[:-2]) + (C, R), dtype=x.dtype, device=x.device)
    if x.numel():
        _lib.check(_lib.load().vq_transpose_bf16(x.data_ptr(), B, R, C, out.data_ptr(),
                                                 _stream(x.device)), "transpose")
    return out


def gemm(a2: torch.Tensor, pw: PackedWeight, bias=None, batch=1, w_shared=True, splits=None):
    """out [batch, M, N] bf16 = a2 [batch * M, K] . W^T (+ bias) on the kernel;
    ``splits`` K slices per output tile (None: the library's choice)."""
    dev = a2.device
    K = a2.shape[-1]
    M = a2.shape[0] // batch
    if (pw.mode != MODE_TMA and DECODE_ONCE_M > 0 and batch * M >= DECODE_ONCE_M
            and (batch == 1 or w_shared)):
        pw = PackedWeight(MODE_TMA, decode(pw), pw.N, pw.K)
    out = torch.empty((batch, M, pw.N), dtype=torch.bfloat16, device=dev)
    err = torch.empty(1, dtype=torch.int32, device=dev)
    b = bias.contiguous() if bias is not None else None
    lib = _lib.load()
    # few output tiles (small M and N): the K steps split over more CTA pairs
    if splits is None:
        splits = int(lib.vq_gemm_dq_splits(batch, M, pw.N, K)) if SPLIT_K else 1
    ws = (torch.empty(splits * M * pw.N, dtype=torch.float32, device=dev) if splits > 1
          else None)
    st = lib.vq_gemm_dq_ex(a2.data_ptr(), batch, M, K, pw.mode, pw.w.data_ptr(),
                           int(bool(w_shared)), pw.N,
                           pw.scale4.data_ptr() if pw.scale4 is not None else None,
                           pw.palette.data_ptr() if pw.palette is not None else None,
                           b.data_ptr() if b is not None else None, out.data_ptr(), pw.N,
                           M * pw.N, splits, ws.data_ptr() if ws is not None else None,
                           err.data_ptr(), _stream(dev))
    _lib.check(st, "quantized_ops::linear_mx (tcgen05 bf16)")
    from voyager_b200 import mxgemm

    if mxgemm.CHECK_ERRORS and int(err.item()) != 0:
        raise _lib.VqError(f"linear_mx: device wait timed out (code {int(err.item())})")
    return out


def _bf16_operand(x):
    return x.dtype == torch.bfloat16 and x.is_cuda


def linear(input, weight, bias, input_scale, weight_scale, block_size, input_code, weight_code,
           weight_layout):
    """linear_mx on the bf16 kernel, or None when the operands are not bf16
    (the caller then keeps the reference composition)."""
    from voyager_b200.gemm import dequantize_mx

    if weight.dim() != 2 or not _bf16_operand(weight) or not _bf16_operand(input):
        return None
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.dim() != 1):
        return None
    a = dequantize_mx(input, input_scale, input_code, block_size)
    if a.dtype != torch.bfloat16 or a.numel() == 0:
        return None
    K = a.shape[-1]
    pw = packed_weight(weight, weight_scale, weight_code, block_size, weight_layout)
    if pw is None or pw.K != K or K % 8:
        return None
    if bias is not None and bias.shape[0] != pw.N:
        return None
    a2 = a.reshape(-1, K)
    if not a2.is_contiguous() or a2.data_ptr() % 16:
        a2 = a2.contiguous()
    out = gemm(a2, pw, bias)
    return out.reshape(tuple(a.shape[:-1]) + (pw.N,))


def matmul(self, other, input_scale, weight_scale, block_size, input_code, weight_code,
           weight_layout):
    """matmul_mx on the bf16 kernel (operands read back by the dequantize
    kernels), or None when they are not bf16 or their batch dims differ."""
    from voyager_b200.gemm import dequantize_mx

    if not _bf16_operand(self) or not _bf16_operand(other) or self.dim() < 2 or other.dim() < 2:
        return None
    if other.dim() == 2:
        # a shared right operand: the weight path (packed once)
        return linear(self, other, None, input_scale, weight_scale, block_size, input_code,
                      weight_code, weight_layout)
    a = dequantize_mx(self, input_scale, input_code, block_size)
    b = dequantize_mx(other, weight_scale, weight_code, block_size)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        return None
    batch_shape = tuple(a.shape[:-2])
    if b.dim() > 2 and tuple(b.shape[:-2]) != batch_shape:
        return None
    M, K = a.shape[-2], a.shape[-1]
    shared = b.dim() == 2
    bt = transpose_last2(b.contiguous()) if weight_layout == "ck" else b.contiguous()
    N = bt.shape[-2]
    if bt.shape[-1] != K or K % 8 or N % 8 or a.numel() == 0:
        return None
    Bt = 1
    for d in batch_shape:
        Bt *= d
    pw = PackedWeight(MODE_TMA, bt, N, K)
    out = gemm(a.reshape(Bt * M, K).contiguous(), pw, None, batch=Bt, w_shared=shared)
    return out.reshape(batch_shape + (M, N))


def decode(pw: PackedWeight) -> torch.Tensor:
    """The weight as the GEMM kernel reads it back (tests: bf16 [N, K])."""
    out = torch.empty((pw.N, pw.K), dtype=torch.bfloat16, device=pw.w.device)
    st = _lib.load().vq_dq_decode(pw.w.data_ptr(), pw.N, pw.K, pw.mode,
                                  pw.scale4.data_ptr() if pw.scale4 is not None else None,
                                  pw.palette.data_ptr(), out.data_ptr(), _stream(pw.w.device))
    _lib.check(st, "dq decode")
    return out


def bmm_nt(a: torch.Tensor, b: torch.Tensor) -> Optional[torch.Tensor]:
    """a [.., M, K] @ b[.., N, K]^T -> [.., M, N] bf16 on the tcgen05 bf16 GEMM
    (float32 sums, one bf16 rounding), b's leading dims equal to a's or
    absent; None when the operands do not fit it (not bf16, K or N not a
    multiple of 8, empty)."""
    if not (_bf16_operand(a) and _bf16_operand(b)) or a.dim() < 2 or b.dim() < 2:
        return None
    M, K = a.shape[-2], a.shape[-1]
    N = b.shape[-2]
    if b.shape[-1] != K or K % 8 or N % 8 or a.numel() == 0 or b.numel() == 0:
        return None
    batch_shape = tuple(a.shape[:-2])
    if b.dim() > 2 and tuple(b.shape[:-2]) != batch_shape:
        return None
    Bt = 1
    for d in batch_shape:
        Bt *= d
    pw = PackedWeight(MODE_TMA, b.contiguous(), N, K)
    out = gemm(a.reshape(Bt * M, K).contiguous(), pw, None, batch=Bt, w_shared=b.dim() == 2)
    return out.reshape(batch_shape + (M, N))
