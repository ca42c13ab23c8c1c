"""W4A8 linear: NVFP4 weights x MXFP8 activations (the C4 benchmark sweep).

Weights: E2M1 codes (bf16 values) [N, K] with E4M3 scales per 16 along K
(`fp4_e2m1,qs=microscaling,bs=16,ax=-1,scale=fp8_e4m3`); activations: E4M3
codes [.., K] with power-of-two scales per 32 (`fp8_e4m3,...,bs=32` with
`--force_scale_power_of_two`).  The reference's ``linear_mx`` takes a single
block size, so this pair is not one reference call; the result is defined as
the reference computes it from the parts: each operand dequantized with its
own block size (``_dequantize_mx``, ``quantized.py:455-472``), then
``aten.linear`` with float32 accumulation, rounded to bf16.

Paths:
  * M <= 16 tokens (HBM-bound): ``vq_w4a8_linear_small`` streams the packed
    weights (0.5625 B per weight) in one launch: 16-byte loads of rows
    permuted at pack time, f16 mma.sync tiles on exact operands (weights
    times their E4M3 scales, raw E4M3 token codes), token scales on the
    float32 block sums, split-K finished by the last CTA of each row block;
  * larger M (compute-bound): the tcgen05 bf16 GEMM (``voyager_b200.dqgemm``)
    with the weight kept as 4-bit palette indices and its E4M3 block-16
    scales, read back in shared memory (code x scale, exact in bf16), and
    the activations read back by the dequantize kernel.
"""

import ctypes

import torch
import torch.nn.functional as F

from voyager_b200 import _lib
from voyager_b200 import ops as _ops
from voyager_b200._cache import TensorCache

SMALL_M = 16
_wpack = TensorCache()
_wdeq = TensorCache()
_wwork = TensorCache()


def _packed_weight(w_codes, w_scale):
    key = (w_codes._version, id(w_scale), w_scale._version)
    hit = _wpack.get(w_codes, key)
    if hit is not None:
        return hit
    N, K = w_codes.shape
    dev = w_codes.device
    wq = torch.empty(N * K // 2, dtype=torch.uint8, device=dev)
    ws = torch.empty(N * K // 16, dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    st = _lib.load().vq_w4_pack_weights(_ops._ref(_ops._vt(w_codes.contiguous())),
                                        _ops._ref(_ops._vt(w_scale.contiguous())),
                                        wq.data_ptr(), ws.data_ptr(), bad.data_ptr(),
                                        _ops._stream(dev))
    _lib.check(st, "w4a8 weight pack")
    ok = int(bad.item()) == 0
    return _wpack.put(w_codes, key, (wq, ws, ok))


def _exact_tokens(a_codes, a_scale, a2, s2) -> bool:
    """The kernel takes the token codes as E4M3 values and their scales as
    powers of two (then every product is the reference's bf16 value):
    vouched for when this package's quantize_mx made them, else checked (one
    host synchronisation)."""
    from voyager_b200 import mxgemm

    if mxgemm._vouched_entry(a_codes, a_scale) is not None:
        return True
    return mxgemm._pack(a2, s2, 128, True)[2]


def _workspace(w_codes, N):
    """The self-cleaning split-K workspace of one weight: float32 [16 * N]
    and the row-block counters, zero when made and left zero by each call."""
    hit = _wwork.get(w_codes, "ws")
    if hit is None:
        dev = w_codes.device
        hit = _wwork.put(w_codes, "ws", (torch.zeros(16 * N, dtype=torch.float32, device=dev),
                                         torch.zeros((N + 255) // 256, dtype=torch.int32,
                                                     device=dev)))
    return hit


def _dequant_weight(w_codes, w_scale):
    key = (w_codes._version, id(w_scale), w_scale._version)
    hit = _wdeq.get(w_codes, key)
    if hit is not None:
        return hit
    return _wdeq.put(w_codes, key, _ops.dequantize(w_codes, w_scale, None, None, 16))


def applies_small(a_codes, w_codes) -> bool:
    K = w_codes.shape[1]
    M = a_codes.numel() // K
    return 0 < M <= SMALL_M and K % 128 == 0


def linear(a_codes: torch.Tensor, a_scale: torch.Tensor, w_codes: torch.Tensor,
           w_scale: torch.Tensor, bias=None) -> torch.Tensor:
    """``[.., K] x [N, K]^T -> [.., N]`` (bf16)."""
    for t in (a_codes, a_scale, w_codes, w_scale):
        if t.dtype != torch.bfloat16 or not t.is_cuda:
            raise NotImplementedError("w4a8.linear takes bf16 CUDA tensors")
    N, K = w_codes.shape
    if a_codes.shape[-1] != K or tuple(w_scale.shape) != (N, K // 16):
        raise ValueError("w4a8.linear: shapes do not match NVFP4 weights [N, K] / [N, K/16]")
    lead = a_codes.shape[:-1]
    M = a_codes.numel() // K
    dev = a_codes.device
    if applies_small(a_codes, w_codes):
        wq, ws, wok = _packed_weight(w_codes, w_scale)
        a2 = a_codes.reshape(M, K).contiguous()
        s2 = a_scale.reshape(M, K // 32).contiguous()
        if wok and _exact_tokens(a_codes, a_scale, a2, s2):
            acc, done = _workspace(w_codes, N)
            out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            b = bias.contiguous() if bias is not None else None
            _lib.check(_lib.load().vq_w4a8_linear_small(
                _ops._ref(_ops._vt(a2)), _ops._ref(_ops._vt(s2)), wq.data_ptr(), ws.data_ptr(),
                N, b.data_ptr() if b is not None else None, ctypes.c_void_p(acc.data_ptr()),
                ctypes.c_void_p(done.data_ptr()), out.data_ptr(), _ops._stream(dev)),
                "w4a8 linear")
            return out.reshape(tuple(lead) + (N,))
    from voyager_b200 import dqgemm

    a = _ops.dequantize(a_codes, a_scale, None, None, 32)
    pw = dqgemm.packed_weight(w_codes, w_scale, None, 16, "kc")
    if pw is not None and K % 8 == 0 and (bias is None or bias.dtype == torch.bfloat16):
        a2 = a.reshape(M, K)
        return dqgemm.gemm(a2 if a2.is_contiguous() else a2.contiguous(), pw,
                           bias).reshape(tuple(lead) + (N,))
    w = _dequant_weight(w_codes, w_scale)
    return F.linear(a, w, bias)
