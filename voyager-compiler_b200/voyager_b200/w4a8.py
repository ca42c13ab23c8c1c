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
    weights (0.5625 B per weight, 18 KB tiles of 256 rows x 128 K) in one
    launch: a persistent grid whose CTAs each take an equal run of tiles,
    bulk copies into a shared-memory ring, f16 mma.sync tiles on exact
    operands (weights times their E4M3 scales, token codes times their
    power-of-two scales relative to the token's largest), row blocks split
    between CTAs summed from float32 pieces by the CTA that adds the last;
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
_wspace = {}


def _packed_weight(w_codes, w_scale):
    key = (w_codes._version, id(w_scale), w_scale._version)
    hit = _wpack.get(w_codes, key)
    if hit is not None:
        return hit
    N, K = w_codes.shape
    dev = w_codes.device
    lib = _lib.load()
    wt = torch.empty(lib.vq_w4_packed_bytes(N, K), dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    st = lib.vq_w4_pack_weights(_ops._ref(_ops._vt(w_codes.contiguous())),
                                _ops._ref(_ops._vt(w_scale.contiguous())), wt.data_ptr(),
                                bad.data_ptr(), _ops._stream(dev))
    _lib.check(st, "w4a8 weight pack")
    ok = int(bad.item()) == 0
    return _wpack.put(w_codes, key, (wt, ok))


def _exact_tokens(a_codes, a_scale, a2, s2) -> bool:
    """The kernel takes the token codes as E4M3 values and their scales as
    powers of two (then every product is the reference's bf16 value):
    vouched for when this package's quantize_mx made them, else checked (one
    host synchronisation)."""
    from voyager_b200 import mxgemm

    if mxgemm._vouched_entry(a_codes, a_scale) is not None:
        return True
    return mxgemm._pack(a2, s2, 128, True)[2]


def _workspace(dev, N, K):
    """The workspace of the calls on the current stream: the float32 sums of
    row blocks split between CTAs and the row-block counters, zero when
    made and left zero by each call.  Calls on one stream never overlap, so
    they share one pair, grown to the largest weight."""
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    need = (_lib.load().vq_w4a8_workspace_bytes(N, K) // 4, (N + 255) // 256)
    hit = _wspace.get(key)
    if hit is None or hit[0].numel() < need[0] or hit[1].numel() < need[1]:
        have = (hit[0].numel(), hit[1].numel()) if hit is not None else (0, 0)
        hit = (torch.zeros(max(need[0], have[0]), dtype=torch.float32, device=dev),
               torch.zeros(max(need[1], have[1]), dtype=torch.int32, device=dev))
        _wspace[key] = hit
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
        wt, wok = _packed_weight(w_codes, w_scale)
        a2 = a_codes.reshape(M, K).contiguous()
        s2 = a_scale.reshape(M, K // 32).contiguous()
        if wok and _exact_tokens(a_codes, a_scale, a2, s2):
            from voyager_b200 import mxgemm

            part, done = _workspace(dev, N, K)
            out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
            # the per-call error word costs a memset between consecutive
            # calls (no overlap of one call's start with the previous one's
            # end): only when checking; the sticky device word always records
            err = (torch.empty(1, dtype=torch.int32, device=dev) if mxgemm.CHECK_ERRORS
                   else None)
            b = bias.contiguous() if bias is not None else None
            _lib.check(_lib.load().vq_w4a8_linear_small(
                _ops._ref(_ops._vt(a2)), _ops._ref(_ops._vt(s2)), wt.data_ptr(), N,
                b.data_ptr() if b is not None else None, ctypes.c_void_p(part.data_ptr()),
                ctypes.c_void_p(done.data_ptr()), err.data_ptr() if err is not None else None,
                out.data_ptr(), _ops._stream(dev)), "w4a8 linear")
            if err is not None and int(err.item()) != 0:
                raise _lib.VqError(f"w4a8 linear: device wait timed out (code {int(err.item())})")
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
