"""The oracle's quantize_mx / linear_mx / matmul_mx behind the op-call
signatures the decoder uses, on CPU torch tensors (bf16 travels as uint16
bits).  Test infrastructure: the reference-side restatement the CUDA decoder
is checked against."""

import numpy as np
import torch

import oracle
from _tt import to_dev, to_np
from oracle.numerics import quantization_map


def _np(t):
    return None if t is None else to_np(t)


def _t(a):
    return to_dev(a, "cpu")


class OracleOps:
    """CPU oracle of ``torch.ops.quantized_ops`` for the decoder (the table
    argument is ignored: the oracle builds its own E4M3 table)."""

    def __init__(self):
        self.qmap = quantization_map("fp8_e4m3")

    def table(self):
        return _t(self.qmap)

    def quantize_mx(self, x, table, axes, block_size, quant_max, pow2=False):
        s, c = oracle.quantize_mx(to_np(x), self.qmap, axes, block_size, quant_max, pow2)
        return _t(s), _t(c)

    def linear_mx(self, x, weight, bias=None, *, input_scale=None, weight_scale=None,
                  block_size=None):
        y = oracle.linear_mx(to_np(x), to_np(weight), _np(bias), input_scale=_np(input_scale),
                             weight_scale=_np(weight_scale), block_size=block_size)
        return _t(y)

    def matmul_mx(self, x, other, *, input_scale=None, weight_scale=None, block_size=None):
        y = oracle.matmul_mx(to_np(x), to_np(other), input_scale=_np(input_scale),
                             weight_scale=_np(weight_scale), block_size=block_size)
        return _t(y)

    def sdpa_mx(self, q, k, v, attn_mask=None, dropout_p=0.0, is_causal=False, *, scale=None,
                enable_gqa=False, query_scale=None, key_scale=None, value_scale=None,
                block_size=None, probs_qmap=None, probs_quant_max=None,
                force_scale_power_of_two=False):
        y = oracle.sdpa_mx(to_np(q), to_np(k), to_np(v), _np(attn_mask), dropout_p, is_causal,
                           scale=scale, enable_gqa=enable_gqa, query_scale=_np(query_scale),
                           key_scale=_np(key_scale), value_scale=_np(value_scale),
                           block_size=block_size, probs_qmap=self.qmap,
                           probs_quant_max=probs_quant_max,
                           force_scale_power_of_two=force_scale_power_of_two)
        return _t(y)


def rel_l2(got: torch.Tensor, want: torch.Tensor) -> float:
    g, w = got.double().cpu(), want.double().cpu()
    return float((g - w).norm() / w.norm())
