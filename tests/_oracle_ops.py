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


def rel_l2(got: torch.Tensor, want: torch.Tensor) -> float:
    g, w = got.double().cpu(), want.double().cpu()
    return float((g - w).norm() / w.norm())
