"""The oracle at the full configuration sizes, against sha256 checksums of
the reference's own outputs on the same seeded inputs (C1, C2, C3's
activation quantize).  Also pins the synthetic input generator."""

import hashlib

import numpy as np
import pytest

import _golden as G
import oracle
from oracle.numerics import quantization_map
from voyager_b200 import synth


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


S = G.full_checksums()


def test_c1_nvfp4_round_trip():
    x = synth.c1_input()
    assert sha(x) == S["c1_input"]
    s, c = oracle.quantize_mx(x, quantization_map("fp4_e2m1"), [-1], 16, 6.0, False,
                              quantization_map("fp8_e4m3"))
    assert sha(s) == S["c1_scale"] and sha(c) == S["c1_codes"]
    assert sha(oracle.dequantize(c, s, None, [-1], 16)) == S["c1_deq"]


def test_c2_weights():
    w = synth.c2_weight()
    assert sha(w) == S["c2_input"]
    s, c = oracle.ops.quantize_mx_threaded(w, G.tables()["lut4_index"], [-1], 64, 1.0)
    assert sha(s) == S["c2_nf4_scale"] and sha(c) == S["c2_nf4_codes"]
    sp = np.array(np.abs(w).max() / np.float32(4096.0), dtype=np.float32).reshape(())
    assert sha(sp) == S["c2_posit8_scale"]
    assert sha(oracle.quantize(w, sp, qmap=quantization_map("posit8_1"))) == S["c2_posit8_codes"]
    si = (np.abs(w).max(axis=1, keepdims=True) / np.float32(127.0)).astype(np.float32)
    assert sha(si) == S["c2_int8_scale"]
    assert sha(oracle.quantize(w, si, qmap=quantization_map("int8"))) == S["c2_int8_codes"]


def test_c3_activation_quantize():
    a, w = synth.c3_operands()
    assert sha(a) == S["c3_a_input"] and sha(w) == S["c3_w_input"]
    s, c = oracle.ops.quantize_mx_threaded(a, quantization_map("fp8_e4m3"), [-1], 32, 448.0, True)
    assert sha(s) == S["c3_a_scale"] and sha(c) == S["c3_a_codes"]
