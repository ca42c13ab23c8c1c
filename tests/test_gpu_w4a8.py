"""W4A8 (NVFP4 weights x MXFP8 activations) against the oracle: each operand
dequantized with its own block size, float32 GEMM, rounded to bf16
(rel-L2 <= 1e-3)."""

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_dev, to_np
from oracle.numerics import quantization_map

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def _operands(m, k, n, seed):
    from voyager_b200.synth import f32_to_bf16_bits

    rng = np.random.Generator(np.random.PCG64(seed))
    a = f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    w = f32_to_bf16_bits((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    sa, ca = oracle.quantize_mx(a, quantization_map("fp8_e4m3"), [-1], 32, 448.0, True)
    sw, cw = oracle.quantize_mx(w, quantization_map("fp4_e2m1"), [-1], 16, 6.0, False,
                                quantization_map("fp8_e4m3"))
    return ca, sa, cw, sw


def _want(ca, sa, cw, sw, bias=None):
    a = oracle.dequantize_mx(ca, sa, None, 32)
    w = oracle.dequantize_mx(cw, sw, None, 16)
    out = oracle.numerics.bf16_bits_to_f32(a) @ oracle.numerics.bf16_bits_to_f32(w).T
    if bias is not None:
        out = out + oracle.numerics.bf16_bits_to_f32(bias)
    return oracle.numerics.f32_to_bf16_bits(out.astype(np.float32))


@pytest.mark.parametrize("m,k,n", [(1, 4096, 4096), (16, 4096, 4096), (5, 128, 72),
                                   (16, 14336, 512), (9, 640, 1000), (128, 512, 256)])
def test_w4a8_linear(m, k, n):
    from voyager_b200 import w4a8

    ca, sa, cw, sw = _operands(m, k, n, seed=m + k + n)
    got = to_np(w4a8.linear(to_dev(ca), to_dev(sa), to_dev(cw), to_dev(sw)))
    want = _want(ca, sa, cw, sw)
    assert got.shape == want.shape
    assert G.rel_l2(got, want) < 1e-3, G.rel_l2(got, want)
    if m <= 16:
        assert w4a8.applies_small(to_dev(ca), to_dev(cw))


def test_w4a8_bias_and_3d():
    from voyager_b200 import w4a8
    from voyager_b200.synth import f32_to_bf16_bits

    ca, sa, cw, sw = _operands(6, 256, 96, seed=3)
    bias = f32_to_bf16_bits(np.random.default_rng(0).standard_normal(96).astype(np.float32))
    got = to_np(w4a8.linear(to_dev(ca).view(2, 3, 256), to_dev(sa).view(2, 3, 8), to_dev(cw),
                            to_dev(sw), to_dev(bias)))
    assert got.shape == (2, 3, 96)
    assert G.rel_l2(got.reshape(6, 96), _want(ca, sa, cw, sw, bias)) < 1e-3


def _operands_from(a_f32, w_f32):
    from voyager_b200.synth import f32_to_bf16_bits

    a, w = f32_to_bf16_bits(a_f32.astype(np.float32)), f32_to_bf16_bits(w_f32.astype(np.float32))
    sa, ca = oracle.quantize_mx(a, quantization_map("fp8_e4m3"), [-1], 32, 448.0, True)
    sw, cw = oracle.quantize_mx(w, quantization_map("fp4_e2m1"), [-1], 16, 6.0, False,
                                quantization_map("fp8_e4m3"))
    return ca, sa, cw, sw


@pytest.mark.parametrize("m", [3, 12])
@pytest.mark.parametrize("case", ["wide_range", "zero_blocks", "tiny", "subnormal_scale",
                                  "large"])
def test_w4a8_token_scale_ranges(case, m):
    """Token block scales the kernel cannot fold into f16 token values: a
    range above 2^15 inside one CTA's K range (the first block large but
    against zero weights, so the result is the small blocks' alone and a
    rounded f16 copy of them would show), bf16-subnormal scales; and ones it
    can: zero blocks and whole zero tokens, very small and very large
    tokens."""
    from voyager_b200 import w4a8

    rng = np.random.default_rng(m * 7 + len(case))
    k, n = 1024, 520
    a = rng.standard_normal((m, k))
    w = rng.standard_normal((n, k)) * (1.0 if case == "subnormal_scale" else 0.02)
    if case == "wide_range":
        a[:, 32:] *= 2.0 ** -20
        w[:, :32] = 0.0
    elif case == "zero_blocks":
        a[:, 64:128] = 0.0
        a[1] = 0.0
    elif case == "tiny":
        a *= 2.0 ** -110
    elif case == "subnormal_scale":
        a *= 2.0 ** -121
    elif case == "large":
        a *= 2.0 ** 60
    ca, sa, cw, sw = _operands_from(a, w)
    got = to_np(w4a8.linear(to_dev(ca), to_dev(sa), to_dev(cw), to_dev(sw)))
    want = _want(ca, sa, cw, sw)
    assert G.rel_l2(got, want) < 1e-3, G.rel_l2(got, want)


def test_w4a8_calls_share_the_workspace():
    """Calls on one stream share the workspace and counters: weights of
    different shapes in turn, each call's result the oracle's as when alone
    (the counters and sums are left at zero, nothing leaks between calls;
    the float32 sums of a shared row block arrive in any order, so repeats
    agree to rounding, not bit for bit)."""
    from voyager_b200 import w4a8

    shapes = [(4, 4096, 1000), (4, 14336, 4096), (4, 640, 8)]
    ops = [tuple(to_dev(x) for x in _operands(m, k, n, seed=k + n)) for m, k, n in shapes]
    first = [to_np(w4a8.linear(*o)) for o in ops]
    for _ in range(2):
        for o, f in zip(ops, first):
            assert G.rel_l2(to_np(w4a8.linear(*o)), f) < 1e-3
    for (m, k, n), o, f in zip(shapes, ops, first):
        ca, sa, cw, sw = (to_np(x) for x in o)
        assert G.rel_l2(f, _want(ca, sa, cw, sw)) < 1e-3
