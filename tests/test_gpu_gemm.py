"""tcgen05 MXFP8 linear_mx against the oracle's dequantize-then-matmul.

Tolerance: rel-L2 <= 1e-3 against the oracle GEMM rounded to the output
dtype (bf16), as the reference's bf16 linear rounds it; the only difference
is the float32 summation order."""

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
    qm = quantization_map("fp8_e4m3")
    sa, ca = oracle.quantize_mx(a, qm, [-1], 32, 448.0, True)
    sw, cw = oracle.quantize_mx(w, qm, [-1], 32, 448.0, True)
    return ca, sa, cw, sw


def _run(ca, sa, cw, sw, bias=None):
    from voyager_b200 import mxgemm

    dca, dsa, dcw, dsw = to_dev(ca), to_dev(sa), to_dev(cw), to_dev(sw)
    assert mxgemm.applies(dca, dcw, dsa, dsw, 32, None, None, "kc", "linear")
    out = mxgemm.linear(dca, dcw, None if bias is None else to_dev(bias), dsa, dsw)
    assert out is not None, "operands were not accepted as exact MXFP8"
    torch.cuda.synchronize()
    return to_np(out)


# M >= 256 takes the CTA-pair kernel (256-row tiles; an odd number of
# 128-row chunks leaves the second CTA of the last pair on padding rows)
SHAPES = [(128, 128, 256), (1, 128, 8), (130, 256, 264), (256, 512, 512), (96, 96, 40),
          (300, 4096, 11008), (1024, 4096, 4096), (520, 640, 1000)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_mxf8_linear(m, k, n):
    ca, sa, cw, sw = _operands(m, k, n, seed=m * 7 + k + n)
    got = _run(ca, sa, cw, sw)
    want = oracle.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    assert got.shape == want.shape and got.dtype == want.dtype
    assert G.rel_l2(got, want) < 1e-3, G.rel_l2(got, want)


def test_mxf8_linear_bias_and_op():
    from voyager_b200.synth import f32_to_bf16_bits

    ca, sa, cw, sw = _operands(200, 384, 136, seed=5)
    bias = f32_to_bf16_bits(np.random.default_rng(1).standard_normal(136).astype(np.float32))
    got = _run(ca, sa, cw, sw, bias)
    want = oracle.linear_mx(ca, cw, bias, input_scale=sa, weight_scale=sw, block_size=32)
    assert G.rel_l2(got, want) < 1e-3
    # through the op (dispatches to the same kernel)
    Q = torch.ops.quantized_ops
    got2 = to_np(Q.linear_mx(to_dev(ca), to_dev(cw), to_dev(bias), input_scale=to_dev(sa),
                             weight_scale=to_dev(sw), block_size=32))
    assert G.rel_l2(got2, want) < 1e-3


def test_mxf8_rejects_non_e4m3_codes():
    """Codes that are not E4M3 values are detected by the pack check and the
    op falls back to dequantize + matmul (still matching the oracle)."""
    from voyager_b200 import mxgemm

    ca, sa, cw, sw = _operands(64, 128, 64, seed=9)
    cw = cw.copy()
    cw[0, 0] = 0x3F81  # 1.0078125: not an E4M3 value
    out = mxgemm.linear(to_dev(ca), to_dev(cw), None, to_dev(sa), to_dev(sw))
    assert out is None
    want = oracle.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    got = to_np(torch.ops.quantized_ops.linear_mx(to_dev(ca), to_dev(cw), None,
                                                   input_scale=to_dev(sa),
                                                   weight_scale=to_dev(sw), block_size=32))
    assert G.rel_l2(got, want) < 1e-3


def test_c3_full_size_rows_sample():
    """C3 at full size (M=8192, K=4096, N=11008) through quantize_mx and
    linear_mx; checked on a 256-row sample against the oracle."""
    from voyager_b200 import synth

    a, w = synth.c3_operands()
    Q = torch.ops.quantized_ops
    e4m3 = to_dev(quantization_map("fp8_e4m3"))
    sa, ca = Q.quantize_mx(to_dev(a), e4m3, [-1], 32, 448.0, True)
    sw, cw = Q.quantize_mx(to_dev(w), e4m3, [-1], 32, 448.0, True)
    out = Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    rows = np.arange(0, 8192, 32)
    want = oracle.linear_mx(to_np(ca)[rows], to_np(cw), None, input_scale=to_np(sa)[rows],
                            weight_scale=to_np(sw), block_size=32)
    assert G.rel_l2(to_np(out)[rows], want) < 1e-3


def test_fused_pack_matches_separate_pack():
    """quantize_mx writes the GEMM operand in the same pass for MXFP8
    activations; the product must equal the one from a separate pack."""
    from voyager_b200 import mxgemm

    g = torch.Generator().manual_seed(11)
    a = torch.randn(300, 512, generator=g).bfloat16().cuda()
    w = (torch.randn(264, 512, generator=g) * 0.02).bfloat16().cuda()
    Q = torch.ops.quantized_ops
    e4m3 = to_dev(quantization_map("fp8_e4m3"))
    sa, ca = Q.quantize_mx(a, e4m3, [-1], 32, 448.0, True)
    sw, cw = Q.quantize_mx(w, e4m3, [-1], 32, 448.0, True)
    assert mxgemm._vouched_entry(ca, sa)[1] is not None  # fused operand present
    fused = mxgemm.linear(ca, cw, None, sa, sw)
    sep = mxgemm.linear(ca.clone(), cw, None, sa, sw)  # clone: no provenance -> pack + check
    torch.cuda.synchronize()
    assert sep is not None and torch.equal(fused, sep)
    want = oracle.linear_mx(to_np(ca), to_np(cw), None, input_scale=to_np(sa),
                            weight_scale=to_np(sw), block_size=32)
    assert G.rel_l2(to_np(fused), want) < 1e-3


# ---------------------------------------------------------------------------
# matmul_mx with MXFP8 operands on the same kernels (batched)
# ---------------------------------------------------------------------------
def _mx_along(x, axis):
    qm = quantization_map("fp8_e4m3")
    s, c = oracle.quantize_mx(x, qm, [axis], 32, 448.0, True)
    return c, s


def _bf16(rng, shape, std):
    from voyager_b200.synth import f32_to_bf16_bits

    return f32_to_bf16_bits((rng.standard_normal(shape) * std).astype(np.float32))


# (batch dims, M, K, N, layout, right operand shared across the batch)
MATMUL_CASES = [((2, 3), 128, 128, 256, "ck", False), ((4,), 300, 256, 264, "ck", False),
                ((2,), 77, 96, 40, "kc", False), ((3,), 512, 128, 512, "ck", True),
                ((), 1000, 640, 520, "ck", False), ((2,), 256, 4096, 1024, "kc", True),
                ((1, 2), 2048, 128, 2048, "ck", False)]


@pytest.mark.parametrize("bdims,m,k,n,layout,shared", MATMUL_CASES)
def test_mxf8_matmul(bdims, m, k, n, layout, shared):
    from voyager_b200 import mxgemm

    rng = np.random.default_rng(m + k + n + len(bdims))
    a = _bf16(rng, bdims + (m, k), 1.0)
    bshape = ((k, n) if layout == "ck" else (n, k))
    b = _bf16(rng, (bshape if shared else bdims + bshape), 0.5)
    ca, sa = _mx_along(a, -1)
    cb, sb = _mx_along(b, -2 if layout == "ck" else -1)
    want = oracle.matmul_mx(ca, cb, input_scale=sa, weight_scale=sb, block_size=32,
                            weight_layout=layout)
    dca, dsa, dcb, dsb = to_dev(ca), to_dev(sa), to_dev(cb), to_dev(sb)
    assert mxgemm.matmul_applies(dca, dcb, dsa, dsb, 32, None, None, layout)
    out = mxgemm.matmul(dca, dcb, dsa, dsb, layout)
    assert out is not None, "operands were not accepted as exact MXFP8"
    got = to_np(out)
    assert got.shape == want.shape
    assert G.rel_l2(got, want) < 1e-3
    # and through the op, twice (the shared operand's pack is cached)
    for _ in range(2):
        got2 = to_np(torch.ops.quantized_ops.matmul_mx(dca, dcb, input_scale=dsa,
                                                       weight_scale=dsb, block_size=32,
                                                       weight_layout=layout))
        assert np.array_equal(got2, got)


def test_mxf8_matmul_from_quantize_mx():
    """Operands straight from the CUDA quantize_mx (vouched, packed in the
    same pass for the left operand) give the same product."""
    Q = torch.ops.quantized_ops
    from voyager_b200.tables import get_quantization_map

    rng = np.random.default_rng(5)
    a, b = _bf16(rng, (2, 4, 256, 128), 1.0), _bf16(rng, (2, 4, 128, 256), 1.0)
    e4m3 = get_quantization_map("fp8_e4m3", torch.device("cuda"))
    sa, ca = Q.quantize_mx(to_dev(a), e4m3, [-1], 32, 448.0, True)
    sb, cb = Q.quantize_mx(to_dev(b), e4m3, [-2], 32, 448.0, True)
    got = to_np(Q.matmul_mx(ca, cb, input_scale=sa, weight_scale=sb, block_size=32))
    want = oracle.matmul_mx(to_np(ca), to_np(cb), input_scale=to_np(sa), weight_scale=to_np(sb),
                            block_size=32)
    assert G.rel_l2(got, want) < 1e-3


# ---------------------------------------------------------------------------
# NVFP4 x NVFP4 linear_mx on tcgen05 kind::mxf4nvf4 (scale_vec::4X)
# ---------------------------------------------------------------------------
def _nvf4(x):
    return oracle.quantize_mx(x, quantization_map("fp4_e2m1"), [-1], 16, 6.0, False,
                              quantization_map("fp8_e4m3"))


NVF4_SHAPES = [(128, 256, 256), (1, 256, 8), (300, 4096, 1000), (77, 96, 40), (1024, 2048, 2048),
               (256, 4104, 264)]


@pytest.mark.parametrize("m,k,n", NVF4_SHAPES)
def test_nvf4_linear(m, k, n, monkeypatch):
    from voyager_b200 import mxgemm
    from voyager_b200.synth import f32_to_bf16_bits

    rng = np.random.Generator(np.random.PCG64(m + k + n))
    a = f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    w = f32_to_bf16_bits((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    bias = f32_to_bf16_bits((rng.standard_normal(n) * 0.1).astype(np.float32)) if m % 2 else None
    sa, ca = _nvf4(a)
    sw, cw = _nvf4(w)
    calls = {"n": 0}
    real = mxgemm.nvf4_linear

    def counting(*args, **kw):
        out = real(*args, **kw)
        calls["n"] += out is not None
        return out

    monkeypatch.setattr(mxgemm, "nvf4_linear", counting)
    got = to_np(torch.ops.quantized_ops.linear_mx(to_dev(ca), to_dev(cw), to_dev(bias),
                                                  input_scale=to_dev(sa), weight_scale=to_dev(sw),
                                                  block_size=16))
    assert calls["n"] == 1, "the NVFP4 kernel did not take the operands"
    want = oracle.linear_mx(ca, cw, bias, input_scale=sa, weight_scale=sw, block_size=16)
    assert G.rel_l2(got, want) < 1e-3
