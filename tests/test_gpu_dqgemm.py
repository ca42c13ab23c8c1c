"""linear_mx / matmul_mx on the tcgen05 bf16 GEMM with the weight read back
in shared memory (``voyager_b200.dqgemm``), against the oracle.

* The in-kernel decode (palette lookup, bf16 product with the block scale)
  is bit-exact against the oracle's ``dequantize_mx`` of the same codes.
* GEMM results: rel-L2 <= 1e-3 against the oracle's dequantize-then-matmul
  (float32 sums rounded once to bf16), as for every GEMM here: only the
  float32 summation order differs.

Weight formats: C2's three (NF4 g64 as stored indices + their 16-level
codebook, posit8_1 and int8 as value codes with block or per-row scales),
NVFP4 (E2M1 x E4M3 scale per 16, the C4 weight), E4M3 codes with
non-power-of-two scales (8-bit palette), and a plain bf16 weight with more
than 256 values (loaded by TMA)."""

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_dev, to_np
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits, index_table, quantization_map

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def _bf16(rng, shape, std):
    return f32_to_bf16_bits((rng.standard_normal(shape) * std).astype(np.float32))


def _nf4_codebook():
    lut = quantization_map("lut4")
    levels = np.unique(bf16_bits_to_f32(lut))
    return f32_to_bf16_bits(levels.astype(np.float32)), index_table(lut)


def weight_format(fmt, w):
    """(codes, scale, codebook, block_size) of a bf16 weight [N, K] quantized
    as the reference's convert stores it."""
    N, K = w.shape
    if fmt == "nf4_g64":
        cb, idx = _nf4_codebook()
        s, c = oracle.quantize_mx(w, idx, [-1], 64, 1.0)
        return c, s, cb, 64
    if fmt == "posit8_bs32":
        s, c = oracle.quantize_mx(w, quantization_map("posit8_1"), [-1], 32, 4096.0)
        return c, s, None, 32
    if fmt == "int8_bs32":
        s, c = oracle.quantize_mx(w, quantization_map("int8"), [-1], 32, 127.0)
        return c, s, None, 32
    if fmt == "int8_row":
        s, c = oracle.quantize_mx(w, quantization_map("int8"), [-1], K, 127.0)
        return c, s, None, K
    if fmt == "nvfp4":
        s, c = oracle.quantize_mx(w, quantization_map("fp4_e2m1"), [-1], 16, 6.0, False,
                                  quantization_map("fp8_e4m3"))
        return c, s, None, 16
    if fmt == "e4m3_amax":
        s, c = oracle.quantize_mx(w, quantization_map("fp8_e4m3"), [-1], 32, 448.0)
        return c, s, None, 32
    if fmt == "bf16":
        return w, None, None, None
    raise ValueError(fmt)


FORMATS = ["nf4_g64", "posit8_bs32", "int8_bs32", "int8_row", "nvfp4", "e4m3_amax", "bf16"]


@pytest.mark.parametrize("fmt", FORMATS[:-1])
@pytest.mark.parametrize("n,k", [(64, 256), (40, 200), (264, 4096)])
def test_decode_bit_exact(fmt, n, k):
    from voyager_b200 import dqgemm

    rng = np.random.default_rng(n + k)
    w = _bf16(rng, (n, k), 0.02)
    if fmt == "nf4_g64" and k % 64:
        k = k // 64 * 64
        w = w[:, :k].copy()
    c, s, cb, bs = weight_format(fmt, w)
    pw = dqgemm.pack(to_dev(c), to_dev(s), to_dev(cb), bs)
    assert pw is not None and pw.mode in (dqgemm.MODE_LUT4, dqgemm.MODE_LUT8)
    want = oracle.dequantize_mx(c, s, cb, bs)
    got = to_np(dqgemm.decode(pw))
    if fmt.startswith("int8"):
        # int8 codes can hold 257 patterns (-128..127 and -0): then -0 shares
        # +0's palette entry, a zero weight either way
        want = np.where(want == 0x8000, np.uint16(0), want)
        got = np.where(got == 0x8000, np.uint16(0), got)
    bad = G.bit_mismatches(got, want)
    assert len(bad) == 0, f"{len(bad)} mismatches, first at {bad[:5]}"


# M x K x N; K tails (not a multiple of 64) and N tails (not of 256) included
SHAPES = [(128, 256, 256), (1, 128, 8), (300, 200, 264), (256, 4096, 1000), (77, 64, 40),
          (1024, 1024, 2048)]


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,k,n", SHAPES)
def test_linear(fmt, m, k, n):
    from voyager_b200 import dqgemm

    if fmt == "nf4_g64" and k % 64:
        pytest.skip("NF4 groups of 64")
    rng = np.random.default_rng(m * 3 + k + n)
    a = _bf16(rng, (m, k), 1.0)
    w = _bf16(rng, (n, k), 0.02)
    bias = _bf16(rng, (n,), 0.1) if m % 2 else None
    c, s, cb, bs = weight_format(fmt, w)
    want = oracle.linear_mx(a, c, bias, weight_scale=s, block_size=bs, weight_code=cb)
    dc, ds, dcb = to_dev(c), to_dev(s), to_dev(cb)
    got = dqgemm.linear(to_dev(a), dc, to_dev(bias), None, ds, bs, None, dcb, "kc")
    assert got is not None
    assert G.rel_l2(to_np(got), want) < 1e-3
    pw = dqgemm.packed_weight(dc, ds, dcb, bs, "kc")
    expect = dqgemm.MODE_TMA if fmt == "bf16" else (
        dqgemm.MODE_LUT4 if fmt in ("nf4_g64", "nvfp4") else dqgemm.MODE_LUT8)
    assert pw.mode == expect
    # through the op (the cached packed weight), with MXFP8 activations
    qm = quantization_map("fp8_e4m3")
    if bs is not None and fmt != "bf16":
        sa, ca = oracle.quantize_mx(a, qm, [-1], bs, 448.0, True)
        want2 = oracle.linear_mx(ca, c, bias, input_scale=sa, weight_scale=s, block_size=bs,
                                 weight_code=cb)
        got2 = torch.ops.quantized_ops.linear_mx(to_dev(ca), dc, to_dev(bias),
                                                 input_scale=to_dev(sa), weight_scale=ds,
                                                 block_size=bs, weight_code=dcb)
        assert G.rel_l2(to_np(got2), want2) < 1e-3


@pytest.mark.parametrize("fmt", ["nf4_g64", "posit8_bs32", "int8_row"])
def test_c2_formats_at_c3_shape(fmt):
    """C2's weight formats on a bf16 weight of C3's shape [11008, 4096] times
    C3's activations [8192, 4096]; the oracle on a sample of 256 rows (rows
    of the product are independent)."""
    from voyager_b200 import dqgemm, synth

    a_np, w_np = synth.c3_operands()
    c, s, cb, bs = weight_format(fmt, w_np)
    dc, ds, dcb = to_dev(c), to_dev(s), to_dev(cb)
    got = to_np(torch.ops.quantized_ops.linear_mx(to_dev(a_np), dc, None, weight_scale=ds,
                                                  block_size=bs, weight_code=dcb))
    pw = dqgemm.packed_weight(dc, ds, dcb, bs, "kc")
    assert pw.mode != dqgemm.MODE_TMA
    rows = np.random.default_rng(1).choice(a_np.shape[0], 256, replace=False)
    want = oracle.linear_mx(a_np[rows], c, None, weight_scale=s, block_size=bs, weight_code=cb)
    assert G.rel_l2(got[rows], want) < 1e-3


def test_ck_weight_layout():
    """A CK-stored weight ([K, N], blocks along dim 0) is transposed once."""
    rng = np.random.default_rng(3)
    K, N = 256, 136
    w = _bf16(rng, (K, N), 0.02)
    s, c = oracle.quantize_mx(w, quantization_map("posit8_1"), [0], 32, 4096.0)
    a = _bf16(rng, (96, K), 1.0)
    want = oracle.linear_mx(a, c, None, weight_scale=s, block_size=32, weight_layout="ck")
    got = torch.ops.quantized_ops.linear_mx(to_dev(a), to_dev(c), None, weight_scale=to_dev(s),
                                            block_size=32, weight_layout="ck")
    assert G.rel_l2(to_np(got), want) < 1e-3


@pytest.mark.parametrize("layout", ["ck", "kc"])
@pytest.mark.parametrize("fmt", ["int8_bs32", "bf16"])
def test_matmul_batched(layout, fmt):
    """matmul_mx of activations (both operands per batch), non-MXFP8."""
    rng = np.random.default_rng(11)
    B, M, K, N = 3, 200, 128, 72
    a = _bf16(rng, (B, M, K), 1.0)
    b = _bf16(rng, (B, K, N) if layout == "ck" else (B, N, K), 1.0)
    if fmt == "bf16":
        ca, sa, cb, sb, bs = a, None, b, None, None
    else:
        qm = quantization_map("int8")
        sa, ca = oracle.quantize_mx(a, qm, [-1], 32, 127.0)
        sb, cb = oracle.quantize_mx(b, qm, [-2 if layout == "ck" else -1], 32, 127.0)
        bs = 32
    want = oracle.matmul_mx(ca, cb, input_scale=sa, weight_scale=sb, block_size=bs,
                            weight_layout=layout)
    got = torch.ops.quantized_ops.matmul_mx(to_dev(ca), to_dev(cb), input_scale=to_dev(sa),
                                            weight_scale=to_dev(sb), block_size=bs,
                                            weight_layout=layout)
    assert G.rel_l2(to_np(got), want) < 1e-3


@pytest.mark.parametrize("m", [128, 1024])
def test_w4a8_large_m(m):
    """C4 at M >= 128: NVFP4 weight (4-bit palette, E4M3 block-16 scales) x
    MXFP8 activations on the bf16 tcgen05 GEMM."""
    from voyager_b200 import w4a8

    rng = np.random.default_rng(m)
    K, N = 4096, 1024
    a = _bf16(rng, (m, K), 1.0)
    w = _bf16(rng, (N, K), 0.02)
    sa, ca = oracle.quantize_mx(a, quantization_map("fp8_e4m3"), [-1], 32, 448.0, True)
    cw, sw, _, _ = weight_format("nvfp4", w)
    want = oracle.linear_mx(oracle.dequantize_mx(ca, sa, None, 32),
                            oracle.dequantize_mx(cw, sw, None, 16))
    got = to_np(w4a8.linear(to_dev(ca), to_dev(sa), to_dev(cw), to_dev(sw)))
    assert G.rel_l2(got, want) < 1e-3


@pytest.mark.parametrize("fmt", ["nvfp4", "posit8_bs32", "bf16"])
@pytest.mark.parametrize("m,k,n,splits", [(128, 4096, 4096, 4), (40, 200, 264, 2),
                                          (130, 1024, 520, 16), (256, 14336, 512, 7)])
def test_split_k(fmt, m, k, n, splits):
    """K steps split over several CTA pairs per output tile (float32 slices
    added in order by the finalize launch) against the oracle and against the
    unsplit kernel; K and N tails, a bias, rows past M in the CTA pair."""
    from voyager_b200 import _lib, dqgemm

    rng = np.random.default_rng(m + k + n + splits)
    a = _bf16(rng, (m, k), 1.0)
    w = _bf16(rng, (n, k), 0.02)
    bias = _bf16(rng, (n,), 0.1)
    c, s, cb, bs = weight_format(fmt, w)
    want = oracle.linear_mx(a, c, bias, weight_scale=s, block_size=bs, weight_code=cb)
    pw = dqgemm.packed_weight(to_dev(c), to_dev(s), to_dev(cb), bs, "kc")
    a_dev = to_dev(a)
    one = to_np(dqgemm.gemm(a_dev, pw, to_dev(bias), splits=1)[0])
    got = to_np(dqgemm.gemm(a_dev, pw, to_dev(bias), splits=splits)[0])
    assert G.rel_l2(got, want) < 1e-3
    assert G.rel_l2(got, one) < 1e-3
    # the library's own choice for C4's M = 128 shapes splits the K steps
    lib = _lib.load()
    assert lib.vq_gemm_dq_splits(1, 128, 4096, 4096) > 1
    assert lib.vq_gemm_dq_splits(1, 128, 4096, 14336) > 1
    assert lib.vq_gemm_dq_splits(1, 8192, 11008, 4096) == 1
    assert lib.vq_gemm_dq_splits(2, 128, 4096, 4096) == 1


@pytest.mark.parametrize("fmt", ["nf4_g64", "posit8_bs32", "int8_row", "nvfp4"])
def test_decode_once_large_m(fmt, monkeypatch):
    """From DECODE_ONCE_M activation rows on, the packed weight is decoded
    once into bf16 (vq_dq_decode) and multiplied by the TMA-mode kernel; both
    that and the in-kernel decode agree with the oracle."""
    from voyager_b200 import dqgemm

    m, k, n = 1024, 1088, 520
    if fmt == "nf4_g64":
        k = 1024
    rng = np.random.default_rng(k + n)
    a = _bf16(rng, (m, k), 1.0)
    w = _bf16(rng, (n, k), 0.02)
    bias = _bf16(rng, (n,), 0.1)
    c, s, cb, bs = weight_format(fmt, w)
    want = oracle.linear_mx(a, c, bias, weight_scale=s, block_size=bs, weight_code=cb)
    pw = dqgemm.packed_weight(to_dev(c), to_dev(s), to_dev(cb), bs, "kc")
    assert pw.mode != dqgemm.MODE_TMA
    monkeypatch.setattr(dqgemm, "DECODE_ONCE_M", 0)  # the in-kernel decode
    in_kernel = to_np(dqgemm.gemm(to_dev(a), pw, to_dev(bias))[0])
    monkeypatch.setattr(dqgemm, "DECODE_ONCE_M", m)  # decoded once
    once = to_np(dqgemm.gemm(to_dev(a), pw, to_dev(bias))[0])
    assert G.rel_l2(in_kernel, want) < 1e-3
    assert G.rel_l2(once, want) < 1e-3
    # the decoded weight is exactly what the kernel decodes in shared memory
    assert G.rel_l2(once, in_kernel) < 1e-3
