"""The outlier CSR side-stream on CUDA against the oracle.

filter_outlier, quantize_mx_outlier, slice_csr_tensor and spmm_csr are
bit-exact (any NaN equals any NaN); linear_mx / matmul_mx with A_data are
within rel-L2 1e-3 of the oracle (the dense GEMM sums in its own order) and
their outlier term is checked bit for bit.  At full size the checks are
properties: the CSR scattered back equals the input's outliers, the fused
quantize equals quantize_mx of the materialised inliers, and a row sample
matches the oracle."""

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_dev, to_np
from oracle.numerics import quantization_map

pytestmark = pytest.mark.gpu

Q = None


@pytest.fixture(scope="module", autouse=True)
def _setup():
    global Q
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    Q = torch.ops.quantized_ops
    yield


def _spiky(shape, seed, frac=0.02, mult=50.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(shape, generator=g)
    n = x.numel()
    k = max(1, int(n * frac))
    pos = torch.randperm(n, generator=g)[:k]
    x.view(-1)[pos] *= mult
    return x.to(dtype)


def _np(t):
    return to_np(t)


def _same(got, want, what=""):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape and got.dtype == want.dtype, (what, got.shape, want.shape,
                                                                 got.dtype, want.dtype)
    bad = G.bit_mismatches(got, want)
    assert len(bad) == 0, f"{what}: {len(bad)} mismatches, first at {bad[:5]}"


# ---------------------------------------------------------------------------
# filter_outlier
# ---------------------------------------------------------------------------
FILTER_CASES = [((1, 1), 0.0, 1.0), ((7, 5), 0.8, 0.3), ((2, 9, 33), 1.7, 0.05),
                ((40, 1), 0.1, 0.5), ((16, 16), -0.5, 1.0), ((12, 20), 1.0, 0.0),
                ((300, 1000), 2.0, 0.06), ((3, 64, 4096), 3.0, 0.02), ((5, 4100), 2.5, 0.001),
                ((33, 70), float("inf"), 0.1), ((33, 70), float("nan"), 0.1)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,thr,pct", FILTER_CASES)
def test_filter_outlier(dtype, shape, thr, pct):
    x = _spiky(shape, seed=shape[-1] + len(shape), dtype=dtype)
    k = min(4, x.numel())
    x.view(-1)[:k] = torch.tensor([0.0, -0.0, float("nan"), float("-inf")])[:k].to(dtype)
    got = Q.filter_outlier(x.cuda(), thr, pct)
    want = oracle.filter_outlier(_np(x), thr, pct)
    for g, w, n in zip(got, want, ("data", "indices", "indptr", "inliers")):
        _same(_np(g), w, n)


def test_filter_outlier_unaligned_input_takes_the_scalar_path():
    base = _spiky((1 + 37 * 64,), seed=5).cuda()
    x = base[1:].view(37, 64)  # 2 bytes past a 16-byte boundary
    assert x.data_ptr() % 16 != 0
    got = Q.filter_outlier(x, 2.0, 0.05)
    want = oracle.filter_outlier(_np(x), 2.0, 0.05)
    for g, w in zip(got, want):
        _same(_np(g), w)


def test_filter_outlier_empty():
    for shape in ((0, 8), (8, 0), (2, 0, 5)):
        x = torch.zeros(shape, dtype=torch.bfloat16, device="cuda")
        d, i, p, inl = Q.filter_outlier(x, 1.0, 0.5)
        assert d.shape[-1] == 0 and inl.shape == x.shape
        assert (p == 0).all()


def test_filter_outlier_many_tiles_against_torch_count():
    """4096 x 4096 (4096 tiles, each waiting on its predecessor): the row
    pointers equal the cumulative per-row counts and the CSR scattered back
    is exactly the input's outliers."""
    x = _spiky((4096, 4096), seed=1, frac=0.01).cuda()
    thr = 4.0
    d, i, p, inl = Q.filter_outlier(x, thr, 0.02)
    keep = (x.abs() > thr) & (x != 0)
    counts = keep.sum(1)
    want_p = torch.cat([torch.zeros(1, device="cuda", dtype=torch.int64), counts.cumsum(0)])
    assert torch.equal(p.long(), want_p)
    nse = int(p[-1])
    rows = torch.repeat_interleave(torch.arange(4096, device="cuda"), counts)
    back = torch.zeros_like(x)
    back[rows, i[:nse].long()] = d[:nse]
    assert torch.equal(back.view(torch.int16), torch.where(keep, x, 0).view(torch.int16))
    assert (i[nse:] == -1).all() and (d[nse:].view(torch.int16) == 0).all()
    assert torch.equal(inl.view(torch.int16), torch.where(x.abs() > thr, 0, x).view(torch.int16))


# ---------------------------------------------------------------------------
# quantize_mx_outlier
# ---------------------------------------------------------------------------
QMO = [  # qmap, axes, bs, quant_max, pow2, scale_qmap
    ("fp4_e2m1", [-1], 16, 6.0, False, "fp8_e4m3"),
    ("fp8_e4m3", [-1], 32, 448.0, True, None),
    ("fp4_e2m1", [-1], 32, 6.0, True, None),
    ("int8", [-1], 32, 127.0, False, None),
    ("int8", [-2], 32, 127.0, False, None),
    ("posit8_1", [-1], 16, 4096.0, False, None),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("fmt", QMO, ids=[f"{q[0]}-ax{q[1][0]}-bs{q[2]}" for q in QMO])
@pytest.mark.parametrize("shape,offset", [((64, 256), 0), ((3, 40, 128), 11), ((130, 96), 0)])
def test_quantize_mx_outlier(dtype, fmt, shape, offset):
    qd, axes, bs, qmax, pow2, sq = fmt
    x = _spiky(shape, seed=sum(shape) + bs, frac=0.01, dtype=dtype)
    qm = quantization_map(qd)
    sqm = None if sq is None else quantization_map(sq)
    got = Q.quantize_mx_outlier(x.cuda(), to_dev(qm), axes, bs, qmax, pow2,
                                None if sqm is None else to_dev(sqm), None, 3.0, 0.02, offset)
    want = oracle.quantize_mx_outlier(_np(x), qm, axes, bs, qmax, pow2, sqm, None, 3.0, 0.02,
                                      offset)
    for g, w, n in zip(got, want, ("data", "indices", "indptr", "scale", "codes")):
        _same(_np(g), w, n)


def test_quantize_mx_outlier_fused_equals_two_pass_c1():
    """C1's NVFP4 input (1 % of elements x50) at full size: the fused
    kernel's codes and scales equal quantize_mx of filter_outlier's inliers."""
    from voyager_b200 import synth

    x = to_dev(synth.c1_input())
    e2m1, e4m3 = to_dev(quantization_map("fp4_e2m1")), to_dev(quantization_map("fp8_e4m3"))
    d, i, p, s, c = Q.quantize_mx_outlier(x, e2m1, [-1], 16, 6.0, False, e4m3, None, 6.0, 0.02)
    d2, i2, p2, inl = Q.filter_outlier(x, 6.0, 0.02)
    s2, c2 = Q.quantize_mx(inl, e2m1, [-1], 16, 6.0, False, e4m3)
    for a, b in ((d, d2), (i, i2), (p, p2), (s, s2), (c, c2)):
        assert torch.equal(a.view(torch.uint8) if a.dtype != torch.int32 else a,
                           b.view(torch.uint8) if b.dtype != torch.int32 else b)
    assert int(p[-1]) == int(((x.abs() > 6.0) & (x != 0)).sum())
    # a row sample against the oracle
    rows = np.arange(0, 4096, 256)
    xs = synth.c1_input()[rows]
    ws_, wc = oracle.quantize_mx(oracle.filter_outlier(xs, 6.0, 1.0)[3], quantization_map(
        "fp4_e2m1"), [-1], 16, 6.0, False, quantization_map("fp8_e4m3"))
    _same(_np(s)[rows], ws_)
    _same(_np(c)[rows], wc)


# ---------------------------------------------------------------------------
# spmm_csr
# ---------------------------------------------------------------------------
def _csr_of(x, thr, pct):
    d, i, p, _ = Q.filter_outlier(x.cuda(), thr, pct)
    return d, i, p


@pytest.mark.parametrize("N", [1, 7, 8, 12, 16, 24, 40, 96, 264])
@pytest.mark.parametrize("bdtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", ["kc", "ck"])
def test_spmm_csr_widths(N, bdtype, layout):
    x = _spiky((48, 300), seed=N, frac=0.05)
    x[5, :] = torch.randn(300).to(x.dtype) * 30  # a long row (> 256 entries)
    d, i, p = _csr_of(x, 2.0, 1.0)
    g = torch.Generator().manual_seed(N + 1)
    Bn = torch.randn((N, 300) if layout == "kc" else (300, N), generator=g).to(bdtype)
    got = Q.spmm_csr(d, i, p, Bn.cuda(), weight_layout=layout)
    want = oracle.spmm_csr(_np(d), _np(i), _np(p), _np(Bn), weight_layout=layout)
    _same(_np(got), want)


def test_spmm_csr_scaled_weight_and_codebook():
    x = _spiky((64, 256), seed=3, frac=0.03)
    d, i, p = _csr_of(x, 3.0, 0.05)
    g = torch.Generator().manual_seed(9)
    w = (torch.randn(96, 256, generator=g) * 0.05).bfloat16().cuda()
    e4m3 = to_dev(quantization_map("fp8_e4m3"))
    sw, cw = Q.quantize_mx(w, e4m3, [-1], 32, 448.0, True)
    got = Q.spmm_csr(d, i, p, cw, sw, None, 32, "kc")
    want = oracle.spmm_csr(_np(d), _np(i), _np(p), _np(cw), _np(sw), None, 32, "kc")
    _same(_np(got), want, "mxfp8 weight")
    # again: the decoded, transposed weight comes from the cache
    _same(_np(Q.spmm_csr(d, i, p, cw, sw, None, 32, "kc")), want, "cached")
    code = to_dev(np.linspace(-1, 1, 16).astype(np.float32)).bfloat16()
    idx = torch.randint(0, 16, (256, 24), generator=g).float().bfloat16().cuda()
    got = Q.spmm_csr(d, i, p, idx, None, code, None, "ck")
    want = oracle.spmm_csr(_np(d), _np(i), _np(p), _np(idx), None, _np(code), None, "ck")
    _same(_np(got), want, "codebook")


def test_spmm_csr_batched_and_offset_pointers():
    x = _spiky((3, 32, 64), seed=4, frac=0.05)
    out = Q.quantize_mx_outlier(x.cuda(), to_dev(quantization_map("fp8_e4m3")), [-1], 32,
                                448.0, True, None, None, 2.5, 0.1, 5)
    d, i, p = out[:3]
    B = torch.randn(3, 64, 40).bfloat16().cuda()
    got = Q.spmm_csr(d, i, p, B, weight_layout="ck")
    want = oracle.spmm_csr(_np(d), _np(i), _np(p), _np(B), weight_layout="ck")
    _same(_np(got), want)


# ---------------------------------------------------------------------------
# slice_csr_tensor
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dim,start,end,sf", [(0, 8, 40, 1.0), (0, 0, 64, 0.4), (0, 63, 64, 1.0),
                                              (0, 10, 10, 1.0), (1, 32, 96, 0.5),
                                              (-1, 100, 256, 0.2), (1, 0, 256, 1.5),
                                              (1, 300, 400, 1.0)])
def test_slice_csr_tensor(dim, start, end, sf):
    x = _spiky((64, 256), seed=11, frac=0.02)
    d, i, p, _ = Q.filter_outlier(x.cuda(), 2.0, 0.05)
    got = Q.slice_csr_tensor(d, i, p, dim, start, end, sf)
    want = oracle.slice_csr_tensor(_np(d), _np(i), _np(p), dim, start, end, sf)
    for g, w in zip(got, want):
        _same(_np(g), w)


# ---------------------------------------------------------------------------
# linear_mx / matmul_mx with the side-stream
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("m,k,n", [(128, 256, 96), (300, 512, 264)])
def test_linear_mx_with_outliers(m, k, n):
    e4m3 = to_dev(quantization_map("fp8_e4m3"))
    x = _spiky((m, k), seed=m, frac=0.01).cuda()
    w = (torch.randn(n, k) * 0.05).bfloat16().cuda()
    d, i, p, sa, ca = Q.quantize_mx_outlier(x, e4m3, [-1], 32, 448.0, True, None, None, 4.0,
                                            0.02)
    sw, cw = Q.quantize_mx(w, e4m3, [-1], 32, 448.0, True)
    got = Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32, A_data=d,
                      A_indices=i, A_indptr=p)
    want = oracle.linear_mx(_np(ca), _np(cw), None, input_scale=_np(sa), weight_scale=_np(sw),
                            block_size=32, A_data=_np(d), A_indices=_np(i), A_indptr=_np(p))
    assert G.rel_l2(_np(got), want) < 1e-3
    # the outlier term exactly: the result is bf16(dense) + spmm in bf16
    dense = Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    sp = Q.spmm_csr(d, i, p, cw, sw, None, 32, "kc")
    _same(_np(sp), oracle.spmm_csr(_np(d), _np(i), _np(p), _np(cw), _np(sw), None, 32, "kc"))
    assert torch.equal(got.view(torch.int16), (dense + sp).view(torch.int16))


def test_matmul_mx_with_outliers_ck():
    e4m3 = to_dev(quantization_map("fp8_e4m3"))
    x = _spiky((128, 256), seed=21, frac=0.01).cuda()
    w = (torch.randn(256, 80) * 0.05).bfloat16().cuda()
    d, i, p, sa, ca = Q.quantize_mx_outlier(x, e4m3, [-1], 32, 448.0, True, None, None, 4.0,
                                            0.02)
    sw, cw = Q.quantize_mx(w, e4m3, [-2], 32, 448.0, True)
    got = Q.matmul_mx(ca, cw, input_scale=sa, weight_scale=sw, block_size=32, A_data=d,
                      A_indices=i, A_indptr=p)
    want = oracle.matmul_mx(_np(ca), _np(cw), input_scale=_np(sa), weight_scale=_np(sw),
                            block_size=32, A_data=_np(d), A_indices=_np(i), A_indptr=_np(p))
    assert G.rel_l2(_np(got), want) < 1e-3


def test_c3_with_outliers_rows_sample():
    """C3 (M=8192, K=4096, N=11008) with the activation's outliers above 4.0
    in a CSR: the MXFP8 GEMM adds spmm_csr in its epilogue.  A row sample of
    the outlier term is bit-exact against the oracle, and the result equals
    bf16(dense) + that term."""
    from voyager_b200 import synth

    a, w = synth.c3_operands()
    a = a.copy()
    rng = np.random.default_rng(0)
    pos = rng.choice(a.size, a.size // 100, replace=False)
    af = oracle.bf16_bits_to_f32(a).reshape(-1)
    af[pos] *= 50
    a = oracle.f32_to_bf16_bits(af.reshape(a.shape))
    e4m3 = to_dev(quantization_map("fp8_e4m3"))
    d, i, p, sa, ca = Q.quantize_mx_outlier(to_dev(a), e4m3, [-1], 32, 448.0, True, None, None,
                                            4.0, 0.02)
    sw, cw = Q.quantize_mx(to_dev(w), e4m3, [-1], 32, 448.0, True)
    out = Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32, A_data=d,
                      A_indices=i, A_indptr=p)
    dense = Q.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    sp = Q.spmm_csr(d, i, p, cw, sw, None, 32, "kc")
    assert torch.equal(out.view(torch.int16), (dense + sp).view(torch.int16))
    rows = np.arange(0, 8192, 512)
    pn, iN, dn = _np(p), _np(i), _np(d)
    sub_p = [0]
    sub_i, sub_d = [], []
    for r in rows:
        sub_i.append(iN[pn[r]:pn[r + 1]])
        sub_d.append(dn[pn[r]:pn[r + 1]])
        sub_p.append(sub_p[-1] + pn[r + 1] - pn[r])
    want = oracle.spmm_csr(np.concatenate(sub_d), np.concatenate(sub_i),
                           np.array(sub_p, dtype=np.int32), _np(cw), _np(sw), None, 32, "kc")
    _same(_np(sp)[rows], want)
