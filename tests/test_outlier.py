"""The outlier CSR side-stream on CPU: the oracle against torch's own CPU
kernels (the arithmetic the reference's ops delegate to), the exact-rounding
FMA helper, the C ABI's threshold rounding and argument checks (no GPU).

The reference ops themselves are pinned by the golden cases
(``tests/test_oracle_golden.py``); these tests widen the coverage to shapes
and widths the fixtures do not hold."""

import ctypes
import math
from fractions import Fraction

import numpy as np
import pytest
import torch

import oracle
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits
from oracle.outlier import fma_f32
from voyager_b200 import _lib


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


# ---------------------------------------------------------------------------
# fused multiply-add restatement
# ---------------------------------------------------------------------------
def _fma_exact(a, b, c):
    """a * b + c in exact rationals, rounded to float32 half-even."""
    if not all(math.isfinite(float(x)) for x in (a, b, c)):
        return np.float32(np.float64(a) * np.float64(b) + np.float64(c))
    v = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
    f = np.float32(float(v))  # nearest double, then float32: fix the tie below
    lo, hi = (f, np.nextafter(f, np.float32(np.inf))) if Fraction(float(f)) <= v else \
        (np.nextafter(f, np.float32(-np.inf)), f)
    dl, dh = v - Fraction(float(lo)), Fraction(float(hi)) - v
    if dl < dh:
        r = lo
    elif dh < dl:
        r = hi
    else:
        r = lo if (lo.view(np.uint32) & 1) == 0 else hi
    if r == 0:
        # exact zero sums are +0 unless both addends are -0 (round-to-nearest)
        p_neg = (np.float64(a) * np.float64(b) == 0) and math.copysign(1, a) * math.copysign(1, b) < 0
        return np.float32(-0.0) if (p_neg and math.copysign(1, c) < 0) else np.float32(0.0)
    return np.float32(r)


def test_fma_matches_exact_rounding():
    rng = np.random.default_rng(0)
    a = rng.standard_normal(3000).astype(np.float32)
    b = rng.standard_normal(3000).astype(np.float32)
    c = rng.standard_normal(3000).astype(np.float32) * np.float32(3)
    # sums that land on float32 ties: c = -(a*b rounded to float32) + tiny
    t = 500
    c[:t] = (-(a[:t].astype(np.float64) * b[:t])).astype(np.float32)
    got = fma_f32(a, b, c)
    want = np.array([_fma_exact(x, y, z) for x, y, z in zip(a, b, c)], dtype=np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_fma_tie_cases():
    # 1 + 2^-24 is exactly between 1 and the next float32; an FMA whose
    # exact result is just above or below that tie must round away from it
    one = np.float32(1.0)
    e = np.float32(2.0 ** -24)
    eps = np.float32(2.0 ** -60)
    # a * b = 2^-24 + 2^-60 (exact in float64), c = 1 -> just above the tie
    got = fma_f32(np.float32(1.0) + np.float32(2.0 ** -23), e, one)
    assert got == np.nextafter(one, np.float32(2))
    # a * b = 2^-24 exactly, c = 1 -> the tie itself: even (1.0)
    assert fma_f32(one, e, one) == one
    assert fma_f32(e, eps, one) == one


# ---------------------------------------------------------------------------
# oracle vs torch's CPU kernels
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("N", [1, 3, 4, 7, 8, 12, 16, 20, 24, 25, 28, 32, 40, 96])
def test_spmm_oracle_matches_torch_sparse_mm(N):
    g = torch.Generator().manual_seed(N)
    X, K = 20, 300
    dense = torch.zeros(X, K)
    for r in range(X):
        nz = int(torch.randint(0, 23, (1,), generator=g))
        dense[r, torch.randperm(K, generator=g)[:nz]] = torch.randn(nz, generator=g) * 30
    dense[3, :] = 0
    dense[5, :280] = torch.randn(280, generator=g)  # a long row
    csr = dense.to_sparse_csr()
    B = torch.randn(K, N, generator=g)
    B[7] = -0.0
    want = torch.sparse.mm(csr, B).numpy()
    got = oracle.spmm_csr(csr.values().numpy(), csr.col_indices().to(torch.int32).numpy(),
                          csr.crow_indices().to(torch.int32).numpy(), B.numpy(),
                          weight_layout="ck")
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _ref_filter(x: torch.Tensor, threshold, max_pct):
    """The reference's filter_outlier body on torch CPU tensors
    (``quantized.py:1007-1042``), restated for widths the fixtures lack."""
    is_out = torch.abs(x) > threshold
    inl = torch.where(is_out, 0, x)
    outl = torch.where(is_out, x, 0)
    R, C = x.shape[-2:]
    max_nnz = int(R * C * max_pct)
    flat = outl.reshape(-1, R, C)
    ds, ixs, ps = [], [], []
    for i in range(flat.shape[0]):
        csr = flat[i].to_sparse_csr()
        crow = csr.crow_indices().to(torch.int32)
        col = csr.col_indices().to(torch.int32)
        val = csr.values()
        nse = int(crow[-1])
        if max_nnz >= nse:
            val = torch.nn.functional.pad(val, (0, max_nnz - nse))
            col = torch.nn.functional.pad(col, (0, max_nnz - nse), value=-1)
        else:
            crow = crow.clamp(max=max_nnz)
            val, col = val[:max_nnz], col[:max_nnz]
        ds.append(val)
        ixs.append(col)
        ps.append(crow)
    b = x.shape[:-2]
    return (torch.stack(ds).reshape(*b, -1), torch.stack(ixs).reshape(*b, -1),
            torch.stack(ps).reshape(*b, -1), inl)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape,thr,pct", [((7, 5), 0.8, 0.3), ((2, 9, 33), 1.7, 0.05),
                                           ((40, 1), 0.1, 0.5), ((16, 16), -0.5, 1.0),
                                           ((12, 20), 1.0, 0.0), ((3, 30, 17), 2.2, 0.002)])
def test_filter_oracle_matches_torch(dtype, shape, thr, pct):
    g = torch.Generator().manual_seed(len(shape) * 100 + shape[-1])
    x = (torch.randn(shape, generator=g) * 1.5).to(dtype)
    x.view(-1)[:4] = torch.tensor([0.0, -0.0, float("nan"), float("inf")]).to(dtype)
    want = _ref_filter(x, thr, pct)
    got = oracle.filter_outlier(_bits(x), thr, pct)
    for gg, ww in zip(got, want):
        w = _bits(ww)
        assert gg.shape == w.shape and gg.dtype == w.dtype
        assert np.array_equal(np.asarray(gg).view(np.uint8), np.ascontiguousarray(w).view(np.uint8))


def test_threshold_rounds_to_the_tensor_dtype():
    # 3.703125 is bf16(3.7): not an outlier of a bfloat16 tensor at 3.7, but
    # it is one of a float32 tensor
    xb = f32_to_bf16_bits(np.array([[3.703125, 3.6875, -3.75]], dtype=np.float32))
    assert oracle.filter_outlier(xb, 3.7, 1.0)[2].tolist() == [0, 1]
    xf = np.array([[3.703125, 3.6875, -3.75]], dtype=np.float32)
    assert oracle.filter_outlier(xf, 3.7, 1.0)[2].tolist() == [0, 2]


# ---------------------------------------------------------------------------
# C ABI (host only)
# ---------------------------------------------------------------------------
def _t(shape, dtype=_lib.VQ_BF16, ptr=0x1000):
    v = _lib.VqTensor()
    v.data = ptr
    v.dtype = dtype
    v.ndim = len(shape)
    for i, s in enumerate(shape):
        v.shape[i] = s
    return v


def _lo1_model(threshold, dtype):
    t32 = np.float32(threshold)
    if dtype == _lib.VQ_BF16:
        tb = f32_to_bf16_bits(np.array([t32], dtype=np.float32))[0]
        if np.isnan(bf16_bits_to_f32(np.array([tb]))[0]):
            return 0x8000
        if (tb & 0x8000) and (tb & 0x7FFF):
            return 0
        return int(tb & 0x7FFF) + 1
    u = int(np.array([t32]).view(np.uint32)[0])
    if np.isnan(t32):
        return 0x80000000
    if (u & 0x80000000) and (u & 0x7FFFFFFF):
        return 0
    return (u & 0x7FFFFFFF) + 1


def test_threshold_bits_host():
    lib = _lib.load()
    rng = np.random.default_rng(3)
    ths = [0.0, -0.0, 1.0, -1.0, 3.7, 1.00390625 + 1e-12, 1e-45, -1e-45, 1e38, 3.5e38,
           float("inf"), float("-inf"), float("nan"), 2.0 ** -130]
    ths += list(rng.standard_normal(200) * 10.0 ** rng.integers(-8, 8, 200))
    for t in ths:
        for dt in (_lib.VQ_BF16, _lib.VQ_F32):
            assert lib.vq_outlier_threshold_bits(t, dt) == _lo1_model(t, dt), (t, dt)


def test_threshold_bits_agree_with_torch_compare():
    """The bit test lo1 <= |x| <= inf equals torch's |x| > threshold for all
    65,536 bfloat16 patterns."""
    lib = _lib.load()
    x = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    ab = (np.arange(65536, dtype=np.uint32) & 0x7FFF)
    for t in (0.0, -0.0, 0.5, 3.7, -2.0, 1e-40, float("inf"), float("nan"), 65504.0):
        lo1 = lib.vq_outlier_threshold_bits(t, _lib.VQ_BF16)
        mine = (ab >= lo1) & (ab <= 0x7F80)
        want = (torch.abs(x) > t).numpy()
        assert np.array_equal(mine, want), t


def test_outlier_entries_reject_bad_arguments():
    lib = _lib.load()
    B = ctypes.byref
    ws = 0x2000
    # a 1-D input is not a matrix
    assert lib.vq_filter_outlier(B(_t([64])), 1.0, 4, 0, 0x10, 0x20, 0x30, None, ws, 1 << 20,
                                 0x40, None) == 1
    # float16 is not provided
    assert lib.vq_filter_outlier(B(_t([8, 8], _lib.VQ_F16)), 1.0, 4, 0, 0x10, 0x20, 0x30, None,
                                 ws, 1 << 20, 0x40, None) == 2
    # too little workspace
    need = lib.vq_filter_outlier_workspace_bytes(B(_t([3, 64, 4096])))
    assert need == (2 * 3 * 32 + 3) * 4 + 16  # tiles of 8192 bf16 elements
    assert lib.vq_filter_outlier(B(_t([3, 64, 4096])), 1.0, 4, 0, 0x10, 0x20, 0x30, None, ws,
                                 need - 1, 0x40, None) == 8
    # missing row pointers / workspace
    assert lib.vq_filter_outlier(B(_t([8, 8])), 1.0, 4, 0, 0x10, 0x20, 0x30, None, None,
                                 1 << 20, None, None) == 6
    assert lib.vq_filter_outlier(B(_t([8, 8])), 1.0, 4, 0, 0x10, 0x20, None, None, ws, 1 << 20,
                                 0x40, None) == 6
    # negative capacity
    assert lib.vq_filter_outlier(B(_t([8, 8])), 1.0, -1, 0, 0x10, 0x20, 0x30, None, ws,
                                 1 << 20, 0x40, None) == 1
    # spmm: output shape and batch mismatches, dtype mismatch
    d = _t([2, 16])
    assert lib.vq_spmm_csr(B(d), 0x10, 0x20, 5, B(_t([32, 8])), B(_t([2, 4, 8])), 0x30,
                           None) == 5
    assert lib.vq_spmm_csr(B(d), 0x10, 0x20, 5, B(_t([3, 32, 8])), B(_t([2, 5, 8])), 0x30,
                           None) == 5
    assert lib.vq_spmm_csr(B(d), 0x10, 0x20, 5, B(_t([32, 8])),
                           B(_t([2, 5, 8], _lib.VQ_F32)), 0x30, None) == 2
    # slice: bad dim, row window outside the matrix, negative column start
    d1 = _t([16])
    assert lib.vq_slice_csr(B(d1), 0x10, 0x20, 8, 2, 0, 4, 16, 0x30, 0x40, 0x50, 0x60,
                            None) == 1
    assert lib.vq_slice_csr(B(d1), 0x10, 0x20, 8, 0, 5, 9, 16, 0x30, 0x40, 0x50, 0x60,
                            None) == 1
    assert lib.vq_slice_csr(B(d1), 0x10, 0x20, 8, 1, -1, 9, 16, 0x30, 0x40, 0x50, 0x60,
                            None) == 1
    # transpose: wrong output shape
    assert lib.vq_transpose(B(_t([4, 6])), B(_t([4, 6])), None) == 5
    # masked quantize: NULL codes
    r = _lib.VqRounder()
    assert lib.vq_quantize_mx_masked(B(_t([4, 32])), B(r), 32, 448.0, 1, 8, None, 1.0,
                                     B(_t([4, 1])), None, None, None, None) == 6


def test_meta_shapes_follow_the_reference_fakes():
    import voyager_b200  # noqa: F401

    Q = torch.ops.quantized_ops
    x = torch.empty(2, 8, 64, device="meta", dtype=torch.bfloat16)
    d, i, p, inl = Q.filter_outlier(x, 1.0, 0.05)
    assert d.shape == (2, 25) and i.dtype == torch.int32 and p.shape == (2, 9)
    assert inl.shape == x.shape
    e4 = torch.empty(65536, device="meta", dtype=torch.bfloat16)
    outs = Q.quantize_mx_outlier(x, e4, [-1], 32, 448.0, True, threshold=2.0)
    assert [tuple(o.shape) for o in outs] == [(2, 5), (2, 5), (2, 9), (2, 8, 2), (2, 8, 64)]
    w = torch.empty(96, 64, device="meta", dtype=torch.bfloat16)
    assert Q.spmm_csr(d, i, p, w).shape == (2, 8, 96)
    assert Q.spmm_csr(d, i, p, w.t(), weight_layout="ck").shape == (2, 8, 96)
    d1, i1, p1 = Q.slice_csr_tensor(d[0], i[0], p[0], 0, 2, 6)
    assert p1.shape == (5,)
