"""The outlier CSR side-stream of quantized_ops, restated in numpy.

Test infrastructure only (see ``oracle/__init__.py``).

Follows ``src/voyager_compiler/ops/quantized.py``: ``_pad_csr`` (:964-990),
``filter_outlier`` (:995-1045), ``quantize_mx_outlier`` (:1078-1130),
``slice_csr_tensor`` (:1173-1216), ``spmm_csr`` (:1245-1311) and the
``A_data`` branch of ``linear_mx`` / ``matmul_mx`` (:560-572, :623-635).

Arithmetic that torch supplies, restated:
* ``torch.abs(x) > threshold`` compares in the tensor's dtype, so the Python
  float is rounded to float32 and, for bfloat16, again to bfloat16;
* ``Tensor.to_sparse_csr`` keeps the nonzero elements in row-major order;
* ``torch.sparse.mm`` (CPU, float32; MKL's sparse kernel in the reference's
  torch build) accumulates each output row over the row's entries in CSR
  order, starting from +0: as a chain of fused multiply-adds, except for
  output widths 4, 8, ..., 24, where the rounded products are added in pairs,
  four entries per step, with its own order for the last one to three
  entries (``_row_pairs``).  Both were found by comparing candidate orders
  with torch's outputs bit for bit, and are pinned by the golden cases.
"""

import math

import numpy as np

from oracle.numerics import BF16, dtype_of, f32_to_bf16_bits, round_to, to_f32
from oracle.ops import dequantize_mx, quantize_mx


def _threshold_as(threshold: float, dt: str) -> np.float32:
    t = np.float32(threshold)
    if dt == BF16:
        return to_f32(f32_to_bf16_bits(np.array(t, dtype=np.float32)))[()]
    return t


def _pad_csr(values, cols, crow, max_nnz):
    """``quantized.py:964-990``: pad to ``max_nnz`` with value 0 / column -1,
    or drop the entries past it and clamp the row pointers."""
    nse = int(crow[-1])
    pad = max_nnz - nse
    if pad >= 0:
        data = np.concatenate([values, np.zeros(pad, dtype=values.dtype)])
        idx = np.concatenate([cols.astype(np.int32), np.full(pad, -1, dtype=np.int32)])
        return data, idx, crow
    crow = np.minimum(crow, max_nnz).astype(np.int32)
    return values[:max_nnz], cols[:max_nnz].astype(np.int32), crow


def filter_outlier(x: np.ndarray, threshold: float, max_pct: float = 0.01):
    """``quantized.py:995-1045`` -> ``(data, indices, indptr, inliers)``."""
    x = np.asarray(x)
    dt = dtype_of(x)
    xf = to_f32(x)
    thr = _threshold_as(threshold, dt)
    with np.errstate(invalid="ignore"):
        is_out = np.abs(xf) > thr
    zero = np.zeros((), dtype=x.dtype)
    inliers = np.where(is_out, zero, x).astype(x.dtype)
    batch = x.shape[:-2]
    R, C = x.shape[-2], x.shape[-1]
    max_nnz = int(math.prod(x.shape[-2:]) * max_pct)
    nb = int(math.prod(batch))
    xs = x.reshape(nb, R, C)
    keep = (is_out & (xf != 0)).reshape(nb, R, C)
    datas, idxs, ptrs = [], [], []
    for b in range(nb):
        rows, cols = np.nonzero(keep[b])
        vals = xs[b][rows, cols]
        counts = np.bincount(rows, minlength=R)
        crow = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        d, i, p = _pad_csr(vals, cols, crow, max_nnz)
        datas.append(d)
        idxs.append(i)
        ptrs.append(p)
    data = np.stack(datas).reshape(*batch, -1)
    indices = np.stack(idxs).reshape(*batch, -1)
    indptr = np.stack(ptrs).reshape(*batch, -1)
    return data, indices, indptr, inliers


def quantize_mx_outlier(x, qmap, axes, block_size, quant_max, force_scale_power_of_two=False,
                        scale_qmap=None, output_code=None, threshold=None, max_pct=0.01,
                        indptr_offset=0):
    """``quantized.py:1078-1130`` -> ``(data, indices, indptr, scale, codes)``."""
    data, indices, indptr, inliers = filter_outlier(x, threshold, max_pct)
    if indptr_offset:
        indptr = (indptr.astype(np.int64) + int(indptr_offset)).astype(np.int32)
    scale, codes = quantize_mx(inliers, qmap, axes, block_size, quant_max,
                               force_scale_power_of_two, scale_qmap, output_code)
    return data, indices, indptr, scale, codes


def slice_csr_tensor(data, indices, indptr, dim=0, start=None, end=None, size_factor=1.0):
    """``quantized.py:1173-1216``."""
    dim = dim + 2 if dim < 0 else dim
    if dim not in (0, 1):
        raise ValueError(f"Cannot slice sparse CSR matrix along dim {dim}")
    data, indices, indptr = np.asarray(data), np.asarray(indices), np.asarray(indptr)
    if dim == 0:
        s, e = int(indptr[start]), int(indptr[end])
        new_indptr = (indptr[start:end + 1].astype(np.int64) - s).astype(np.int32)
        values, cols = data[s:e], indices[s:e]
    else:
        mask = (indices >= start) & (indices < end)
        lengths = np.diff(indptr.astype(np.int64))
        nse = int(indptr[-1])
        m = mask[:nse].astype(np.int64)
        bounds = np.concatenate([[0], np.cumsum(lengths)])
        counts = np.array([m[bounds[r]:bounds[r + 1]].sum() for r in range(len(lengths))],
                          dtype=np.int64)
        new_indptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        values = data[mask]
        cols = (indices[mask].astype(np.int64) - start).astype(np.int32)
    max_nnz = int(data.shape[0] * size_factor)
    return _pad_csr(values, cols, new_indptr, max_nnz)


def fma_f32(a, b, c):
    """float32 ``a * b + c`` rounded once (round-half-even), elementwise:
    the product is exact in float64; the float64 sum's error term decides
    the float32 rounding where that sum lands exactly between two floats."""
    a = np.asarray(a, dtype=np.float32).astype(np.float64)
    b = np.asarray(b, dtype=np.float32).astype(np.float64)
    c = np.asarray(c, dtype=np.float32).astype(np.float64)
    with np.errstate(all="ignore"):
        p = a * b
        s = p + c
        bb = s - p
        t = (p - (s - bb)) + (c - bb)  # p + c == s + t exactly (when finite)
        r = s.astype(np.float32)
        d = s - r.astype(np.float64)
        up = np.nextafter(r, np.float32(np.inf))
        dn = np.nextafter(r, np.float32(-np.inf))
        half_up = (up.astype(np.float64) - r.astype(np.float64)) / 2
        half_dn = (r.astype(np.float64) - dn.astype(np.float64)) / 2
        fin = np.isfinite(s) & np.isfinite(t) & np.isfinite(r)
        tie_above = fin & (t != 0) & (d == half_up) & (t > 0)  # exact value past the tie
        tie_below = fin & (t != 0) & (d == -half_dn) & (t < 0)
    r = np.where(tie_above, up, r)
    r = np.where(tie_below, dn, r)
    return r.astype(np.float32)


def _mul(a, b):
    return (np.float32(a) * np.asarray(b, dtype=np.float32)).astype(np.float32)


def _add(a, b):
    with np.errstate(all="ignore"):
        return (np.asarray(a, dtype=np.float32) + np.asarray(b, dtype=np.float32)).astype(
            np.float32)


def _row_fma(vals, rows, N):
    acc = np.zeros(N, dtype=np.float32)
    for v, b in zip(vals, rows):
        acc = fma_f32(v, b, acc)
    return acc


def _row_pairs(vals, rows, N):
    """Widths 4..24 (multiples of 4): ``acc += p0 + p1; acc += p2 + p3`` per
    four entries, then the last n % 4 as ``+p``, ``+p +p`` or
    ``(acc + p2) + (p0 + p1)``."""
    acc = np.zeros(N, dtype=np.float32)
    n = len(vals)
    q = n // 4 * 4
    p = [_mul(v, b) for v, b in zip(vals, rows)]
    for j in range(0, q, 2):
        acc = _add(acc, _add(p[j], p[j + 1]))
    r = n - q
    if r == 1:
        acc = _add(acc, p[q])
    elif r == 2:
        acc = _add(_add(acc, p[q]), p[q + 1])
    elif r == 3:
        acc = _add(_add(acc, p[q + 2]), _add(p[q], p[q + 1]))
    return acc


def spmm_csr(data, indices, indptr, B, B_scale=None, B_code=None, block_size=None,
             weight_layout="kc"):
    """``quantized.py:1245-1311``: B decoded and scaled (in B's dtype), a
    KC-stored B transposed, then each CSR batch times B in float32, rounded
    to B's dtype."""
    assert weight_layout in ("kc", "ck"), weight_layout
    Bd = dequantize_mx(np.asarray(B), B_scale, B_code, block_size)
    out_dt = dtype_of(Bd)
    Bf = to_f32(Bd)
    if weight_layout == "kc":
        Bf = np.swapaxes(Bf, -1, -2)
    indptr, indices, data = np.asarray(indptr), np.asarray(indices), np.asarray(data)
    batch = indptr.shape[:-1]
    nb = int(math.prod(batch))
    ip = indptr.reshape(-1, indptr.shape[-1]).astype(np.int64)
    ix = indices.reshape(-1, indices.shape[-1]).astype(np.int64)
    dv = data.reshape(-1, data.shape[-1])
    if Bf.ndim > 2:
        Bf = Bf.reshape(nb, Bf.shape[-2], Bf.shape[-1])
    X = ip.shape[1] - 1
    L = dv.shape[1]
    outs = []
    for i in range(nb):
        Bb = Bf[i] if Bf.ndim == 3 else Bf
        K, N = Bb.shape
        crow = np.clip(ip[i] - ip[i][0], 0, L)
        crow = np.maximum.accumulate(crow)
        end = int(crow[-1])
        cols = np.clip(ix[i, :end], 0, K - 1)
        vals = to_f32(dv[i, :end])
        o = np.zeros((X, N), dtype=np.float32)
        row = _row_pairs if (N % 4 == 0 and 4 <= N <= 24) else _row_fma
        for r in range(X):
            a, b = int(crow[r]), int(crow[r + 1])
            o[r] = row(vals[a:b], Bb[cols[a:b]], N)
        outs.append(o)
    out = np.stack(outs).reshape(*batch, X, -1)
    return round_to(out, out_dt)


def add_spmm(dense, sp):
    """``dense_out + spmm_out`` (``quantized.py:572``) of two tensors of one
    dtype."""
    dt = dtype_of(dense)
    with np.errstate(all="ignore"):
        return round_to((to_f32(dense) + to_f32(sp)).astype(np.float32), dt)
