"""The quantized_ops numerics, restated in numpy.

Test infrastructure only (see ``oracle/__init__.py``).

Each function follows the reference op of the same name in
``src/voyager_compiler/ops/quantized.py`` and reproduces torch's eager CPU
rounding at every op boundary: binary ops are evaluated in float32 and
rounded once to the result dtype; a 0-d scale does not take part in type
promotion (its float32 value is used unrounded); ``vmap`` rounds its input to
bfloat16 (NaN -> ``0xFFFF``) before the gather and casts table entries to
bfloat16 before widening back.
"""

import math
from concurrent.futures import ThreadPoolExecutor
from typing import List, Optional, Sequence

import numpy as np

from oracle.numerics import (
    BF16,
    F32,
    QMAP_SIZE,
    bf16_bits_to_f32,
    dtype_of,
    f32_to_bf16_bits,
    round_to,
    to_f32,
)

FP32_MIN_NORMAL = np.float32(2.0**-126)


def _promote(a: np.ndarray, b: np.ndarray) -> str:
    """Result dtype of ``a (op) b`` under torch's rules for float operands:
    a 0-d operand does not promote a dimensioned one."""
    da, db = dtype_of(a), dtype_of(b)
    if np.ndim(b) == 0 and np.ndim(a) > 0:
        return da
    if np.ndim(a) == 0 and np.ndim(b) > 0:
        return db
    return F32 if F32 in (da, db) else BF16


def _binary(a, b, op):
    r = _promote(a, b)
    with np.errstate(all="ignore"):
        out = op(to_f32(a), to_f32(b)).astype(np.float32)
    return round_to(out, r)


def table_as_bf16(qmap: np.ndarray) -> np.ndarray:
    """A table's entries as bfloat16 bits (``vmap`` assigns them into a
    bfloat16 tensor, ``quantized.py:199-201``)."""
    q = np.asarray(qmap)
    if q.dtype == np.uint16:
        return q
    return f32_to_bf16_bits(q.astype(np.float32))


# ---------------------------------------------------------------------------
def expand(scale: np.ndarray, shape: Sequence[int], block_size: int) -> np.ndarray:
    """``quantized.py:158-171``: repeat along every dim whose size differs,
    then slice the ragged tail."""
    s = np.asarray(scale)
    while s.ndim < len(shape):
        s = s[None]
    for d in range(len(shape)):
        if s.shape[d] != shape[d]:
            s = np.repeat(s, block_size, axis=d)
    if list(s.shape) != list(shape):
        s = s[tuple(slice(0, x) for x in shape)]
    return s


def vmap(x: np.ndarray, qmap: np.ndarray) -> np.ndarray:
    """``quantized.py:174-203``: gather by the bfloat16 bit pattern."""
    d = dtype_of(x)
    idx = x if d == BF16 else f32_to_bf16_bits(x)
    out = table_as_bf16(qmap)[np.asarray(idx, dtype=np.uint16)]
    return out if d == BF16 else bf16_bits_to_f32(out)


def codebook_edges(cb: np.ndarray) -> np.ndarray:
    """``(codebook[..., :-1] + codebook[..., 1:]) / 2`` in the codebook's
    dtype (``quantized.py:292-293``): a bfloat16 codebook rounds the sum to
    bfloat16 (the halving is then exact), a float32 one stays float32."""
    cb = np.asarray(cb)
    if cb.dtype == np.uint16:
        s = f32_to_bf16_bits((to_f32(cb[..., :-1]) + to_f32(cb[..., 1:])).astype(np.float32))
        return to_f32(f32_to_bf16_bits((to_f32(s) / np.float32(2)).astype(np.float32)))
    c = cb.astype(np.float32)
    return ((c[..., :-1] + c[..., 1:]) / np.float32(2)).astype(np.float32)


def region_view(x: np.ndarray, counts):
    """``_region_view`` (``quantized.py:211-248``): the tensor split into
    ``counts[i]`` regions along each axis, region axes first; returns the
    view and the permutation that puts the axes back."""
    counts = tuple(counts)
    if len(counts) != x.ndim:
        raise ValueError(
            f"a {list(counts)} region codebook tiles {len(counts)} axes, "
            f"but the tensor reaching it has {x.ndim}")
    if any(e % c for e, c in zip(x.shape, counts)):
        raise ValueError(
            f"a {list(counts)} region codebook does not divide the {list(x.shape)} tensor "
            "reaching it")
    split = []
    for e, c in zip(x.shape, counts):
        split += [c, e // c]
    order = list(range(0, 2 * len(counts), 2)) + list(range(1, 2 * len(counts), 2))
    inverse = [0] * len(order)
    for pos, ax in enumerate(order):
        inverse[ax] = pos
    return x.reshape(split).transpose(order), inverse


def _encode(x: np.ndarray, codebook: np.ndarray, bounds) -> np.ndarray:
    """``quantized.py:251-309``: search the midpoints of the bfloat16-rounded
    input; return the entry, or the index when ``bounds`` are given.  A
    codebook ``[*counts, k]`` holds one table per region of the input."""
    cb = np.asarray(codebook)
    cbf = to_f32(cb) if cb.dtype == np.uint16 else cb.astype(np.float32)
    edges = codebook_edges(cb) if bounds is None else to_f32(np.asarray(bounds))
    xr = bf16_bits_to_f32(f32_to_bf16_bits(to_f32(x)))
    if cb.ndim == 1:
        index = np.searchsorted(edges, xr, side="left")
        picked = index.astype(np.float32) if bounds is not None else cbf[index]
        return round_to(picked.astype(np.float32), dtype_of(x))
    moved, inverse = region_view(xr, cb.shape[:-1])
    regions = cb.size // cb.shape[-1]
    flat = moved.reshape(regions, -1)
    table = cbf.reshape(regions, -1)
    edge = edges.reshape(regions, -1)
    out = np.empty(flat.shape, dtype=np.float32)
    for r in range(regions):
        index = np.searchsorted(edge[r], flat[r], side="left")
        out[r] = index.astype(np.float32) if bounds is not None else table[r][index]
    out = out.reshape(moved.shape).transpose(inverse).reshape(np.shape(x))
    return round_to(out, dtype_of(x))


def decode(x: np.ndarray, codebook: np.ndarray) -> np.ndarray:
    """``quantized.py:312-337``: each stored index read back as its entry
    (one table per region for a ``[*counts, k]`` codebook), in the input's
    dtype."""
    cb = np.asarray(codebook)
    cbf = to_f32(cb) if cb.dtype == np.uint16 else cb.astype(np.float32)
    idx = to_f32(x).astype(np.int64)
    if cb.ndim == 1:
        return round_to(cbf[idx], dtype_of(x))
    moved, inverse = region_view(idx, cb.shape[:-1])
    regions = cb.size // cb.shape[-1]
    table = cbf.reshape(regions, -1)
    picked = np.take_along_axis(table, moved.reshape(regions, -1), axis=1)
    picked = picked.reshape(moved.shape).transpose(inverse).reshape(idx.shape)
    return round_to(picked.astype(np.float32), dtype_of(x))


def quantize(
    x: np.ndarray,
    scale: np.ndarray,
    zero_point: Optional[np.ndarray] = None,
    axes=None,
    block_size: Optional[int] = None,
    qmap: Optional[np.ndarray] = None,
    output_code: Optional[np.ndarray] = None,
) -> np.ndarray:
    """``quantized.py:340-397``."""
    assert qmap is not None
    if block_size is not None:
        scale = expand(scale, x.shape, block_size)
        if zero_point is not None:
            zero_point = expand(zero_point, x.shape, block_size)
    t = _binary(x, scale, np.divide)
    if zero_point is not None:
        t = _binary(t, zero_point, np.add)
    q = np.asarray(qmap)
    if q.size == QMAP_SIZE and q.ndim == 1:
        return vmap(t, q)
    return _encode(t, q, output_code)


def dequantize(
    x: np.ndarray,
    scale: np.ndarray,
    zero_point: Optional[np.ndarray] = None,
    axes=None,
    block_size: Optional[int] = None,
    input_qmap: Optional[np.ndarray] = None,
    output_qmap: Optional[np.ndarray] = None,
) -> np.ndarray:
    """``quantized.py:400-452``."""
    if input_qmap is not None:
        x = vmap(x, input_qmap)
    if block_size is not None:
        scale = expand(scale, x.shape, block_size)
        if zero_point is not None:
            zero_point = expand(zero_point, x.shape, block_size)
    if zero_point is None:
        y = _binary(x, scale, np.multiply)
    else:
        y = _binary(_binary(x, zero_point, np.subtract), scale, np.multiply)
    if output_qmap is not None:
        y = vmap(y, output_qmap)
    return y


# ---------------------------------------------------------------------------
def _norm_axes(axes, ndim) -> List[int]:
    axes = [axes] if isinstance(axes, int) else list(axes)
    return sorted(a + ndim if a < 0 else a for a in axes)


def _reshape_to_blocks(a: np.ndarray, axes: List[int], bs: int):
    """``mx_utils.py:68-127``: a block axis after each blocked axis, the
    ragged tail zero-padded."""
    shape = list(a.shape)
    pad = [(0, 0)] * a.ndim
    for ax in axes:
        if shape[ax] % bs:
            pad[ax] = (0, bs - shape[ax] % bs)
    if any(p[1] for p in pad):
        a = np.pad(a, pad, mode="constant")
    new_shape = []
    for d, n in enumerate(a.shape):
        if d in axes:
            if n >= bs:
                new_shape += [n // bs, bs]
            else:
                new_shape += [1, n]
        else:
            new_shape.append(n)
    reduce_axes = []
    shift = 0
    for d in range(a.ndim):
        if d in axes:
            reduce_axes.append(d + shift + 1)
            shift += 1
    return a.reshape(new_shape), reduce_axes


def _abs_max(blocked: np.ndarray, reduce_axes: List[int], dtype: str) -> np.ndarray:
    """NaN-propagating max of |x| over the block axes, in the input dtype."""
    if dtype == BF16:
        mag = (blocked & np.uint16(0x7FFF)).astype(np.uint16)
        # Non-negative bfloat16 order equals integer order; every NaN
        # pattern sorts above +inf, so an integer max propagates NaN.
        m = mag.max(axis=tuple(reduce_axes))
        return m.astype(np.uint16)
    with np.errstate(invalid="ignore"):
        return np.max(np.abs(blocked), axis=tuple(reduce_axes)).astype(np.float32)


def _floor_log2_of(amax: np.ndarray, dtype: str) -> np.ndarray:
    """``mx_utils.py:48-53``: ``floor(log2(amax + 2^-126 * (amax == 0)))``,
    with the log2 rounded to ``dtype`` before the floor."""
    a = to_f32(amax)
    with np.errstate(all="ignore"):
        a = np.where(a == 0, FP32_MIN_NORMAL, a).astype(np.float32)
        lg = np.log2(a).astype(np.float32)
        lg = to_f32(round_to(lg, dtype))
        return np.floor(lg).astype(np.float32)


def calculate_mx_qparam(
    x: np.ndarray,
    axes,
    block_size: int,
    quant_max: float,
    force_scale_power_of_two: bool = False,
    scale_qmap: Optional[np.ndarray] = None,
) -> np.ndarray:
    """``quantized.py:787-851``."""
    assert block_size > 0
    d = dtype_of(x)
    axes = _norm_axes(axes, x.ndim)
    blocked, red = _reshape_to_blocks(np.asarray(x), axes, block_size)
    amax = _abs_max(blocked, red, d)
    if force_scale_power_of_two:
        shexp = _floor_log2_of(amax, d)
        shexp = to_f32(round_to(shexp - np.float32(np.floor(np.log2(quant_max))), d))
        with np.errstate(all="ignore"):
            scale = round_to(np.power(np.float32(2), shexp).astype(np.float32), d)
    else:
        with np.errstate(all="ignore"):
            scale = round_to(to_f32(amax) / np.float32(quant_max), d)
        if scale_qmap is not None:
            scale = vmap(scale, scale_qmap)
    sf = to_f32(scale)
    with np.errstate(invalid="ignore"):
        keep = sf > 0
    return np.where(keep, scale, round_to(np.float32(1.0), d)).astype(scale.dtype)


def quantize_mx(
    x: np.ndarray,
    qmap: np.ndarray,
    axes,
    block_size: int,
    quant_max: float,
    force_scale_power_of_two: bool = False,
    scale_qmap: Optional[np.ndarray] = None,
    output_code: Optional[np.ndarray] = None,
):
    """``quantized.py:854-881`` -> ``(scale, codes)``."""
    scale = calculate_mx_qparam(
        x, axes, block_size, quant_max, force_scale_power_of_two, scale_qmap
    )
    codes = quantize(x, scale, None, axes, block_size, qmap, output_code)
    return scale, codes


def quantize_mx_threaded(x, qmap, axes, block_size, quant_max, pow2=False,
                         scale_qmap=None, threads: int = 8):
    """``quantize_mx`` over row chunks on ``threads`` host threads (numpy
    releases the GIL in its kernels).  Blocks run along the last axis only."""
    assert list(_norm_axes(axes, x.ndim)) == [x.ndim - 1]
    rows = x.reshape(-1, x.shape[-1])
    n = rows.shape[0]
    bounds = np.linspace(0, n, threads + 1).astype(int)

    def work(i):
        lo, hi = bounds[i], bounds[i + 1]
        return quantize_mx(rows[lo:hi], qmap, [-1], block_size, quant_max, pow2, scale_qmap)

    with ThreadPoolExecutor(threads) as ex:
        parts = list(ex.map(work, range(threads)))
    s = np.concatenate([p[0] for p in parts])
    c = np.concatenate([p[1] for p in parts])
    return s.reshape(x.shape[:-1] + (s.shape[-1],)), c.reshape(x.shape)


def quantize_affine(x, qmap, axes, block_size, quant_min, quant_max, scale_qmap=None):
    """``quantized.py:884-948``: per-block min/max -> scale, zero point, codes."""
    (axis,) = axes
    d = dtype_of(x)
    ax = [axis % x.ndim]
    blocked, red = _reshape_to_blocks(np.asarray(x), ax, block_size)
    v = to_f32(blocked)
    with np.errstate(all="ignore"):
        low = round_to(np.min(v, axis=tuple(red)), d)
        high = round_to(np.max(v, axis=tuple(red)), d)
        scale = round_to(
            to_f32(round_to(to_f32(high) - to_f32(low), d))
            / np.float32(quant_max - quant_min), d)
        one = round_to(np.float32(1.0), d)
        scale = np.where(to_f32(scale) > 0, scale, one).astype(scale.dtype)
        if scale_qmap is not None:
            scale = vmap(scale, scale_qmap)
            scale = np.where(to_f32(scale) > 0, scale, one).astype(scale.dtype)
        neg = round_to(-to_f32(low), d)
        zp = round_to(to_f32(round_to(to_f32(neg) / to_f32(scale), d)) + np.float32(quant_min), d)
        if scale_qmap is not None:
            zp = vmap(zp, scale_qmap)
    value = quantize(x, scale, zp, ax, block_size, qmap)
    return scale, zp, value


# ---------------------------------------------------------------------------
def dequantize_mx(x, scale, code, block_size):
    """``quantized.py:455-472`` (``_dequantize_mx`` / ``_decode_and_scale``)."""
    if code is None and scale is None:
        return x
    if code is not None:
        x = decode(x, code)
    if scale is not None:
        x = _binary(x, expand(scale, x.shape, block_size), np.multiply)
    return x


def _with_outliers(dense, A_data, A_indices, A_indptr, weight, weight_scale, weight_code,
                   block_size, weight_layout):
    """``dense_out + spmm_csr(A_*, weight, ...)`` (``quantized.py:560-572``)."""
    if A_data is None:
        return dense
    from oracle.outlier import add_spmm, spmm_csr

    sp = spmm_csr(A_data, A_indices, A_indptr, weight, weight_scale, weight_code, block_size,
                  weight_layout)
    return add_spmm(dense, sp)


def linear_mx(x, weight, bias=None, *, input_scale=None, weight_scale=None,
              block_size=None, input_code=None, weight_code=None, A_data=None,
              A_indices=None, A_indptr=None, weight_layout="kc",
              out_fp32=False) -> np.ndarray:
    """``quantized.py:522-574``: dequantize both operands, then a GEMM that
    accumulates in float32 and rounds once to the operands' dtype, as the
    reference's ``aten.linear`` does (plus the outlier CSR's ``spmm_csr``
    with the weight, when given).  ``out_fp32`` skips that rounding.
    GEMM results are compared within a relative-L2 tolerance, not bitwise:
    the summation order is the implementation's."""
    if A_data is not None:
        dense = linear_mx(x, weight, bias, input_scale=input_scale, weight_scale=weight_scale,
                          block_size=block_size, input_code=input_code,
                          weight_code=weight_code, weight_layout=weight_layout)
        return _with_outliers(dense, A_data, A_indices, A_indptr, weight, weight_scale,
                              weight_code, block_size, weight_layout)
    xa = dequantize_mx(x, input_scale, input_code, block_size)
    wa = dequantize_mx(weight, weight_scale, weight_code, block_size)
    a, w = to_f32(xa), to_f32(wa)
    if weight_layout == "ck":
        w = np.swapaxes(w, -1, -2)
    out = a.astype(np.float32) @ np.swapaxes(w, -1, -2).astype(np.float32)
    if bias is not None:
        out = out + to_f32(bias)
    out = out.astype(np.float32)
    if out_fp32:
        return out
    dt = BF16 if (dtype_of(xa) == BF16 and dtype_of(wa) == BF16) else F32
    return round_to(out, dt)


def matmul_mx(x, other, *, input_scale=None, weight_scale=None,
              block_size=None, input_code=None, weight_code=None, A_data=None,
              A_indices=None, A_indptr=None, weight_layout="ck",
              out_fp32=False) -> np.ndarray:
    """``quantized.py:589-637``; rounding and the outlier CSR as in
    ``linear_mx``."""
    if A_data is not None:
        dense = matmul_mx(x, other, input_scale=input_scale, weight_scale=weight_scale,
                          block_size=block_size, input_code=input_code,
                          weight_code=weight_code, weight_layout=weight_layout)
        return _with_outliers(dense, A_data, A_indices, A_indptr, other, weight_scale,
                              weight_code, block_size, weight_layout)
    xa = dequantize_mx(x, input_scale, input_code, block_size)
    ba = dequantize_mx(other, weight_scale, weight_code, block_size)
    a, b = to_f32(xa), to_f32(ba)
    if weight_layout == "kc":
        b = np.swapaxes(b, -1, -2)
    out = np.matmul(a.astype(np.float32), b.astype(np.float32)).astype(np.float32)
    if out_fp32:
        return out
    dt = BF16 if (dtype_of(xa) == BF16 and dtype_of(ba) == BF16) else F32
    return round_to(out, dt)


def _softmax_last(x_f32: np.ndarray) -> np.ndarray:
    """float32 softmax along the last axis: exp(x - max) / sum, every step in
    float32 (a row of -inf only gives NaN, as in torch)."""
    m = np.max(x_f32, axis=-1, keepdims=True)
    with np.errstate(invalid="ignore", over="ignore"):
        e = np.exp((x_f32 - m).astype(np.float32)).astype(np.float32)
        s = np.sum(e, axis=-1, keepdims=True, dtype=np.float32)
        return (e / s).astype(np.float32)


def _masked(scores: np.ndarray, mask) -> np.ndarray:
    """``quantized.py:772-780``: a bool mask keeps where true (-inf
    elsewhere), a float mask adds; scores are bf16 bits."""
    if mask is None:
        return scores
    mask = np.asarray(mask)
    if mask.dtype == np.bool_:
        neg = np.uint16(0xFF80) if scores.dtype == np.uint16 else np.float32(-np.inf)
        return np.where(mask, scores, neg).astype(scores.dtype)
    return _binary(scores, mask, np.add)


def sdpa_mx(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False,
            query_residual=None, key_residual=None, value_residual=None,
            residual_mask=None, *, scale=None, enable_gqa=False, query_scale=None,
            key_scale=None, value_scale=None, block_size=None, input_code=None,
            weight_code=None, probs_qmap=None, probs_quant_max=None,
            probs_scale_qmap=None, probs_code=None, force_scale_power_of_two=False):
    """``quantized.py:663-769``: dequantize the three operands, scores =
    bf16(bf16(q k^T) * scale) under the mask, softmax (float32 inside, bf16
    out), probabilities through ``quantize_mx`` along the keys and back,
    then ``probs @ v`` (float32 accumulation, bf16 out)."""
    if is_causal and attn_mask is not None:
        raise ValueError("is_causal excludes an explicit attn_mask")
    q = dequantize_mx(query, query_scale, input_code, block_size)
    k = dequantize_mx(key, key_scale, weight_code, block_size)
    v = dequantize_mx(value, value_scale, weight_code, block_size)
    d = dtype_of(q)
    residual = key_residual is not None
    if enable_gqa:
        g = q.shape[-3] // k.shape[-3]
        k, v = np.repeat(k, g, axis=-3), np.repeat(v, g, axis=-3)
        if residual:
            key_residual = np.repeat(key_residual, g, axis=-3)
            value_residual = np.repeat(value_residual, g, axis=-3)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    sc = np.float32(scale)
    raw = np.matmul(to_f32(q), np.swapaxes(to_f32(k), -1, -2)).astype(np.float32)
    scores = round_to(to_f32(round_to(raw, d)) * sc, d)
    if is_causal:
        attn_mask = np.tril(np.ones(scores.shape[-2:], dtype=np.bool_))
    scores = _masked(scores, attn_mask)
    keys = scores.shape[-1]
    if residual:
        rraw = np.matmul(to_f32(query_residual),
                         np.swapaxes(to_f32(key_residual), -1, -2)).astype(np.float32)
        rs = round_to(to_f32(round_to(rraw, d)) * sc, d)
        scores = np.concatenate([scores, _masked(rs, residual_mask)], axis=-1)
    probs = round_to(_softmax_last(to_f32(scores)), d)
    probs, rprobs = probs[..., :keys], probs[..., keys:]
    if probs_qmap is not None:
        ps, pc = quantize_mx(np.ascontiguousarray(probs), probs_qmap, [-1], block_size,
                             probs_quant_max, force_scale_power_of_two, probs_scale_qmap,
                             probs_code)
        probs = dequantize_mx(pc, ps, input_code, block_size)
    out = round_to(np.matmul(to_f32(probs), to_f32(v)).astype(np.float32), d)
    if residual:
        ro = round_to(np.matmul(to_f32(rprobs), to_f32(value_residual)).astype(np.float32), d)
        out = _binary(out, ro, np.add)
    return out
