"""The C ABI: the library loads without a GPU, exports every entry point the
header declares, and rejects bad arguments with a status before any launch
(host pointers are never dereferenced on those paths)."""

import ctypes
import os
import re

import numpy as np
import pytest

import _golden as G
from voyager_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "voyager_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(vq_[a-z0-9_]+)\s*\(", src)))


def test_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared()
    assert "vq_quantize_mx" in names and "vq_rounder_from_table" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the binding declares a signature for each of them
    assert set(names) <= set(_lib.exported_symbols())


def test_status_strings():
    lib = _lib.load()
    for code, text in _lib.STATUS.items():
        assert lib.vq_status_string(code).decode() == text
    assert lib.vq_version().decode().startswith("voyager_b200")


@pytest.mark.parametrize("name", [k for k in G.tables() if k != "lut4_index"])
def test_classifier_exact(name):
    """Every reference table becomes a rounder equal to it on all inputs
    (analytic kinds evaluated on the host with the device's code)."""
    lib = _lib.load()
    t = np.ascontiguousarray(G.tables()[name])
    r = _lib.VqRounder()
    assert lib.vq_rounder_from_table(t.ctypes.data, ctypes.byref(r)) == 0
    if r.kind == _lib.VQ_R_TABLE:
        return
    got = np.array([lib.vq_rounder_eval_host(ctypes.byref(r), i) for i in range(65536)],
                   dtype=np.uint16)
    assert np.array_equal(got, t)


def test_classifier_kinds():
    lib = _lib.load()
    expect = {"fp4_e2m1": _lib.VQ_R_MINIFLOAT, "fp8_e4m3": _lib.VQ_R_MINIFLOAT,
              "int8": _lib.VQ_R_INT, "uint4": _lib.VQ_R_INT, "posit8_1": _lib.VQ_R_POSIT,
              "lut4": _lib.VQ_R_STEP, "identity": _lib.VQ_R_IDENTITY}
    for name, kind in expect.items():
        t = np.ascontiguousarray(G.tables()[name])
        r = _lib.VqRounder()
        lib.vq_rounder_from_table(t.ctypes.data, ctypes.byref(r))
        assert r.kind == kind, (name, r.describe())
    # hardware-conversion candidates for the tensor-core formats
    for name, hw in (("fp8_e4m3", 1), ("fp8_e5m2", 2), ("fp4_e2m1", 3), ("fp6_e2m3", 0)):
        t = np.ascontiguousarray(G.tables()[name])
        r = _lib.VqRounder()
        lib.vq_rounder_from_table(t.ctypes.data, ctypes.byref(r))
        assert r.hw == hw, name


def test_random_table_stays_table():
    lib = _lib.load()
    t = np.random.default_rng(0).integers(0, 65536, 65536).astype(np.uint16)
    r = _lib.VqRounder()
    assert lib.vq_rounder_from_table(t.ctypes.data, ctypes.byref(r)) == 0
    assert r.kind == _lib.VQ_R_TABLE


def _t(shape, dtype=_lib.VQ_BF16, data=0x1000):
    v = _lib.VqTensor()
    v.data = data
    v.dtype = dtype
    v.ndim = len(shape)
    for i, s in enumerate(shape):
        v.shape[i] = s
    return v


def _rounder():
    r = _lib.VqRounder()
    r.kind = _lib.VQ_R_IDENTITY
    return r


def test_quantize_rejects_bad_arguments():
    lib = _lib.load()
    B = ctypes.byref
    x, s, r = _t([4, 8]), _t([]), _rounder()
    # NULL qmap / input
    assert lib.vq_quantize(B(x), B(s), None, 0, None, B(_t([4, 8])), None) == 6
    assert lib.vq_quantize(None, B(s), None, 0, B(r), B(_t([4, 8])), None) == 6
    # output dtype must be the promoted one (bf16 / 0-d f32 -> bf16)
    assert lib.vq_quantize(B(x), B(_t([], _lib.VQ_F32)), None, 0, B(r),
                           B(_t([4, 8], _lib.VQ_F32)), None) == 1
    # output shape
    assert lib.vq_quantize(B(x), B(s), None, 0, B(r), B(_t([4, 9])), None) == 5
    # scale that does not broadcast
    assert lib.vq_quantize(B(x), B(_t([3, 8])), None, 0, B(r), B(_t([4, 8])), None) == 5
    # expand() cannot cover the input: [4, 1] blocks of 4 on 8 columns
    assert lib.vq_quantize(B(x), B(_t([4, 1])), None, 4, B(r), B(_t([4, 8])), None) == 5
    # unsupported dtype
    assert lib.vq_quantize(B(_t([4, 8], _lib.VQ_F16)), B(s), None, 0, B(r),
                           B(_t([4, 8], _lib.VQ_F16)), None) == 2
    # a TABLE rounder without its table
    bad = _lib.VqRounder()
    bad.kind = _lib.VQ_R_TABLE
    assert lib.vq_quantize(B(x), B(s), None, 0, B(bad), B(_t([4, 8])), None) == 6


def test_mx_rejects_bad_arguments():
    lib = _lib.load()
    B = ctypes.byref
    x, r = _t([4, 32]), _rounder()
    axes = (ctypes.c_int64 * 1)(-1)
    # block size 0
    assert lib.vq_quantize_mx(B(x), B(r), axes, 1, 0, 6.0, 0, 0, None, B(_t([4, 2])),
                              B(_t([4, 32])), None) == 1
    # axis out of range
    bad_axes = (ctypes.c_int64 * 1)(5)
    assert lib.vq_quantize_mx(B(x), B(r), bad_axes, 1, 16, 6.0, 0, 0, None, B(_t([4, 2])),
                              B(_t([4, 32])), None) == 1
    # wrong scale shape (ceil(32/16) = 2 blocks)
    assert lib.vq_quantize_mx(B(x), B(r), axes, 1, 16, 6.0, 0, 0, None, B(_t([4, 3])),
                              B(_t([4, 32])), None) == 5
    # scale dtype must be the input's
    assert lib.vq_calculate_mx_qparam(B(x), axes, 1, 16, 6.0, 0, 0, None,
                                      B(_t([4, 2], _lib.VQ_F32)), None) == 1
    # empty input: nothing to launch
    assert lib.vq_calculate_mx_qparam(B(_t([0, 32])), axes, 1, 16, 6.0, 0, 0, None,
                                      B(_t([0, 2])), None) == 0


def test_table_kinds_fit_the_byte_coded_form():
    """The kinds the kernels evaluate from shared memory (TABLE, POSIT,
    STEP) are staged as byte codes into a 256-entry palette when the table
    has at most 256 distinct patterns: every such reference table does but
    posit16_1 (7,168 patterns), which keeps the 128 KB bf16 form.  The
    palette gathers back to the table exactly."""
    lib = _lib.load()
    staged = (_lib.VQ_R_TABLE, _lib.VQ_R_POSIT, _lib.VQ_R_STEP)
    wide = []
    for name, t in G.tables().items():
        if name == "lut4_index":
            continue
        t = np.ascontiguousarray(t)
        r = _lib.VqRounder()
        assert lib.vq_rounder_from_table(t.ctypes.data, ctypes.byref(r)) == 0
        if r.kind not in staged:
            continue
        uniq, inv = np.unique(t, return_inverse=True)
        if uniq.size > 256:
            wide.append(name)
            continue
        pal = np.zeros(256, dtype=np.uint16)
        pal[:uniq.size] = uniq
        assert np.array_equal(pal[inv.astype(np.uint8).reshape(-1)], t), name
    assert wide == ["posit16_1"], wide


def test_noalloc_rejects_before_touching_its_scratch():
    """vq_linear_mxf8_noalloc refuses what the GEMM would refuse before it
    packs into the shared array (no device pointer is touched here)."""
    lib = _lib.load()
    B = ctypes.byref
    a, s = _t([64, 256]), _t([64, 8])
    w, wsf, out = 0x10000, 0x20000, 0x30000
    # N not a multiple of 8
    assert lib.vq_linear_mxf8_noalloc(B(a), B(s), w, wsf, 12, None, out, 16, None) == 2
    # ldo below N, and not a multiple of 8
    assert lib.vq_linear_mxf8_noalloc(B(a), B(s), w, wsf, 16, None, out, 8, None) == 2
    assert lib.vq_linear_mxf8_noalloc(B(a), B(s), w, wsf, 16, None, out, 20, None) == 2
    # misaligned output, weight or scale atoms, odd bias address
    assert lib.vq_linear_mxf8_noalloc(B(a), B(s), w, wsf, 16, None, out + 8, 16, None) == 3
    assert lib.vq_linear_mxf8_noalloc(B(a), B(s), w + 4, wsf, 16, None, out, 16, None) == 3
    assert lib.vq_linear_mxf8_noalloc(B(a), B(s), w, wsf + 2, 16, None, out, 16, None) == 3
    assert lib.vq_linear_mxf8_noalloc(B(a), B(s), w, wsf, 16, 0x40001, out, 16, None) == 3
    # NULL status pointer
    assert lib.vq_linear_mxf8_noalloc_status(None, None) == 6
    assert lib.vq_device_errors(None, 0, None) == 6


def test_barrier_rejects_bad_limits():
    lib = _lib.load()
    flags, mine, err = 0x10000, 0x20000, 0x30000
    # the wait limit must lie in [1 us, 10 s]; checked before the launch
    assert lib.vq_tp_barrier_ex(flags, mine, 0, 2, 1, 999, err, None) == 1
    assert lib.vq_tp_barrier_ex(flags, mine, 0, 2, 1, 10_000_000_001, err, None) == 1
    assert lib.vq_tp_barrier_ex(flags, mine, 2, 2, 1, 10**6, err, None) == 1
    assert lib.vq_tp_barrier_ex(None, mine, 0, 2, 1, 10**6, err, None) == 6
