"""Loading and comparing the golden fixtures under ``tests/golden/``."""

import json
import os
from functools import lru_cache

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


@lru_cache(None)
def tables():
    with np.load(os.path.join(GOLDEN, "tables.npz")) as z:
        return {k: z[k] for k in z.files}


@lru_cache(None)
def scale_maps():
    with np.load(os.path.join(GOLDEN, "scale_maps.npz")) as z:
        return {k: z[k] for k in z.files}


@lru_cache(None)
def _small():
    with open(os.path.join(GOLDEN, "ops_small.json")) as f:
        cases = json.load(f)
    with np.load(os.path.join(GOLDEN, "ops_small.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    return cases, arrays


def small_cases():
    return _small()[0]


def resolve_case(case):
    """-> (inputs list, kwargs dict, expected outputs list) as numpy."""
    _, arrays = _small()
    t = tables()
    inputs = [None if k is None else arrays[k] for k in case["inputs"]]
    kwargs = {}
    for k, v in case["kwargs"].items():
        if isinstance(v, dict) and "array" in v:
            kwargs[k] = arrays[v["array"]]
        elif isinstance(v, dict) and "table" in v:
            kwargs[k] = t[v["table"]]
        else:
            kwargs[k] = v
    outputs = [arrays[k] for k in case["outputs"]]
    return inputs, kwargs, outputs


@lru_cache(None)
def full_checksums():
    with open(os.path.join(GOLDEN, "full_checksums.json")) as f:
        return json.load(f)


def as_float(a):
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def bit_mismatches(got, want):
    """Positions that differ bit-for-bit, except that any NaN equals any NaN."""
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, (got.shape, want.shape)
    assert got.dtype == want.dtype, (got.dtype, want.dtype)
    g = got.view(np.uint8).reshape(got.size, -1) if got.size else got.reshape(0, 1)
    w = want.view(np.uint8).reshape(want.size, -1) if want.size else want.reshape(0, 1)
    bad = (g != w).any(axis=1)
    nan = np.isnan(as_float(got)).reshape(-1) & np.isnan(as_float(want)).reshape(-1)
    return np.where(bad & ~nan)[0]


def rel_l2(got, want):
    g = as_float(got).astype(np.float64)
    w = as_float(want).astype(np.float64)
    return float(np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30))
