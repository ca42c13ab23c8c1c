"""The CPU oracle against the reference's own outputs (golden fixtures).

Pins the oracle before it is trusted as the checker for the CUDA path:
every value table exhaustively, the block-scale maps exhaustively over
bfloat16 amax values, and every small op case bit for bit.
"""

import numpy as np
import pytest

import _golden as G
import oracle
from oracle.numerics import quantization_map

TABLES = [k for k in G.tables() if k != "lut4_index"]


@pytest.mark.parametrize("name", TABLES)
def test_table_exhaustive(name):
    mine = quantization_map(None if name == "identity" else name)
    assert len(G.bit_mismatches(mine, G.tables()[name])) == 0
    # NaN payloads too: the tables must be identical bit for bit.
    assert np.array_equal(mine, G.tables()[name])


def test_lut4_index_table():
    from oracle.numerics import index_table

    assert np.array_equal(index_table(quantization_map("lut4")), G.tables()["lut4_index"])


def _map_cases():
    return [k for k in G.scale_maps() if k != "f32_inputs"]


@pytest.mark.parametrize("key", _map_cases())
def test_scale_map(key):
    m = G.scale_maps()
    if "_bf16_" in key:
        x = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(-1, 1)
    else:
        x = m["f32_inputs"].reshape(-1, 1)
    kind, _, rest = key.split("_", 2)
    if kind == "pow2":
        got = oracle.calculate_mx_qparam(x, [-1], 1, float(rest), True)
    else:
        parts = rest.split("_", 1)
        sq = None if len(parts) == 1 or parts[1] == "None" else quantization_map(parts[1])
        got = oracle.calculate_mx_qparam(x, [-1], 1, float(parts[0]), False, sq)
    assert len(G.bit_mismatches(got.reshape(-1), m[key])) == 0


CASES = G.small_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_small_case(case):
    ins, kw, outs = G.resolve_case(case)
    fn = getattr(oracle, case["op"])
    r = fn(*ins) if case["op"] == "vmap" else fn(*ins, **kw)
    got = list(r) if isinstance(r, tuple) else [r]
    assert len(got) == len(outs)
    for g, w in zip(got, outs):
        assert g.shape == w.shape and g.dtype == w.dtype
        if case["op"] in ("linear_mx", "matmul_mx", "sdpa_mx"):
            # The reference's CPU bf16 GEMM (and softmax) sums in its own
            # order (sdpa_mx: 0-1 differing elements per case, rel-L2 < 2e-5).
            assert G.rel_l2(g, w) < 1e-3
        else:
            assert len(G.bit_mismatches(g, w)) == 0
