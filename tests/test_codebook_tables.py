"""The codebook tables the library builds on the host (voyager_b200.codebook)
against the oracle's encode / decode, on the CPU: every bf16 pattern through
every region's table, for bfloat16 and float32 codebooks, entry and index
outputs.  On the GPU, vq_codebook_lookup only gathers from these tables (its
own parity tests run there)."""

import numpy as np
import pytest
import torch

import oracle
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits


def _levels(shape, seed, bf16):
    v = np.sort(np.random.default_rng(seed).standard_normal(shape).astype(np.float32), axis=-1)
    return f32_to_bf16_bits(v) if bf16 else v


def _torch(a):
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(a.copy())


def _bits(t):
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


ALL = np.arange(65536, dtype=np.uint32).astype(np.uint16)


@pytest.mark.parametrize("cb_bf16", [True, False])
@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("index", [False, True])
def test_encode_tables_match_oracle(cb_bf16, out, index):
    from voyager_b200 import codebook as cbm

    R, k = 3, 8
    cb = _levels((R, 1, k), 11 + R, cb_bf16)
    # row r of x: every bf16 pattern, quantized against region r's codebook
    x = np.tile(ALL, (R, 1))
    xs = x if out == "bf16" else bf16_bits_to_f32(x)
    bounds = oracle.ops.codebook_edges(cb) if index else None
    want = oracle.ops._encode(xs, cb, bounds)
    dt = torch.bfloat16 if out == "bf16" else torch.float32
    got = cbm.encode_tables(_torch(cb), None if bounds is None else torch.from_numpy(bounds), dt,
                            "cpu").reshape(R, 65536)
    g, w = _bits(got), want
    nan = np.isnan(bf16_bits_to_f32(g) if g.dtype == np.uint16 else g) & \
        np.isnan(bf16_bits_to_f32(w) if w.dtype == np.uint16 else w)
    assert np.array_equal(g[~nan], w[~nan])


@pytest.mark.parametrize("cb_bf16", [True, False])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_decode_tables_match_oracle(cb_bf16, dtype):
    from voyager_b200 import codebook as cbm

    R, k = 4, 16
    cb = _levels((R, 1, k), 5, cb_bf16)
    idx = np.tile(np.arange(k, dtype=np.float32), (R, 1))
    xs = f32_to_bf16_bits(idx) if dtype == "bf16" else idx
    want = oracle.ops.decode(xs, cb)
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    table = cbm.decode_tables(_torch(cb), dt, "cpu").reshape(R, 65536)
    pat = f32_to_bf16_bits(np.arange(k, dtype=np.float32)).astype(np.int64)
    assert np.array_equal(_bits(table[:, pat]), want)


def test_region_counts_errors_match_oracle():
    from voyager_b200 import codebook as cbm

    cb = torch.zeros((4, 5, 4))
    with pytest.raises(ValueError):
        cbm.region_counts(cb, (6, 40))          # 4 does not divide 6
    with pytest.raises(ValueError):
        oracle.ops.region_view(np.zeros((6, 40)), (4, 5))
    with pytest.raises(ValueError):
        cbm.region_counts(torch.zeros((1, 1, 2, 4)), (6, 40))  # three axes on a 2-D tensor
    assert cbm.region_counts(cb, (8, 40)) == [4, 5]
    assert cbm.region_counts(torch.zeros(16), (3, 7)) == [1, 1]
