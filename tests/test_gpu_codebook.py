"""Codebook quantize / decode on CUDA against the oracle: region grids
([*counts, k], one table per region of the tensor), index outputs (bounds),
and float32 codebooks whose entries bfloat16 cannot hold.  Bit-exact."""

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_dev, to_np

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


def _levels(shape, seed, bf16):
    v = np.sort(np.random.default_rng(seed).standard_normal(shape).astype(np.float32), axis=-1)
    return oracle.f32_to_bf16_bits(v) if bf16 else v


def _same(got, want):
    assert got.shape == want.shape and got.dtype == want.dtype, (got.shape, want.shape)
    bad = G.bit_mismatches(got, want)
    assert len(bad) == 0, f"{len(bad)} mismatches, first at {bad[:5]}"


CASES = [  # input shape, codebook shape
    ((2, 4, 8, 32), (1, 4, 1, 1, 16)),   # one table per head
    ((2, 4, 8, 32), (2, 2, 1, 2, 8)),    # a grid over three axes
    ((8, 64), (1, 4, 8)),                # groups of 16 channels
    ((6, 40), (3, 5, 4)),
    ((33, 16), (16,)),                   # 1-D
]


@pytest.mark.parametrize("xdtype", ["bf16", "f32"])
@pytest.mark.parametrize("cb_bf16", [True, False])
@pytest.mark.parametrize("shape,cshape", CASES)
def test_quantize_codebook(shape, cshape, cb_bf16, xdtype):
    rng = np.random.default_rng(sum(shape) + len(cshape))
    x = rng.standard_normal(shape).astype(np.float32) * 1.5
    x = oracle.f32_to_bf16_bits(x) if xdtype == "bf16" else x
    scale = np.array(0.75, dtype=np.float32)
    cb = _levels(cshape, len(shape) * 7 + cshape[-1], cb_bf16)
    got = to_np(Q.quantize(to_dev(x), to_dev(scale), qmap=to_dev(cb)))
    _same(got, oracle.quantize(x, scale, qmap=cb))
    # the index variant (bounds = the midpoints, as a compiled graph stores them)
    bounds = oracle.ops.codebook_edges(cb)
    bounds = oracle.f32_to_bf16_bits(bounds) if cb_bf16 else bounds
    got = to_np(Q.quantize(to_dev(x), to_dev(scale), qmap=to_dev(cb), output_code=to_dev(bounds)))
    _same(got, oracle.quantize(x, scale, qmap=cb, output_code=bounds))


def test_region_grid_must_fit():
    x = to_dev(np.zeros((6, 40), dtype=np.float32))
    cb = to_dev(_levels((4, 5, 4), 1, False))  # 4 does not divide 6
    with pytest.raises(ValueError):
        Q.quantize(x, to_dev(np.array(1.0, dtype=np.float32)), qmap=cb)
    with pytest.raises(ValueError):
        # a grid of three axes on a 2-D tensor
        Q.quantize(x, to_dev(np.array(1.0, dtype=np.float32)), qmap=to_dev(_levels((1, 1, 2, 4), 2, False)))


@pytest.mark.parametrize("cb_bf16", [True, False])
def test_decode_region_grid_through_linear(cb_bf16):
    rng = np.random.default_rng(5)
    idx = oracle.f32_to_bf16_bits(rng.integers(0, 8, size=(24, 64)).astype(np.float32))
    xa = oracle.f32_to_bf16_bits(rng.standard_normal((16, 64)).astype(np.float32))
    code = _levels((4, 1, 8), 9, cb_bf16)
    got = to_np(Q.linear_mx(to_dev(xa), to_dev(idx), None, weight_code=to_dev(code)))
    want = oracle.linear_mx(xa, idx, None, weight_code=code)
    assert G.rel_l2(got, want) < 1e-3
    # the decoded weight itself, bit for bit
    from voyager_b200 import codebook as cbm

    dec = to_np(cbm.decode(to_dev(idx), to_dev(code)))
    _same(dec, oracle.ops.decode(idx, code))


def test_decode_float32_codes_of_float32_entries():
    """float32 indices through a float32 codebook whose entries are not
    bfloat16 values: the per-region path keeps them exact."""
    from voyager_b200 import codebook as cbm

    idx = np.random.default_rng(2).integers(0, 16, size=(8, 32)).astype(np.float32)
    code = _levels((16,), 4, False)
    _same(to_np(cbm.decode(to_dev(idx), to_dev(code))), oracle.ops.decode(idx, code))
