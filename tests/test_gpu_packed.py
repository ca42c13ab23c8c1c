"""Packed MXFP8 storage on the device: operands quantized by the oracle,
packed in the GEMM layout (row_multiple 256 for the weight, 128 for the
activation), written to a VQMX file, loaded and registered with
packed.to_device, then multiplied by torch.ops.quantized_ops.linear_mx:
the product matches the oracle's linear_mx (rel-L2 < 1e-3), and the GEMM
reads the loaded bytes (the cache holds them; no packing again)."""

import os

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from oracle.numerics import quantization_map

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def _mx(rng, shape, std):
    x = oracle.f32_to_bf16_bits((rng.standard_normal(shape) * std).astype(np.float32))
    s, c = oracle.quantize_mx(x, quantization_map("fp8_e4m3"), [-1], 32, 448.0, True)
    return c, s


@pytest.mark.parametrize("verify", [True, False])
def test_loaded_operands_feed_the_gemm(tmp_path, verify, monkeypatch):
    from voyager_b200 import mxgemm, packed
    from _tt import to_np

    rng = np.random.default_rng(7)
    M, K, N = 300, 512, 264
    ca, sa = _mx(rng, (M, K), 1.0)
    cw, sw = _mx(rng, (N, K), 0.02)
    paths = []
    for name, (c, s), rm in (("a", (ca, sa), 128), ("w", (cw, sw), 256)):
        path = os.path.join(tmp_path, name + ".vqmx")
        packed.save(path, packed.pack_mxfp8(c, s, row_multiple=rm))
        paths.append(path)
    pa, pw = packed.load(paths[0]), packed.load(paths[1])
    da, dsa = packed.to_device(pa, "cuda", weight=False, verify=verify)
    dw, dsw = packed.to_device(pw, "cuda", weight=True, verify=verify)
    # the registered bytes are the loaded ones
    key = (dw._version, id(dsw), dsw._version)
    hit = mxgemm._wcache.get(dw, key)
    assert hit is not None and hit[2]
    assert np.array_equal(hit[0].cpu().numpy(), pw.codes)
    assert np.array_equal(hit[1].cpu().numpy(), pw.scales)
    entry = mxgemm._vouched_entry(da, dsa)
    assert entry is not None and np.array_equal(entry[1][0].cpu().numpy(), pa.codes)
    # the GEMM packs nothing more
    calls = {"n": 0}
    real = mxgemm._pack

    def counting(*a, **k):
        calls["n"] += 1
        return real(*a, **k)

    monkeypatch.setattr(mxgemm, "_pack", counting)
    got = to_np(torch.ops.quantized_ops.linear_mx(da, dw, None, input_scale=dsa,
                                                  weight_scale=dsw, block_size=32))
    assert calls["n"] == 0
    want = oracle.linear_mx(ca, cw, None, input_scale=sa, weight_scale=sw, block_size=32)
    assert G.rel_l2(got, want) < 1e-3


def test_unverified_nan_operand_is_not_registered():
    from voyager_b200 import mxgemm, packed

    rng = np.random.default_rng(8)
    ca, sa = _mx(rng, (128, 256), 1.0)
    ca[3, 5] = 0x7FFF  # a NaN code
    p = packed.pack_mxfp8(ca, sa, row_multiple=128)
    da, dsa = packed.to_device(p, "cuda", weight=False, verify=False)
    assert mxgemm._vouched_entry(da, dsa) is None
