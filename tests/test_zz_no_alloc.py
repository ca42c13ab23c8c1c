"""The allocation-free MXFP8 linear entry point, vq_linear_mxf8_noalloc.

Some callers cannot call cudaMalloc: a runtime with its own fixed memory
pool, code that runs under a strict memory budget, or a hook invoked where
allocation is forbidden.  This entry point packs the activations into a
fixed device array inside the library instead of caller- or
allocator-provided scratch, then runs the same tcgen05 kernel.  The test
calls it through the C ABI and checks it against the allocating path
(mxgemm.linear -> vq_mx_pack + vq_gemm_mxf8) on two calls in a row, with
the tolerance of the other GEMM tests (rel-L2 <= 1e-3; the kernels are the
same, so the results are expected to be identical).

It lives in its own file so that it is collected last."""

import ctypes

import numpy as np
import pytest
import torch

import _golden as G
import oracle
from _tt import to_dev, to_np
from oracle.numerics import quantization_map

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def _mx(rng, shape, std):
    from voyager_b200.synth import f32_to_bf16_bits

    x = f32_to_bf16_bits((rng.standard_normal(shape) * std).astype(np.float32))
    s, c = oracle.quantize_mx(x, quantization_map("fp8_e4m3"), [-1], 32, 448.0, True)
    return c, s


def _noalloc(ca, sa, pw, pws, n, bias=None):
    from voyager_b200 import _lib
    from voyager_b200.ops import _ref, _stream, _vt

    a, s = to_dev(ca), to_dev(sa)
    out = torch.empty((a.shape[0], n), dtype=torch.bfloat16, device="cuda")
    st = _lib.load().vq_linear_mxf8_noalloc(
        _ref(_vt(a)), _ref(_vt(s)), pw.data_ptr(), pws.data_ptr(), n,
        None if bias is None else bias.data_ptr(), out.data_ptr(), n,
        _stream(torch.device("cuda")))
    assert st == 0, _lib.STATUS.get(st, st)
    torch.cuda.synchronize()
    return to_np(out)


def _status():
    from voyager_b200 import _lib
    from voyager_b200.ops import _stream

    code = ctypes.c_int32(-1)
    st = _lib.load().vq_linear_mxf8_noalloc_status(ctypes.byref(code),
                                                   _stream(torch.device("cuda")))
    assert st == 0, _lib.STATUS.get(st, st)
    return code.value


def test_noalloc_matches_allocating_path_twice():
    from voyager_b200 import mxgemm

    rng = np.random.default_rng(2024)
    K, N = 4096, 1536
    cw, sw = _mx(rng, (N, K), 0.02)
    dcw, dsw = to_dev(cw), to_dev(sw)
    pw, pws, ok = mxgemm.packed_weight(dcw, dsw)
    assert ok
    from voyager_b200.synth import f32_to_bf16_bits

    bias = f32_to_bf16_bits((rng.standard_normal(N) * 0.5).astype(np.float32))
    for m, b in ((300, None), (77, bias)):  # two calls in a row, different shapes and data
        ca, sa = _mx(rng, (m, K), 1.0)
        db = None if b is None else to_dev(b)
        want = to_np(mxgemm.linear(to_dev(ca), dcw, db, to_dev(sa), dsw))
        got = _noalloc(ca, sa, pw, pws, N, db)
        assert got.shape == want.shape
        assert G.rel_l2(got, want) < 1e-3
        ref = oracle.linear_mx(ca, cw, b, input_scale=sa, weight_scale=sw, block_size=32)
        assert G.rel_l2(got, ref) < 1e-3
        # the kernel's error word in the fixed array: no bounded wait gave up
        assert _status() == 0


def test_noalloc_rejects_oversize():
    from voyager_b200 import _lib
    from voyager_b200.ops import _ref, _vt

    # 4096 x 8192 codes pack to 32 MiB, over the 16 MiB scratch: rejected
    # before anything is launched
    a = torch.zeros((4096, 8192), dtype=torch.bfloat16, device="cuda")
    s = torch.ones((4096, 256), dtype=torch.bfloat16, device="cuda")
    dummy = torch.empty(16, dtype=torch.uint8, device="cuda")
    out = torch.empty((4096, 8), dtype=torch.bfloat16, device="cuda")
    st = _lib.load().vq_linear_mxf8_noalloc(_ref(_vt(a)), _ref(_vt(s)), dummy.data_ptr(),
                                            dummy.data_ptr(), 8, None, out.data_ptr(), 8, None)
    assert st == 8
