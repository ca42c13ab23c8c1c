"""Host-side policies and argument checks of the newer entry points, on CPU
(no kernel runs: every call here is decided or rejected before any launch).

* ``vq_gemm_dq_splits``: the K-split count of the bf16 dequant GEMM -- split
  only GEMMs with fewer output tiles than CTA pairs, never batched ones, and
  never when the float32 slices would cost more than the tail they recover.
* ``vq_gemm_dq_ex``, ``vq_stream_probe``, ``vq_amax_observe``: bad arguments
  come back as status codes."""

import ctypes

import pytest

from voyager_b200 import _lib

VQ_OK, VQ_ERR_INVALID, VQ_ERR_UNSUPPORTED, VQ_ERR_ALIGNMENT, VQ_ERR_NULL = 0, 1, 2, 3, 6


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_split_choice(lib):
    # C4's M = 128 points with 16 output tiles split; 56 tiles do not gain
    assert lib.vq_gemm_dq_splits(1, 128, 4096, 4096) > 1
    assert lib.vq_gemm_dq_splits(1, 128, 4096, 14336) > 1
    assert lib.vq_gemm_dq_splits(1, 128, 14336, 4096) == 1
    # a wave of tiles or more, or a batch: no split
    assert lib.vq_gemm_dq_splits(1, 1024, 4096, 4096) == 1
    assert lib.vq_gemm_dq_splits(1, 8192, 11008, 4096) == 1
    assert lib.vq_gemm_dq_splits(2, 128, 4096, 4096) == 1
    # every split divides the K steps into slices of at least 8 steps
    for M, N, K in [(128, 4096, 4096), (16, 4096, 4096), (64, 512, 14336), (8, 1024, 8192)]:
        s = lib.vq_gemm_dq_splits(1, M, N, K)
        ks = (K + 63) // 64
        assert s >= 1 and ks % s == 0 and (s == 1 or ks // s >= 8)
    # nonsense sizes: no split rather than an error
    assert lib.vq_gemm_dq_splits(0, 128, 4096, 4096) == 1


def _dq_ex(lib, batch=1, M=128, K=4096, N=4096, splits=4, ws=64):
    # fake, 16-byte aligned device addresses: rejected calls never use them
    a, w, out, err = 1 << 20, 2 << 20, 3 << 20, 4 << 20
    return lib.vq_gemm_dq_ex(a, batch, M, K, 0, w, 1, N, None, None, None, out, N, M * N,
                             splits, ws, err, None)


def test_gemm_dq_ex_rejects(lib):
    assert _dq_ex(lib, splits=0) == VQ_ERR_INVALID
    assert _dq_ex(lib, splits=3) == VQ_ERR_INVALID        # 64 K steps do not split in 3
    assert _dq_ex(lib, batch=2, splits=4) == VQ_ERR_UNSUPPORTED
    assert _dq_ex(lib, ws=None) == VQ_ERR_NULL
    assert _dq_ex(lib, ws=(5 << 20) + 8) == VQ_ERR_ALIGNMENT


def test_stream_probe_rejects(lib):
    assert lib.vq_stream_probe(None, -16, None, 0, None) == VQ_ERR_INVALID
    assert lib.vq_stream_probe(None, 16, None, 0, None) == VQ_ERR_NULL
    assert lib.vq_stream_probe(1 << 20, 17, None, 0, None) == VQ_ERR_ALIGNMENT
    assert lib.vq_stream_probe((1 << 20) + 8, 16, None, 0, None) == VQ_ERR_ALIGNMENT
    assert lib.vq_stream_probe(None, 0, None, 0, None) == VQ_OK  # nothing to move


def _vt(shape, dtype=_lib.VQ_F32, data=1 << 20):
    v = _lib.VqTensor()
    v.data = data
    v.dtype = dtype
    v.ndim = len(shape)
    for i, s in enumerate(shape):
        v.shape[i] = s
    return v


def test_amax_observe_rejects(lib):
    hist, scale, ws = 2 << 20, 3 << 20, 4 << 20
    call = lambda t, per_ch=0, axis=0, L=1, h=hist, ws_=ws: lib.vq_amax_observe(
        ctypes.byref(t), per_ch, axis, h, L, scale, 127.0, 0, 0, ws_, None)
    assert call(_vt([4, 4]), h=None) == VQ_ERR_NULL
    assert call(_vt([4, 4]), ws_=None) == VQ_ERR_NULL
    assert call(_vt([4, 4], dtype=_lib.VQ_I32)) == VQ_ERR_UNSUPPORTED
    assert call(_vt([0, 4])) == VQ_ERR_INVALID              # amax of nothing
    assert call(_vt([4, 4]), L=0) == VQ_ERR_INVALID
    assert call(_vt([4, 4]), per_ch=1, axis=2) == VQ_ERR_INVALID
    assert call(_vt([]), per_ch=1, axis=0) == VQ_ERR_INVALID  # 0-d has no channel axis
    assert call(_vt([4, 4], data=(1 << 20) + 2)) == VQ_ERR_ALIGNMENT
