"""Bounded device waits run out safely and report it.

Every spin in this library's kernels is limited by %globaltimer and ends
with an error code instead of a trap.  Here the tensor-parallel flag
barrier runs on one GPU as rank 0 of 2 with a wait limit of a few
milliseconds: rank 1's flag is never set (its "peer" array is a buffer of
this GPU that nothing reads), so that wait must give up, write 100 + 1 into
the launch's error word and into the library's sticky device word, and
leave the context usable.  No fault, trap or hang is involved."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import voyager_b200  # noqa: F401

    yield


def _barrier(mine, fake_peer, epoch, timeout_ns):
    from voyager_b200 import _lib
    from voyager_b200.ops import _stream

    dev = mine.device
    ptrs = torch.tensor([mine.data_ptr(), fake_peer.data_ptr()], dtype=torch.int64, device=dev)
    err = torch.full((1,), -1, dtype=torch.int32, device=dev)
    err.zero_()
    st = _lib.load().vq_tp_barrier_ex(ptrs.data_ptr(), mine.data_ptr(), 0, 2, epoch, timeout_ns,
                                      err.data_ptr(), _stream(dev))
    assert st == 0, _lib.STATUS.get(st, st)
    torch.cuda.synchronize()
    return int(err.item())


def test_barrier_wait_runs_out_and_reports():
    import voyager_b200
    from voyager_b200 import _lib

    voyager_b200.check_errors()  # start from a clear word
    mine = torch.zeros(64, dtype=torch.int32, device="cuda")
    peer = torch.zeros(64, dtype=torch.int32, device="cuda")
    # rank 1 never arrives: the wait on mine[1] gives up after 2 ms
    assert _barrier(mine, peer, 1, 2_000_000) == 101
    # rank 0's own arrival and the store for rank 1 still happened
    assert int(mine[0].item()) == 1 and int(peer[0].item()) == 1
    code = ctypes.c_int32(0)
    lib = _lib.load()
    assert lib.vq_device_errors(ctypes.byref(code), 0, None) == 0
    assert code.value == 101
    with pytest.raises(_lib.VqError, match="code 101"):
        voyager_b200.check_errors()
    # cleared by the check; the context still works
    assert lib.vq_device_errors(ctypes.byref(code), 0, None) == 0
    assert code.value == 0
    # with rank 1's flag at the epoch, the same barrier passes
    mine[1] = 2
    assert _barrier(mine, peer, 2, 2_000_000) == 0
    voyager_b200.check_errors()


def _barrier_dev(ptrs_list, mine, counter, rank, timeout_ns):
    from voyager_b200 import _lib
    from voyager_b200.ops import _stream

    dev = mine.device
    ptrs = torch.tensor(ptrs_list, dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = _lib.load().vq_tp_barrier_dev(ptrs.data_ptr(), mine.data_ptr(), rank, len(ptrs_list),
                                       counter.data_ptr(), timeout_ns, err.data_ptr(),
                                       _stream(dev))
    assert st == 0, _lib.STATUS.get(st, st)
    torch.cuda.synchronize()
    return int(err.item())


def test_device_epoch_barrier():
    """The barrier whose epoch lives on the device (the form a captured CUDA
    graph can replay): one rank passes at once and advances its counter;
    rank 0 of 2 whose peer never arrives gives up after its limit with
    code 101, and the counter still advances by one per call."""
    import voyager_b200

    voyager_b200.check_errors()
    mine = torch.zeros(64, dtype=torch.int32, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i in range(3):
        assert _barrier_dev([mine.data_ptr()], mine, counter, 0, 2_000_000) == 0
        assert int(counter.item()) == i + 1 and int(mine[0].item()) == i + 1
    mine.zero_()
    counter.zero_()
    peer = torch.zeros(64, dtype=torch.int32, device="cuda")
    assert _barrier_dev([mine.data_ptr(), peer.data_ptr()], mine, counter, 0, 2_000_000) == 101
    assert int(counter.item()) == 1 and int(mine[0].item()) == 1 and int(peer[0].item()) == 1
    assert _barrier_dev([mine.data_ptr(), peer.data_ptr()], mine, counter, 0, 2_000_000) == 101
    assert int(counter.item()) == 2 and int(peer[0].item()) == 2
    with pytest.raises(Exception):
        voyager_b200.check_errors()  # the sticky word holds the timeout
    voyager_b200.check_errors()
