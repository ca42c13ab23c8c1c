"""Symmetric-memory workspace for the tensor-parallel decoder.

One symmetric buffer per process group, mapped on every rank and bound to an
NVLS multicast object (``torch.distributed._symmetric_memory``): the
producer kernels of ``vq_tp.cu`` store through the multicast address, so one
store fills every rank's copy; ``barrier()`` is ``k_tp_barrier`` on flags at
the start of the same buffer (release / acquire, bounded wait).

Layout (byte offsets, each region 256-byte aligned):
  flags     uint32 [64]      this rank's barrier flags (one per peer)
  stats     float  [world, T]
  operands  named regions: E4M3 bytes [T, K] + UE8M0 atoms [K/128][T/128][512]
  raw       named byte regions (e.g. a GEMM output every rank fills)
"""

import os
from typing import Dict, Tuple

import torch
import torch.distributed as dist

from voyager_b200 import _lib

CHECK_ERRORS = os.environ.get("VQ_CHECK_ERRORS", "0") == "1"
BARRIER_WAIT_NS = 2_000_000_000  # a barrier wait gives up (and records it) after 2 s
_ALIGN = 256


def _up(n: int, a: int = _ALIGN) -> int:
    return (n + a - 1) // a * a


def multicast_available(group=None) -> bool:
    """Symmetric memory with an NVLS multicast address on this group."""
    try:
        import torch.distributed._symmetric_memory as symm_mem  # noqa: F401
        from torch._C._distributed_c10d import _SymmetricMemory
    except Exception:
        return False
    if not (dist.is_initialized() and torch.cuda.is_available()):
        return False
    from torch._C._autograd import DeviceType

    return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA,
                                                       torch.cuda.current_device()))


class Workspace:
    """The symmetric buffer of one group for T tokens and the named operand
    widths ``operands = {name: K}``."""

    def __init__(self, group, tokens: int, operands: Dict[str, int], device,
                 raw: Dict[str, int] = None):
        import torch.distributed._symmetric_memory as symm_mem

        group = group if group is not None else dist.group.WORLD
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T = tokens
        if tokens % 128:
            raise ValueError(f"token count {tokens} is not a multiple of 128")
        self.RT = tokens // 128
        off = _up(64 * 4)
        self.stats_off = off
        off += _up(self.world * tokens * 4)
        self.regions: Dict[str, Tuple[int, int, int]] = {}
        for name, K in operands.items():
            if K % 128:
                raise ValueError(f"operand {name}: width {K} is not a multiple of 128")
            p_off = off
            off += _up(tokens * K)
            a_off = off
            off += _up((K // 128) * self.RT * 512)
            self.regions[name] = (K, p_off, a_off)
        self.raw: Dict[str, int] = {}
        for name, nbytes in (raw or {}).items():
            self.raw[name] = off
            off += _up(nbytes)
        self.nbytes = off
        self.buf = symm_mem.empty(off, dtype=torch.uint8, device=device)
        self.buf[: _up(64 * 4)].zero_()
        self.handle = symm_mem.rendezvous(self.buf, group)
        self.base = self.buf.data_ptr()
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        # the tensor may start inside the symmetric allocation: peer and
        # multicast addresses of this tensor are the allocation's plus it
        delta = self.base - ptrs[self.rank]
        if int(self.handle.multicast_ptr) == 0:
            raise RuntimeError("symmetric memory has no multicast address on this group")
        self.mc = int(self.handle.multicast_ptr) + delta
        peers = [p + delta for p in ptrs]
        self.peer_flags = torch.tensor(peers, dtype=torch.int64, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        # the barrier epoch, kept on the device (graph replays advance it)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        # flags are zero everywhere before anyone signals
        torch.cuda.synchronize(device)
        dist.barrier(group)

    # addresses -----------------------------------------------------------
    def stats_mc(self) -> int:
        return self.mc + self.stats_off

    def stats_local(self) -> int:
        return self.base + self.stats_off

    def operand(self, name: str):
        """(K, local bytes, local atoms, multicast bytes, multicast atoms)."""
        K, p, a = self.regions[name]
        return K, self.base + p, self.base + a, self.mc + p, self.mc + a

    def raw_region(self, name: str):
        """(local address, multicast address) of a raw region."""
        off = self.raw[name]
        return self.base + off, self.mc + off

    def raw_tensor(self, name: str, shape, dtype) -> torch.Tensor:
        """The local copy of a raw region as a tensor (a view of the buffer)."""
        off = self.raw[name]
        n = 1
        for d in shape:
            n *= d
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        return self.buf[off:off + nbytes].view(dtype).view(*shape)

    # synchronisation -----------------------------------------------------
    def barrier(self, stream: int):
        st = _lib.load().vq_tp_barrier_dev(self.peer_flags.data_ptr(), self.base, self.rank,
                                           self.world, self.counter.data_ptr(), BARRIER_WAIT_NS,
                                           self.err.data_ptr(), stream)
        _lib.check(st, "tensor-parallel barrier")

    def check(self):
        e = int(self.err.item())
        if e:
            raise _lib.VqError(f"tensor-parallel barrier: wait for rank {e - 100} timed out")


def pad_k_chunks(w: torch.Tensor, world: int) -> torch.Tensor:
    """[N, K] -> [N, world * Kp]: the K columns in `world` equal chunks, each
    zero-padded from K / world to the next multiple of 128 (the operand
    layout the ranks' column shards of the activation have)."""
    n, k = w.shape
    if k % world:
        raise ValueError(f"K={k} does not split into {world} chunks")
    c = k // world
    cp = (c + 127) // 128 * 128
    out = torch.zeros((n, world, cp), dtype=w.dtype, device=w.device)
    out[:, :, :c] = w.reshape(n, world, c)
    return out.reshape(n, world * cp)
