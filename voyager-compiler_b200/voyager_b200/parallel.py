"""Sharding the hot path over the GPUs of one box (one process per GPU).

* Quantize / dequantize / quantize_mx: the blocks run along the last dim, so
  rows are independent.  ``shard_rows`` gives each rank a contiguous row
  range; no collective is needed and results stay sharded (weak scaling).
  A per-tensor scale is precomputed by the observer; when a caller wants it
  from the data, ``global_amax`` is the one scalar all-reduce(MAX) it takes.
* ``linear_mx`` (MXFP8 / W4A8 large configs): tensor parallel over N.  Each
  rank holds ``weight[N/g, K]`` codes and scales (``shard_n``) and computes
  ``Y[:, N/g]``; ``NShardedLinear`` gives every rank the full ``[M, N]``,
  either by storing the tiles through an NVLS multicast address from the
  GEMM epilogue or by an NCCL all-gather of the column blocks.

The local GEMM is a callable, so the same gather logic runs on CPU ranks
(gloo) in the tests with the oracle as the local compute.
"""

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def shard_bounds(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) of n items for rank (the first n % world ranks
    take one more)."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def shard_rows(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    lo, hi = shard_bounds(t.shape[0], rank, world)
    return t[lo:hi]


def shard_n(weight: torch.Tensor, weight_scale: Optional[torch.Tensor], rank: int, world: int,
            multiple: int = 8):
    """Rows [N/g] of a [N, K] weight (and its [N, K/bs] scales).  N must
    split into equal shards that are multiples of ``multiple`` (the GEMM's
    N granularity), so the all-gather moves equal blocks."""
    n = weight.shape[0]
    if n % world or (n // world) % multiple:
        raise ValueError(f"N={n} does not split into {world} shards of a multiple of {multiple}")
    step = n // world
    sl = slice(rank * step, (rank + 1) * step)
    return weight[sl], (None if weight_scale is None else weight_scale[sl])


def global_amax(x: torch.Tensor, group=None) -> torch.Tensor:
    """max |x| over all ranks' shards (one scalar all-reduce)."""
    m = x.detach().abs().amax().float().reshape(1)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    return m.reshape(())


def all_gather_columns(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """[M, n] per rank -> [M, n * world] (rank r's block at columns r*n)."""
    world = dist.get_world_size(group)
    if world == 1:
        return y_local
    y_local = y_local.contiguous()
    m, n = y_local.shape
    buf = torch.empty((world * m, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local, group=group)
    return buf.view(world, m, n).permute(1, 0, 2).reshape(m, world * n)


class NShardedLinear:
    """Tensor-parallel ``linear_mx``: each rank computes its N/g output
    columns; every rank ends with the full [.., N].

    Two ways to share the columns:
      * ``multicast`` (default when the group has NVLS multicast and the
        operands are MXFP8): the local tcgen05 GEMM, then its [M, N/g]
        columns copied with whole-row 16-byte pieces through the multicast
        address of a symmetric output buffer (one store lands in every
        rank's copy), then one flag barrier.  The result is a view of that
        buffer, valid until the next call.  (Storing through the multicast
        address straight from the GEMM epilogue, one row per thread, sends
        scattered 16-byte pieces and runs at half the speed.)
      * otherwise: the local product (``local``, by default
        ``torch.ops.quantized_ops.linear_mx``) all-gathered with NCCL."""

    def __init__(self, weight: torch.Tensor, weight_scale: Optional[torch.Tensor],
                 bias: Optional[torch.Tensor] = None, *, block_size: int = 32,
                 group=None, local: Optional[Callable] = None,
                 multicast: Optional[bool] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_full = weight.shape[0]
        self.w, self.ws = shard_n(weight, weight_scale, self.rank, self.world)
        self.b = None
        if bias is not None:
            step = bias.shape[0] // self.world
            self.b = bias[self.rank * step:(self.rank + 1) * step]
        self.block_size = block_size
        self.local = local or self._linear_mx
        if multicast is None:
            multicast = False
            if self.world > 1 and local is None and weight.is_cuda:
                from voyager_b200.tp import multicast_available

                multicast = multicast_available(group)
        self.multicast = multicast
        self._ws = None

    def _linear_mx(self, x, w, b, input_scale):
        return torch.ops.quantized_ops.linear_mx(x, w, b, input_scale=input_scale,
                                                 weight_scale=self.ws, block_size=self.block_size)

    def _multicast(self, x, input_scale):
        """The local columns stored straight into every rank's output; None
        when the operands do not take the MXFP8 GEMM."""
        from voyager_b200 import _lib, mxgemm
        from voyager_b200.ops import _stream
        from voyager_b200.tp import Workspace

        if not mxgemm.applies(x, self.w, input_scale, self.ws, self.block_size, None, None,
                              "kc", "linear"):
            return None
        entry = mxgemm._vouched_entry(x, input_scale)
        K = x.shape[-1]
        M = x.numel() // K
        if entry is not None and entry[1] is not None:
            pa, pas = entry[1]
        else:
            pa, pas, ok = mxgemm._pack(x.reshape(-1, K).contiguous(),
                                       input_scale.reshape(-1, input_scale.shape[-1]).contiguous(),
                                       128, entry is None)
            if not ok:
                return None
        pw, pws, ok = mxgemm.packed_weight(self.w, self.ws)
        if not ok:
            return None
        if self._ws is None or self._ws.raw_shape != (M, self.n_full):
            Mp = (M + 127) // 128 * 128
            self._ws = None
            self._ws = Workspace(self.group, Mp, {}, x.device, raw={"out": M * self.n_full * 2})
            self._ws.raw_shape = (M, self.n_full)
            self._err = torch.zeros(1, dtype=torch.int32, device=x.device)
        ws = self._ws
        _, mc = ws.raw_region("out")
        n = self.w.shape[0]
        col = self.rank * n
        b = None if self.b is None else self.b.contiguous().data_ptr()
        stream = _stream(x.device)
        lib = _lib.load()
        local = torch.empty((M, n), dtype=torch.bfloat16, device=x.device)
        st = lib.vq_gemm_mxf8_ex(pa.data_ptr(), pas.data_ptr(), pw.data_ptr(), pws.data_ptr(),
                                 M, n, K, b, None, 0, local.data_ptr(), n, 0,
                                 self._err.data_ptr(), stream)
        _lib.check(st, "linear_mx (tensor parallel)")
        # whole-row pieces of the local columns into every rank's output
        _lib.check(lib.vq_tp_copy_multicast(local.data_ptr(), n * 2, M, n * 2, mc + col * 2,
                                            self.n_full * 2, stream),
                   "linear_mx (tensor parallel, multicast copy)")
        ws.barrier(stream)
        y = ws.raw_tensor("out", (M, self.n_full), torch.bfloat16)
        return y.reshape(tuple(x.shape[:-1]) + (self.n_full,))

    def __call__(self, x: torch.Tensor, input_scale: Optional[torch.Tensor] = None):
        if self.multicast:
            y = self._multicast(x, input_scale)
            if y is not None:
                return y
        y = self.local(x, self.w, self.b, input_scale)
        lead = y.shape[:-1]
        y2 = all_gather_columns(y.reshape(-1, y.shape[-1]), self.group)
        return y2.reshape(tuple(lead) + (y2.shape[-1],))
