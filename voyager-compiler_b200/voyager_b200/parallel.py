"""Sharding the hot path over the GPUs of one box (one process per GPU).

* Quantize / dequantize / quantize_mx: the blocks run along the last dim, so
  rows are independent.  ``shard_rows`` gives each rank a contiguous row
  range; no collective is needed and results stay sharded (weak scaling).
  A per-tensor scale is precomputed by the observer; when a caller wants it
  from the data, ``global_amax`` is the one scalar all-reduce(MAX) it takes.
* ``linear_mx`` (MXFP8 / W4A8 large configs): tensor parallel over N.  Each
  rank holds ``weight[N/g, K]`` codes and scales (``shard_n``), computes
  ``Y[:, N/g]`` with its local kernel, and ``NShardedLinear`` all-gathers the
  column blocks over NCCL (NVLink) into the full ``[M, N]``.

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
    """Tensor-parallel ``linear_mx``: the local shard's product, all-gathered
    along N.  ``local`` computes ``(input, weight_shard, bias_shard, kwargs)``
    -> ``[.., N/g]``; by default ``torch.ops.quantized_ops.linear_mx``."""

    def __init__(self, weight: torch.Tensor, weight_scale: Optional[torch.Tensor],
                 bias: Optional[torch.Tensor] = None, *, block_size: int = 32,
                 group=None, local: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.w, self.ws = shard_n(weight, weight_scale, self.rank, self.world)
        self.b = None
        if bias is not None:
            step = bias.shape[0] // self.world
            self.b = bias[self.rank * step:(self.rank + 1) * step]
        self.block_size = block_size
        self.local = local or self._linear_mx

    def _linear_mx(self, x, w, b, input_scale):
        return torch.ops.quantized_ops.linear_mx(x, w, b, input_scale=input_scale,
                                                 weight_scale=self.ws, block_size=self.block_size)

    def __call__(self, x: torch.Tensor, input_scale: Optional[torch.Tensor] = None):
        y = self.local(x, self.w, self.b, input_scale)
        lead = y.shape[:-1]
        y2 = all_gather_columns(y.reshape(-1, y.shape[-1]), self.group)
        return y2.reshape(tuple(lead) + (y2.shape[-1],))
