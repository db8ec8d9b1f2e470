"""Event sharding across GPUs (one process per GPU, torch.distributed).

Events are independent, so a multi-GPU run splits the event list: each rank
runs the fused op on its own packed shard with a local ``cu_seqlens``, and
the only cross-rank traffic is

* the sum of the per-rank ``dW`` / ``db`` partials, gathered and reduced by
  the same kernel on every rank, so that the result is bitwise identical on
  every rank and from run to run (an NCCL all-reduce would not fix the
  summation order), and
* all-gathers of per-rank outputs (when wanted) and timings.

The partition is longest-processing-time first on ``L^2`` (the cost of an
event is proportional to its number of pairs): events sorted by length,
each given to the currently least-loaded rank. Ties break by rank, so every
rank computes the same partition without communicating.
"""

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
from torch import Tensor


def lpt_partition(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Indices of the events each rank owns, balanced on sum of L^2."""
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    loads = [0] * world
    shards: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        shards[r].append(i)
        loads[r] += int(lengths[i]) ** 2
    for s in shards:
        s.sort()
    return shards


def shard_loads(lengths: Sequence[int], shards: List[List[int]]) -> List[int]:
    return [sum(int(lengths[i]) ** 2 for i in s) for s in shards]


def pack_events(lengths: Sequence[int], index: Sequence[int]) -> Tuple[List[int], Tensor]:
    """Lengths and int32 ``cu_seqlens`` of the selected events, packed."""
    sel = [int(lengths[i]) for i in index]
    cu = torch.zeros(len(sel) + 1, dtype=torch.int32)
    if sel:
        cu[1:] = torch.cumsum(torch.tensor(sel, dtype=torch.int64), 0).to(torch.int32)
    return sel, cu


def ordered_sum(t: Tensor, group: Optional[dist.ProcessGroup] = None) -> Tensor:
    """Sum of ``t`` over ranks, bitwise the same on every rank.

    One all-gather into a [world, n] buffer and one reduction over its rank
    axis: every rank runs the same reduction on the same gathered values, so
    the result does not depend on the rank or on the collective's internal
    order (an all-reduce may add in a topology-dependent order). Two launches
    in all; a list all-gather and a loop of adds took ~18 small kernels a
    step at 8 ranks."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return t.clone()
    world = dist.get_world_size(group)
    flat = t.contiguous().view(-1)
    buf = torch.empty(world * flat.numel(), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(buf, flat, group=group)
    return buf.view(world, -1).sum(0).view_as(t)


def gather_rows(t: Tensor, group: Optional[dist.ProcessGroup] = None,
                sizes: Optional[Sequence[int]] = None) -> List[Tensor]:
    """All-gather per-rank tensors whose first dimension differs by rank.

    ``sizes`` are every rank's row counts when the caller knows them (the
    LPT partition is computed identically on every rank), which saves the
    size exchange and its device-to-host read; without them the sizes are
    all-gathered first.
    """
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return [t]
    world = dist.get_world_size(group)
    if sizes is None:
        n = torch.tensor([t.shape[0]], dtype=torch.int64, device=t.device)
        got = [torch.empty_like(n) for _ in range(world)]
        dist.all_gather(got, n, group=group)
        sizes = [int(x) for x in torch.cat(got).tolist()]
    gatherer = RowGather(list(sizes), tuple(t.shape[1:]), t.dtype, t.device, group)
    gatherer.start(t).wait()
    return gatherer.parts()


class RowGather:
    """All-gather of per-rank row blocks of known, unequal sizes.

    The send and receive buffers are allocated once (every rank pads its
    block to the largest size), so a training loop issues one
    ``all_gather_into_tensor`` per step with no allocation and no host
    synchronisation; ``start`` returns the collective's work handle, so the
    transfer can overlap the work that follows (NCCL runs on its own stream).
    """

    def __init__(self, sizes: Sequence[int], row_shape: Tuple[int, ...], dtype: torch.dtype,
                 device: torch.device, group: Optional[dist.ProcessGroup] = None) -> None:
        self.sizes = [int(n) for n in sizes]
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.top = max(self.sizes) if self.sizes else 0
        self.send = torch.zeros((self.top,) + tuple(row_shape), dtype=dtype, device=device)
        self.recv = torch.empty((len(self.sizes) * self.top,) + tuple(row_shape), dtype=dtype,
                                device=device)

    def start(self, t: Optional[Tensor] = None):
        """Copy ``t`` (this rank's rows; None if already written to
        ``send``) and issue the all-gather; returns the work handle."""
        if t is not None:
            self.send[: t.shape[0]].copy_(t)
        return dist.all_gather_into_tensor(self.recv, self.send, group=self.group,
                                           async_op=True)

    def parts(self) -> List[Tensor]:
        return [self.recv[r * self.top: r * self.top + n] for r, n in enumerate(self.sizes)]

    def bytes_received(self) -> int:
        return (len(self.sizes) - 1) * self.send.numel() * self.send.element_size()


def gather_over_ranks(value: float, device: torch.device,
                      group: Optional[dist.ProcessGroup] = None) -> List[float]:
    """Every rank's value of a per-rank scalar, in rank order (one all-gather):
    the per-rank step times, whose maximum is the job's and whose spread is
    the partition's imbalance."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return [float(value)]
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    out = torch.empty(dist.get_world_size(group), dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(out, t, group=group)
    return [float(x) for x in out.tolist()]


def max_over_ranks(value: float, device: torch.device,
                   group: Optional[dist.ProcessGroup] = None) -> float:
    """Maximum of a per-rank scalar (e.g. a device-timed duration)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
