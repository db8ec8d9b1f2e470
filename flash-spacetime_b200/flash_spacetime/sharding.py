"""Event sharding across GPUs (one process per GPU, torch.distributed).

Events are independent, so a multi-GPU run splits the event list: each rank
runs the fused op on its own packed shard with a local ``cu_seqlens``, and
the only cross-rank traffic is

* the sum of the per-rank ``dW`` / ``db`` partials, gathered and added in
  rank order so that the result is bitwise identical on every rank and from
  run to run (an NCCL all-reduce would not fix the summation order), and
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
    """Sum of ``t`` over ranks, added in rank order (deterministic)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return t.clone()
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, t.contiguous(), group=group)
    acc = parts[0].clone()
    for x in parts[1:]:
        acc += x
    return acc


def gather_rows(t: Tensor, group: Optional[dist.ProcessGroup] = None) -> List[Tensor]:
    """All-gather per-rank tensors whose first dimension differs by rank."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return [t]
    world = dist.get_world_size(group)
    n = torch.tensor([t.shape[0]], dtype=torch.int64, device=t.device)
    sizes = [torch.empty_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    rows = [int(s.item()) for s in sizes]
    top = max(rows)
    pad = t.new_zeros((top,) + tuple(t.shape[1:]))
    pad[: t.shape[0]] = t
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return [p[:r] for p, r in zip(parts, rows)]


def max_over_ranks(value: float, device: torch.device,
                   group: Optional[dist.ProcessGroup] = None) -> float:
    """Maximum of a per-rank scalar (e.g. a device-timed duration)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
