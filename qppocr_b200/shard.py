"""Sharding of independent units (det/cls images, rec lines) across the GPUs
of one node, one process per GPU.

The reference engine runs a batch through one device session
(crates/qppocr-core engine.rs: det -> crop -> cls -> rec per image list).  On
a multi-GPU node the units are independent, so each rank takes a contiguous
range of the batch, runs it through its own session on its own GPU, and the
per-rank results are gathered on the host in rank order.  There is no
data-path collective; the process group carries only the result gather and
timing reductions.
"""
from typing import Any, List, Optional, Sequence, Tuple


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of rank `rank`'s contiguous share of n units: the first
    n % world ranks take one unit more, so shares differ by at most one."""
    if world <= 0 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def local_shard(items: Sequence[Any], world: int, rank: int) -> Sequence[Any]:
    """This rank's contiguous slice of `items` (a list or an array batch)."""
    a, b = shard_bounds(len(items), world, rank)
    return items[a:b]


def gather_shards(local: List[Any], world: int, rank: int, dst: int = 0,
                  group: Optional[Any] = None) -> Optional[List[Any]]:
    """Gather every rank's list of per-unit results on rank `dst`, concatenated
    in rank order (= the original unit order); other ranks get None.  Uses the
    process group's object gather (host side; any backend)."""
    if world == 1:
        return list(local)
    import torch.distributed as dist

    parts = [None] * world if rank == dst else None
    dist.gather_object(list(local), parts, dst=dst, group=group)
    if rank != dst:
        return None
    out: List[Any] = []
    for p in parts:
        out.extend(p)
    return out


def max_over_ranks(x: float, world: int, device: Optional[str] = None) -> float:
    """Max of a per-rank scalar (e.g. device time of the timed region) over all
    ranks; `device` is "cuda" under NCCL, None (CPU tensor) under gloo."""
    if world == 1:
        return float(x)
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
