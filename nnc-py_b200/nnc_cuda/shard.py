"""Batch sharding across the GPUs of one node (data parallel over samples).

Every hot-path operator works per sample, so a forward of a global batch
splits into contiguous per-rank shards with no exchange inside the path; the
only collective is the final gather of the outputs to rank 0 (BASELINE
config 5: "batch 1024 split evenly across 1/2/4/8 B200 ... outputs are
gathered to GPU0"). These helpers hold the host-side rules that bench.py and
the tests share; they work with any torch.distributed backend (NCCL on the
GPUs, gloo in the CPU tests).
"""

from __future__ import annotations


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first sample, sample count) of `rank`'s shard.

    The cuda target compiles one per-GPU batch, so the global batch must
    divide evenly; shards are contiguous and in rank order, so gathering them
    in rank order restores the global batch order.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not split evenly over {world} ranks")
    per = global_batch // world
    return rank * per, per


def gather_to_rank0(local, world: int, dist):
    """Concatenates every rank's `local` [per, ...] tensor in rank order on
    rank 0 (other ranks receive None). One all_gather: every rank takes part,
    as collectives require."""
    import torch

    if world == 1:
        return local
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local)
    return torch.cat(parts, 0) if dist.get_rank() == 0 else None


def max_over_ranks(value: float, world: int, dist, device=None) -> float:
    """The largest of the ranks' values (the timing rule: a multi-GPU step
    lasts as long as its slowest rank)."""
    import torch

    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
