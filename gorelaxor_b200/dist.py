"""Independent streams over the GPUs of one box (no collective on the step).

Streams are partitioned in contiguous blocks, stream s on rank ⌊s·G/N⌋ of G
ranks; each rank holds its own copy of the weights and its streams' state.
The only cross-rank traffic is the job timing (a max over ranks) and, on
request, gathering results to rank 0 — ordinary torch.distributed calls on
the host side, never inside a frame.
"""

from __future__ import annotations


def partition(n_streams: int, world: int, rank: int) -> range:
    """The streams rank `rank` owns: stream s goes to rank ⌊s·world/n⌋."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    lo = -(-rank * n_streams // world)
    hi = -(-(rank + 1) * n_streams // world)
    return range(lo, hi)


def owner(stream: int, n_streams: int, world: int) -> int:
    return stream * world // n_streams


def max_over_ranks(value: float, device=None) -> float:
    """The slowest rank's value (a job is as fast as its slowest GPU)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
