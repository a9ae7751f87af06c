"""Data-parallel host logic: independent utterances sharded over GPUs.

The reference runs independent recognition contexts that share read-only
weights (src/FunAsrNet.Server/SpeechRuntime.cs:18-22,
doc/concurrency-and-memory.md:5-7).  Across GPUs the same holds: one model
replica per GPU, sessions assigned round-robin, no collective on the data path.
torch.distributed is used only for the barrier and the max-over-ranks timing.
"""
from __future__ import annotations


def assign_sessions(n_sessions: int, world: int, rank: int) -> list[int]:
    """Round-robin session ids owned by `rank` (disjoint, covering 0..n-1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid world/rank")
    return list(range(rank, n_sessions, world))


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """Max of a per-rank scalar (device time, wall time) across all ranks."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, dist=None, device=None) -> float:
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def throughput(tokens_per_rank: int, world: int, max_seconds: float) -> float:
    """Whole-job tokens/s: every rank's tokens over the slowest rank's time."""
    return tokens_per_rank * world / max_seconds
