"""Work split across GPUs: one process per GPU, no data-path collective.

A separation is independent per track (the chunk crossfade never crosses a track), so ranks
take whole tracks round-robin and only the timing is reduced (a max over ranks): a batch of
tracks is split across GPUs, and a single-track job runs one replica per GPU.

One long track can also be split by output samples (Plan.separate_part): rank r writes the
samples of sample_range_for_rank, running the chunks that reach them; the chunks at the edge
of two ranges run on both, so the ranks exchange nothing and each range is the same floats
a single GPU writes.
"""
from __future__ import annotations


def tracks_for_rank(n_tracks: int, rank: int, world: int) -> list[int]:
    """Round-robin assignment: rank r takes tracks r, r + world, r + 2*world, ..."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_tracks, world))


def sample_range_for_rank(n_samples: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, nearly equal output-sample ranges, rank r the r-th: [begin, end)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return n_samples * rank // world, n_samples * (rank + 1) // world


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of a per-rank scalar over the default process group (identity when alone)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
