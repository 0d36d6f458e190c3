"""Image-level data parallelism of the encoder: one process per GPU, a full
weight replica per GPU, images sharded by index, no collective on the data
path (the encoder has no cross-image dependency).  The only collective is
the timing reduction (max over ranks), outside the timed region."""
from __future__ import annotations


def shard_range(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """(first image, count) of `rank`: contiguous, sizes differ by at most 1."""
    if world <= 0 or not 0 <= rank < world or n_total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(n_total, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def image_seed(index: int, base: int = 100) -> int:
    """Seed of image `index` of the job (the same on every rank)."""
    return base + index


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank float over the default process group (identity
    without one)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
