"""Image-wise sharding of an encoder batch over one process per GPU.

The DA3 encoder's images are independent (every block mixes tokens only
within an image), so a batch of B images splits into contiguous per-rank
shards with no exchange on the data path.  What the ranks share is host-side
plumbing: which images each rank owns, the max-over-ranks step time, and an
optional final gather of the per-rank outputs to rank 0.  These helpers work
with any torch.distributed backend: NCCL on the GPUs, gloo for CPU tests.
"""
from __future__ import annotations

from typing import Optional, Tuple


def image_shard(total: int, rank: int, world: int) -> Tuple[int, int]:
    """(first image, image count) of `rank`'s contiguous shard of `total`
    images: counts differ by at most one, lower ranks take the extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if total < 0:
        raise ValueError(f"negative image count {total}")
    base, extra = divmod(total, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def max_over_ranks(value: float, group=None, device=None) -> float:
    """The maximum of `value` over all ranks (a step time: the slowest rank
    sets the job's time).  Returns `value` unchanged without a process group."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_images(local, total: int, group=None, dst: int = 0) -> Optional["object"]:
    """Gathers every rank's `[count, ...]` output shard into one
    `[total, ...]` tensor on rank `dst` (None on the other ranks), in image
    order.  Shards follow image_shard(total, rank, world)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        if local.shape[0] != total:
            raise ValueError(f"single process holds {local.shape[0]} of {total} images")
        return local
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    _, count = image_shard(total, rank, world)
    if local.shape[0] != count:
        raise ValueError(f"rank {rank} holds {local.shape[0]} images, its shard has {count}")
    # all_gather needs equal sizes: pad each shard to the largest count
    width = image_shard(total, 0, world)[1]
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:count] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    if rank != dst:
        return None
    return torch.cat([p[: image_shard(total, r, world)[1]] for r, p in enumerate(parts)], dim=0)
