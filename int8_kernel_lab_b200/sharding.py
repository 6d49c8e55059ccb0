"""Batch sharding across ranks (one process per GPU).

Every image is an independent convolution, so the batch splits with no
collective on the data path: rank r owns images [start, stop) of an even split,
holds only that slice of the NHWC input and NHWK output, and a full copy of the
filter and bias.  A collective appears only to gather outputs for verification.
"""
from __future__ import annotations

from .shape import ConvShape


def shard_range(n: int, rank: int, world: int):
    """Images [start, stop) of `rank`: an even split, the first n % world ranks
    taking one extra image."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    per, extra = divmod(n, world)
    start = rank * per + min(rank, extra)
    return start, start + per + (1 if rank < extra else 0)


def shard_shape(shape: ConvShape, rank: int, world: int) -> ConvShape:
    lo, hi = shard_range(shape.n, rank, world)
    return shape.with_batch(hi - lo)


def input_slice(x, shape: ConvShape, rank: int, world: int):
    """This rank's images of a flat NHWC input (numpy array or tensor)."""
    lo, hi = shard_range(shape.n, rank, world)
    per = shape.h * shape.w * shape.c
    return x[lo * per:hi * per]


def gather_outputs(y_local, shape: ConvShape, rank: int, world: int, dist, group=None):
    """Gathers every rank's flat NHWK slice to rank 0 (torch.distributed, any
    backend: NCCL on GPUs, gloo on CPU).  Returns the full output on rank 0 and
    None elsewhere.  Uneven splits are padded to the largest slice for the
    collective and trimmed afterwards."""
    import torch

    per_image = shape.out_h * shape.out_w * shape.k
    counts = [(hi - lo) * per_image for lo, hi in
              (shard_range(shape.n, r, world) for r in range(world))]
    width = max(counts)
    padded = torch.zeros(width, dtype=y_local.dtype, device=y_local.device)
    padded[:y_local.numel()] = y_local
    if rank == 0:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.gather(padded, gather_list=parts, dst=0, group=group)
        return torch.cat([p[:c] for p, c in zip(parts, counts)])
    dist.gather(padded, dst=0, group=group)
    return None
