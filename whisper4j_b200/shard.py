"""Independent audio streams sharded over the GPUs of one node, one process per GPU.

The reference decodes its 30 s chunks one after another (WhisperModel.java:334-430, each chunk's
decodeWithFallback at :319-321 / :377-389); chunks share nothing but the weights (the
previous-text prompt is off by default, :711), so the streams of a job split across ranks with
no exchange on the data path: stream i goes to rank i mod world_size, each rank holds a full
weight replica on its own device and decodes its streams in one device loop.  The only
collective is the final gather of the (small) results to rank 0, over whatever process group
the caller runs (NCCL on the GPU box, gloo in the CPU tests).
"""
from __future__ import annotations

from typing import Callable, Sequence


def shard_streams(n_streams: int, world_size: int, rank: int) -> list[int]:
    """Stream indices of `rank`: i with i mod world_size == rank, in ascending order."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world size {world_size}")
    if n_streams < 0:
        raise ValueError("n_streams must be >= 0")
    return list(range(rank, n_streams, world_size))


def decode_sharded(n_streams: int, decode_shard: Callable[[list[int]], Sequence], group=None):
    """Decode this rank's share of `n_streams` with `decode_shard(indices) -> results` (one per
    index, in order) and gather every rank's results to rank 0 in stream order.

    Returns the full list of n_streams results on rank 0 and None elsewhere.  With no
    initialised process group this is a single-rank run.  A rank that raises propagates the
    error before the gather; the other ranks then fail in the gather with the process
    group's timeout rather than hang.
    """
    import torch.distributed as dist

    distributed = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if distributed else 1
    rank = dist.get_rank(group) if distributed else 0
    mine = shard_streams(n_streams, world, rank)
    results = list(decode_shard(mine))
    if len(results) != len(mine):
        raise RuntimeError(f"decode_shard returned {len(results)} results for {len(mine)} streams")
    if not distributed:
        return results
    gathered = [None] * world if rank == 0 else None
    dist.gather_object((mine, results), gathered, dst=0, group=group)
    if rank != 0:
        return None
    out = [None] * n_streams
    for idx, res in gathered:
        for i, r in zip(idx, res):
            out[i] = r
    return out
