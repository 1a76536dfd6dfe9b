"""Data-parallel encoding of a base set across the GPUs of one box (one process per GPU).

Base vectors are independent, so the base set is split into contiguous shards, one per rank, and
nothing crosses GPUs on the data path.  Exactly two collectives run:

* one broadcast of the frozen codebooks (C_all, H x D float32) from rank 0 -- the replica every
  encoder then builds its Gram matrix from on its own GPU;
* one all-reduce (sum) of the per-shard [beam SSE, final SSE] doubles, giving the total MSE
  (MeanMseFromPrecomp over the whole base, reference src/linkage/linkage_tools.cpp:170-219).

ILS perturbations are keyed by the global vector id (reference icm.cpp:950-960), so every shard
passes its global offset and the sharded result equals the single-GPU one bit for bit.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int   # global id of the shard's first vector
    count: int


def shard_range(n_total: int, world: int, rank: int) -> Shard:
    """Contiguous split of n_total vectors: the first n_total % world ranks get one extra."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError("rank must be in [0, world)")
    if n_total < 0:
        raise ValueError("n_total must be >= 0")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return Shard(rank, world, start, base + (1 if rank < extra else 0))


def broadcast_codebooks(C_all, src: int = 0, group=None):
    """Replicates rank ``src``'s codebooks into ``C_all`` (a tensor of the right shape on every
    rank) with one broadcast.  Returns the tensor."""
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.broadcast(C_all, src=src, group=group)
    return C_all


def reduce_sse(sse, group=None):
    """Sums the per-shard [beam SSE, final SSE] (float64 tensor of 2) over ranks, in place."""
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(sse, group=group)
    return sse


def encode_shard(encode_fn, X_shard, shard: Shard, **kw):
    """Runs ``encode_fn(X_shard, sample_id_offset=shard.start, **kw)`` (the host or device encode
    entry point of an Encoder) for this rank's shard."""
    return encode_fn(X_shard, sample_id_offset=shard.start, **kw)


def total_mse(sse_sum, n_total: int):
    s = np.asarray(sse_sum, np.float64)
    return s / max(int(n_total), 1)
