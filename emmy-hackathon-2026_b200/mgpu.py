"""Multi-GPU sharding of the hot path: one process per GPU, torch.distributed.

The reference is single-GPU.  Every workload of the hot path partitions into
independent units -- rows of A (B replicated), rows of the softmax matrix,
ranges of a pointwise vector, batch*head of attention -- so the data path
needs no collective.  Two drivers are provided:

* weak scaling (``bench.py --gpus N``): every rank processes its own batch;
  only a barrier and a max-over-ranks time use the process group;
* strong scaling of one problem (:func:`sharded_gemm`): rank 0's B is
  broadcast, each rank computes its row slab of C = A B on its own GPU, and
  the slabs are all-gathered -- NCCL over NVLink only for the broadcast and
  the gather, as the hot-path plan prescribes.

The compute step is a callback so the collective plumbing can be exercised
with the ``gloo`` backend on CPU; on GPUs the callback is the C-ABI GEMM.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    start: int
    count: int


def partition(units: int, world: int, rank: int, align: int = 1) -> Shard:
    """Contiguous shard of ``units`` for ``rank``: every shard but the last is a
    multiple of ``align`` units; the last rank takes the remainder (4097 rows
    over 8 ranks -> seven shards of 512 and one of 513 with align 1)."""
    if world <= 0 or not 0 <= rank < world or align <= 0 or units < 0:
        raise ValueError("bad partition request")
    base = (units // world) // align * align
    start = base * rank
    count = base if rank < world - 1 else units - base * (world - 1)
    return Shard(start, count)


def init_from_env(backend: str, timeout_s: float = 120.0):
    """Join the process group torchrun describes (RANK / WORLD_SIZE / MASTER_*),
    with a short timeout so a missing rank ends collectives with an error."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kwargs = {}
        if backend == "nccl":
            import torch
            kwargs["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return rank, world


def sharded_gemm(a_rows, b, m: int, rank: int, world: int, compute, torch, device=None):
    """Strong-scaling C = A B over the process group.

    ``a_rows`` is this rank's row slab of A (``partition(m, world, rank)``),
    ``b`` is B on rank 0 and an allocated tensor of the same shape elsewhere
    (it is overwritten by the broadcast).  ``compute(a_rows, b) -> c_rows``
    runs the local GEMM.  Returns the full C on every rank."""
    import torch.distributed as dist
    if world > 1:
        dist.broadcast(b, src=0)
    c_rows = compute(a_rows, b)
    if world == 1:
        return c_rows
    shards = [partition(m, world, r) for r in range(world)]
    width = max(s.count for s in shards)
    padded = torch.zeros((width, c_rows.shape[1]), dtype=c_rows.dtype, device=device)
    padded[: c_rows.shape[0]] = c_rows
    gathered = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(gathered, padded)
    return torch.cat([g[: s.count] for g, s in zip(gathered, shards)], dim=0)
