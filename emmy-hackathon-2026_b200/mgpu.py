"""Multi-GPU sharding of the hot path: one process per GPU, torch.distributed.

The reference is single-GPU (its runner drives one device,
tools/local_runner.py:246-342).  Every workload of the hot path partitions
into independent units, so one problem is split over the ranks with no
collective inside the computation:

* GEMM (and the ragged GEMM): rows of A, B replicated -- each rank computes
  its row slab of C;
* row softmax: rows of the matrix;
* pointwise add: contiguous element ranges (multiples of 4 elements, so every
  shard keeps 16-byte vector accesses);
* attention: batch * heads.

NCCL over NVLink moves data only where the problem needs it: the broadcast of
B from rank 0 (:func:`sharded_gemm`) and the all-gather of the output slabs
(:func:`all_gather_slabs`); attention's K and V are sharded by head along
with Q, so they need no broadcast.  ``bench.py --gpus N`` times the
partitioned problem twice: kernels only, with every rank's shard already in
its HBM (strong scaling, max over ranks), and end to end through these
functions with the collectives included.

The compute step is a callback so the collective plumbing runs with the
``gloo`` backend on CPU in the tests; on GPUs the callback is a C-ABI call.
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


def all_gather_slabs(local, units: int, rank: int, world: int, torch, align: int = 1):
    """Concatenate every rank's slab (dim 0; rank r holds ``partition(units,
    world, r, align)``) into the full tensor on every rank.  Slabs are padded
    to the largest one so the gather is one equal-sized collective."""
    import torch.distributed as dist
    if world == 1:
        return local
    shards = [partition(units, world, r, align) for r in range(world)]
    if local.shape[0] != shards[rank].count:
        raise ValueError("local slab does not match this rank's shard")
    width = max(s.count for s in shards)
    tail = tuple(local.shape[1:])
    if local.shape[0] == width:
        padded = local.contiguous()
    else:
        padded = torch.zeros((width,) + tail, dtype=local.dtype, device=local.device)
        padded[: local.shape[0]] = local
    out = torch.empty((world * width,) + tail, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded)
    if all(s.count == width for s in shards):
        return out
    return torch.cat([out[r * width: r * width + s.count] for r, s in enumerate(shards)], dim=0)


def sharded_gemm(a_rows, b, m: int, rank: int, world: int, compute, torch, device=None, align: int = 1):
    """Strong-scaling C = A B over the process group.

    ``a_rows`` is this rank's row slab of A (``partition(m, world, rank,
    align)``), ``b`` is B on rank 0 and an allocated tensor of the same shape
    elsewhere (it is overwritten by the broadcast).  ``compute(a_rows, b) ->
    c_rows`` runs the local GEMM.  Returns the full C on every rank."""
    import torch.distributed as dist
    if world > 1:
        dist.broadcast(b, src=0)
    c_rows = compute(a_rows, b)
    return all_gather_slabs(c_rows, m, rank, world, torch, align)


def sharded_slabs(inputs, units: int, rank: int, world: int, compute, torch, align: int = 1):
    """Strong scaling of a row-independent operation: ``inputs`` are this
    rank's slabs (dim 0 = its ``partition(units, world, rank, align)``) --
    rows of the softmax matrix, element ranges of the pointwise operands,
    heads of Q, K and V -- ``compute(*inputs) -> out_slab`` runs the local
    kernel, and the output slabs are all-gathered.  Returns the full output
    on every rank."""
    out = compute(*inputs)
    return all_gather_slabs(out, units, rank, world, torch, align)
