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


def gather_start(local, units: int, rank: int, world: int, torch, align: int = 1):
    """Start the all-gather of this rank's slab (dim 0; rank r holds
    ``partition(units, world, r, align)``) without waiting for it.  Returns a
    function that waits and returns the full tensor.  Slabs are padded to the
    largest one so the gather is one equal-sized collective; on GPUs it runs
    on the process group's own stream, so kernels issued after this call
    overlap it."""
    import torch.distributed as dist
    shards = [partition(units, world, r, align) for r in range(world)]
    if local.shape[0] != shards[rank].count:
        raise ValueError("local slab does not match this rank's shard")
    if world == 1:
        return lambda: local
    width = max(s.count for s in shards)
    tail = tuple(local.shape[1:])
    if local.shape[0] == width:
        padded = local.contiguous()
    else:
        padded = torch.zeros((width,) + tail, dtype=local.dtype, device=local.device)
        padded[: local.shape[0]] = local
    out = torch.empty((world * width,) + tail, dtype=local.dtype, device=local.device)
    work = dist.all_gather_into_tensor(out, padded, async_op=True)

    def finish():
        work.wait()
        if all(s.count == width for s in shards):
            return out
        return torch.cat([out[r * width: r * width + s.count] for r, s in enumerate(shards)], dim=0)
    return finish


def all_gather_slabs(local, units: int, rank: int, world: int, torch, align: int = 1):
    """Concatenate every rank's slab (dim 0; rank r holds ``partition(units,
    world, r, align)``) into the full tensor on every rank."""
    return gather_start(local, units, rank, world, torch, align)()


def column_panels(n: int, panels: int):
    """``panels`` contiguous column ranges of an n-wide B (the last one takes
    the remainder)."""
    return [partition(n, panels, p) for p in range(panels)]


def sharded_gemm(a_rows, b, m: int, rank: int, world: int, compute, torch, align: int = 1):
    """Strong-scaling C = A B over the process group.

    ``a_rows`` is this rank's row slab of A (``partition(m, world, rank,
    align)``).  ``b`` is B on rank 0 and an allocated tensor of the same
    shape elsewhere (overwritten by the broadcast), or a list of B's column
    panels in that form (each its own contiguous tensor: [K, width], or
    [width, K] for a transposed B; :func:`column_panels` gives the ranges).
    ``compute(a_rows, b_panel, index) -> c_panel`` runs the local GEMM of
    panel ``index`` and returns its [rows, width] result, which must stay
    valid until this call returns.  Returns the full C on every rank.

    With several panels the steps overlap: every panel's broadcast is issued
    at once and runs in order on the process group's stream; the GEMM of
    panel p waits only for panel p, and the all-gather of panel p's C runs
    while panel p + 1 computes.  Panels pay off when each panel's GEMM still
    fills the GPU (2048 x 2048 x 4096 per rank at 2 GPUs: 128 tiles, as many
    waves as the unsplit 2048 x 4096)."""
    import torch.distributed as dist
    panels = list(b) if isinstance(b, (list, tuple)) else [b]
    bcast = [dist.broadcast(p, src=0, async_op=True) for p in panels] if world > 1 else []
    finishers = []
    for i, panel in enumerate(panels):
        if bcast:
            bcast[i].wait()
        finishers.append(gather_start(compute(a_rows, panel, i), m, rank, world, torch, align))
    parts = [f() for f in finishers]
    return parts[0] if len(parts) == 1 else torch.cat(parts, dim=1)


def sharded_slabs(inputs, units: int, rank: int, world: int, compute, torch, align: int = 1, pieces: int = 1):
    """Strong scaling of a row-independent operation: ``inputs`` are this
    rank's slabs (dim 0 = its ``partition(units, world, rank, align)``) --
    rows of the softmax matrix, element ranges of the pointwise operands,
    heads of Q, K and V.  ``compute(*input_pieces, piece) -> out_piece`` runs
    the local kernel on rows ``piece`` (a :class:`Shard` within this rank's
    slab) and returns that piece's output, which must stay valid until this
    call returns.  The output is all-gathered; returns the full output on
    every rank.

    With ``pieces`` > 1 the slab is cut into that many row pieces and the
    all-gather of piece i runs while piece i + 1 computes.  That needs equal
    shards on every rank, cut into equal pieces (multiples of ``align``);
    otherwise the slab runs as one piece."""
    shards = [partition(units, world, r, align) for r in range(world)]
    count = shards[rank].count
    if (pieces > 1 and all(s.count == count for s in shards) and count % pieces == 0
            and (count // pieces) % align == 0):
        step = count // pieces
    else:
        pieces, step = 1, count
    if pieces == 1:
        return all_gather_slabs(compute(*inputs, Shard(0, count)), units, rank, world, torch, align)
    finishers = []
    for i in range(pieces):
        piece = Shard(i * step, step)
        out = compute(*(x[piece.start:piece.start + step] for x in inputs), piece)
        finishers.append(gather_start(out, step * world, rank, world, torch))
    # gathered piece i is [world * step] rows, rank-major; rank r's piece i
    # belongs at rows r * count + i * step of the full output
    parts = [f() for f in finishers]
    tail = tuple(parts[0].shape[1:])
    full = torch.empty((world * count,) + tail, dtype=parts[0].dtype, device=parts[0].device)
    view = full.view((world, pieces, step) + tail)
    for i, g in enumerate(parts):
        view[:, i].copy_(g.view((world, step) + tail))
    return full
