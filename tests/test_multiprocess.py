"""Multi-rank host logic on CPU with the gloo backend (world_size 2): shard
plans, the broadcast / all-gather plumbing of the strong-scaling GEMM, and a
rank that fails -- all without a GPU."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT, pkg


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("units,world,align", [(4097, 8, 1), (1 << 24, 8, 4), (64, 8, 1), (4096, 3, 128), (5, 8, 1)])
def test_partition_covers_exactly_once(units, world, align):
    mgpu = pkg("mgpu")
    shards = [mgpu.partition(units, world, r, align) for r in range(world)]
    covered = np.zeros(units, dtype=np.int64)
    for s in shards:
        covered[s.start:s.start + s.count] += 1
    assert (covered == 1).all()
    assert all(s.count % align == 0 for s in shards[:-1])


def _worker(rank, world, port, mode, results):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import importlib
    mgpu = importlib.import_module("emmy-hackathon-2026_b200.mgpu")
    import torch.distributed as dist
    mgpu.init_from_env("gloo", timeout_s=20)
    try:
        m, k, n = 37, 16, 9
        rng = np.random.default_rng(0)
        a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32))
        b_full = torch.from_numpy(rng.standard_normal((k, n)).astype(np.float32))
        shard = mgpu.partition(m, world, rank)
        b = b_full.clone() if rank == 0 else torch.zeros_like(b_full)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before its collective")

        # test-only compute callback standing in for the GPU GEMM
        def compute(ar, bb):
            return ar @ bb
        c = mgpu.sharded_gemm(a[shard.start:shard.start + shard.count].clone(), b, m, rank, world, compute, torch)
        results[rank] = float((c - a @ b_full).abs().max())
    except Exception as exc:  # reported to the parent
        results[rank] = f"error: {type(exc).__name__}: {exc}"
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, mode):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
            p.join()
    return dict(results)


def test_sharded_gemm_gloo_world2():
    results = _run(2, "ok")
    assert set(results) == {0, 1}, results
    assert all(isinstance(v, float) and v < 1e-4 for v in results.values()), results


def test_failed_rank_surfaces_as_error_not_hang():
    """Rank 1 raises before joining the broadcast; rank 0's collective must end
    with an error (short process-group timeout), not wait forever."""
    results = _run(2, "fail")
    assert "error" in str(results.get(1, ""))
    assert 0 in results and "error" in str(results[0]), results
