"""Multi-rank host logic on CPU with the gloo backend (world_size 2): shard
plans, the broadcast / all-gather plumbing of every partitioned workload
(GEMM, ragged GEMM, softmax, add, attention), and a rank that fails -- all
without a GPU."""
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


def test_library_partition_matches_python():
    """b2k_mgpu_partition (host arithmetic in the C library) gives the shards
    mgpu.partition gives."""
    rt, mgpu = pkg("runtime"), pkg("mgpu")
    for units, world, align in [(4097, 8, 1), (1 << 24, 8, 4), (5, 8, 1), (4096, 3, 128), (64, 2, 1), (0, 4, 1)]:
        for r in range(world):
            s = mgpu.partition(units, world, r, align)
            assert rt.mgpu_partition(units, world, r, align) == (s.start, s.count)
    with pytest.raises(rt.B2KError):
        rt.mgpu_partition(10, 2, 2, 1)


def _worker(rank, world, port, mode, results):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import importlib
    mgpu = importlib.import_module("emmy-hackathon-2026_b200.mgpu")
    import torch.distributed as dist
    mgpu.init_from_env("gloo", timeout_s=20)
    try:
        rng = np.random.default_rng(0)
        if mode in ("ok", "fail", "ragged", "panels"):
            # rows of A over the ranks, B broadcast from rank 0 (4097-like ragged
            # shards with mode "ragged": the last rank takes the remainder)
            m, k, n = (37, 16, 9) if mode != "ragged" else (131, 12, 10)
            align = 1 if mode != "ragged" else 32
            a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32))
            b_full = torch.from_numpy(rng.standard_normal((k, n)).astype(np.float32))
            shard = mgpu.partition(m, world, rank, align)
            b = b_full.clone() if rank == 0 else torch.zeros_like(b_full)
            if mode == "fail" and rank == 1:
                raise RuntimeError("rank 1 fails before its collective")

            if mode == "panels":
                # B broadcast as three column panels (widths 3, 3, 3), one GEMM per panel
                pans = mgpu.column_panels(n, 3)
                b = [b[:, p.start:p.start + p.count].contiguous() for p in pans]

            # test-only compute callback standing in for the GPU GEMM
            def compute(ar, bb, i):
                return ar @ bb
            c = mgpu.sharded_gemm(a[shard.start:shard.start + shard.count].clone(), b, m, rank, world, compute, torch,
                                  align=align)
            results[rank] = float((c - a @ b_full).abs().max())
        elif mode == "softmax":
            rows, cols = 12, 33  # rows per rank 6 / 6, in three pieces of 2 rows
            x = torch.from_numpy(rng.standard_normal((rows, cols)).astype(np.float32))
            sh = mgpu.partition(rows, world, rank)
            seen = []

            def soft(xs, piece):
                seen.append((piece.start, piece.count))
                return torch.softmax(xs, dim=-1)
            y = mgpu.sharded_slabs((x[sh.start:sh.start + sh.count],), rows, rank, world, soft, torch, pieces=3)
            assert seen == [(0, 2), (2, 2), (4, 2)], seen
            results[rank] = float((y - torch.softmax(x, dim=-1)).abs().max())
        elif mode == "add":
            n = 1003  # shards of 500 and 503 elements (align 4)
            a = torch.from_numpy(rng.standard_normal(n).astype(np.float32))
            b = torch.from_numpy(rng.standard_normal(n).astype(np.float32))
            sh = mgpu.partition(n, world, rank, 4)
            # unequal shards: the pieces request falls back to one piece
            c = mgpu.sharded_slabs((a[sh.start:sh.start + sh.count], b[sh.start:sh.start + sh.count]), n, rank,
                                   world, lambda x, y, piece: x + y, torch, align=4, pieces=2)
            results[rank] = float((c - (a + b)).abs().max())
        elif mode == "attention":
            bh, s, d = 6, 16, 8  # heads 3 / 3; K and V sharded with Q, nothing broadcast
            q, k, v = (torch.from_numpy(rng.standard_normal((bh, s, d)).astype(np.float32)) for _ in range(3))
            sh = mgpu.partition(bh, world, rank)
            sl = slice(sh.start, sh.start + sh.count)

            def attend(qq, kk, vv, piece=None):
                return torch.softmax(qq @ kk.transpose(1, 2) / d ** 0.5, dim=-1) @ vv
            o = mgpu.sharded_slabs((q[sl], k[sl], v[sl]), bh, rank, world, attend, torch, pieces=3)
            results[rank] = float((o - attend(q, k, v)).abs().max())
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


@pytest.mark.parametrize("mode", ["ok", "ragged", "panels", "softmax", "add", "attention"])
def test_sharded_gloo_world2(mode):
    """Each partitioned workload (GEMM rows of A with B broadcast -- even and
    ragged shards, whole or as column panels --, softmax rows and attention
    heads in pieces gathered while the next computes, add element ranges)
    gathers to the unsharded result on every rank."""
    results = _run(2, mode)
    assert set(results) == {0, 1}, results
    assert all(isinstance(v, float) and v < 1e-4 for v in results.values()), results


def test_failed_rank_surfaces_as_error_not_hang():
    """Rank 1 raises before joining the broadcast; rank 0's collective must end
    with an error (short process-group timeout), not wait forever."""
    results = _run(2, "fail")
    assert "error" in str(results.get(1, ""))
    assert 0 in results and "error" in str(results[0]), results
