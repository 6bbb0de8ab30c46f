"""Multi-GPU host logic on CPU: partitioning, and a world-size-2 gloo run of
the column-sharded GEMM (A replicated, B/C column panels, all-gather of the
panels, panel-major -> row-major) and of batch sharding."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_split_range_covers_exactly_once():
    from b2blas import shard

    for total in (0, 1, 7, 8, 4096, 8193):
        for parts in (1, 2, 3, 8):
            for align in (1, 8):
                seen = []
                prev_end = 0
                for r in range(parts):
                    b, e = shard.split_range(total, parts, r, align)
                    assert b == prev_end and e >= b
                    if r < parts - 1 and e < total:
                        assert e % align == 0
                    seen.extend(range(b, e))
                    prev_end = e
                assert seen == list(range(total))


def test_column_panels_aligned():
    from b2blas import shard

    w = shard.column_panels(8192, 8, 8)
    assert w == [1024] * 8
    w = shard.column_panels(1000, 3, 8)
    assert sum(w) == 1000 and all(x % 8 == 0 for x in w[:-1])


def test_panels_to_rowmajor_host():
    from b2blas import shard

    m, widths = 3, [2, 3, 1]
    full = np.arange(m * sum(widths)).reshape(m, sum(widths))
    panels = np.concatenate([full[:, c0:c0 + w].ravel() for c0, w in zip([0, 2, 5], widths)])
    assert np.array_equal(shard.panels_to_rowmajor_host(panels, m, widths), full.ravel())


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cublas-rs_b200"))
    from b2blas import shard

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        m, n, k = 16, 40, 12
        A = rng.standard_normal((m, k))
        B = rng.standard_normal((k, n))
        widths = shard.column_panels(n, world, 8)
        c0 = sum(widths[:rank])
        Bp = shard.panel_of(B.ravel(), k, n, c0, c0 + widths[rank]).reshape(k, widths[rank])
        Cp = (A @ Bp).ravel()  # this rank's panel (the GPU GEMM's job)
        maxw = max(widths)
        send = torch.zeros(m * maxw, dtype=torch.float64)
        send[:Cp.size] = torch.from_numpy(Cp)
        gathered = [torch.zeros(m * maxw, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, send)
        panels = np.concatenate([g.numpy()[:m * w] for g, w in zip(gathered, widths)])
        C = shard.panels_to_rowmajor_host(panels, m, widths).reshape(m, n)
        ok_cols = np.allclose(C, A @ B)
        # batch sharding: every batch computed exactly once across ranks
        b0, b1 = shard.batch_shard(4096, world, rank)
        counts = torch.zeros(4096, dtype=torch.int64)
        counts[b0:b1] += 1
        dist.all_reduce(counts)
        ok_batch = bool((counts == 1).all())
        q.put((rank, ok_cols, ok_batch))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_column_and_batch_sharding():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = sorted(q.get(timeout=10) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert results == [(0, True, True), (1, True, True)]


def test_rank_failure_is_seen_by_peer():
    # A rank that raises before the collective: the peer's collective ends
    # with an error within the process-group timeout instead of hanging.
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode != 0  # the failing rank
    assert q.get(timeout=10) == ("rank0", "error")


def _failing_worker(rank, world, port, q):
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise SystemExit(3)
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put(("rank0", "completed"))
    except Exception:
        q.put(("rank0", "error"))
