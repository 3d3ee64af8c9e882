"""Multi-rank host logic on CPU (gloo, world size 2): the (batch, head) sharding used by bench.py
covers every pair exactly once and reproduces the single-process result without any data exchange,
the elapsed time reported is the max over ranks, and a rank that dies before the timing collective
makes the survivor fail with an error instead of hanging."""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 30.0) -> None:
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _shard_worker(rank: int, world: int, port: int, out) -> None:
    _init(rank, world, port)
    import bench
    from oracle import tiled_forward

    b, h, n, d = 3, 5, 40, 16  # 15 pairs: uneven split
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((b * h, n, d)).astype(np.float32) for _ in range(3))
    lo, hi = bench.shard(b * h, rank, world)
    o_local, m_local = tiled_forward(q[lo:hi], k[lo:hi], v[lo:hi], True)  # this rank's pairs only
    ms = bench.max_over_ranks(10.0 + 5.0 * rank)
    gathered = [None] * world
    dist.all_gather_object(gathered, (lo, hi, o_local, m_local))
    if rank == 0:
        out.put((gathered, ms, q, k, v))
    dist.barrier()
    dist.destroy_process_group()


def test_sharding_covers_pairs_and_matches_single_process() -> None:
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, ms, q, k, v = q_out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ranges = [(lo, hi) for lo, hi, _, _ in gathered]
    assert ranges[0][0] == 0 and ranges[-1][1] == 15
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))  # contiguous, disjoint, complete
    from oracle import tiled_forward

    o_full, m_full = tiled_forward(q, k, v, True)
    o_cat = np.concatenate([g[2] for g in gathered])
    m_cat = np.concatenate([g[3] for g in gathered])
    np.testing.assert_array_equal(o_cat, o_full)  # sharding changes nothing: pairs are independent
    np.testing.assert_array_equal(m_cat, m_full)
    assert ms == 15.0  # max over ranks


def _dead_rank_worker(rank: int, world: int, port: int, out) -> None:
    _init(rank, world, port, timeout_s=5.0)
    import bench

    if rank == 1:
        os._exit(0)  # leaves between steps, before the timing collective
    try:
        bench.max_over_ranks(1.0)
        out.put("returned")
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        out.put(f"error: {type(e).__name__}")


def test_dead_rank_is_an_error_not_a_hang() -> None:
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, world, port, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    res = q_out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res.startswith("error"), res


@pytest.mark.parametrize("pairs,world", [(1024, 1), (1024, 2), (1024, 8), (15, 4), (3, 8)])
def test_shard_arithmetic(pairs: int, world: int) -> None:
    sys.path.insert(0, ROOT)
    import bench

    spans = [bench.shard(pairs, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == pairs
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1 and sum(sizes) == pairs
