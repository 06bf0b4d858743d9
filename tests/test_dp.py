"""Request-level DP (fmd_b200.dp): the LPT partition and the host-side gather,
single process and as two gloo ranks on CPU."""

from __future__ import annotations

import importlib
import os
import socket

import numpy as np
import pytest

from conftest import PKG  # noqa: F401  (imports the package as fmd_b200)

dp = importlib.import_module("fmd_b200.dp")
syn = importlib.import_module("fmd_b200.synthetic")


def _queue(n=256, seed=3):
    rng = np.random.default_rng(seed)
    lens = syn.log_uniform_lengths(rng, n, 300, 16000)
    stops = np.minimum(rng.geometric(1.0 / 800, n), 4096)
    return lens, np.full(n, 4096), stops


@pytest.mark.parametrize("n_ranks", [1, 2, 3, 8])
def test_partition_covers_every_request_once(n_ranks):
    lens, max_new, stops = _queue()
    part = dp.partition(lens, max_new, n_ranks, expected_new=stops)
    allidx = np.concatenate(part.shards)
    assert sorted(allidx.tolist()) == list(range(len(lens)))
    for sh in part.shards:
        assert np.all(np.diff(sh) > 0), "each shard keeps queue order"


@pytest.mark.parametrize("n_ranks", [2, 4, 8])
def test_partition_is_balanced(n_ranks):
    lens, max_new, stops = _queue(n=2048)
    cost = dp.request_cost(lens, max_new, stops)
    part = dp.partition(lens, max_new, n_ranks, expected_new=stops)
    # list scheduling bound: no rank exceeds the mean by more than one request
    assert part.loads.max() <= cost.sum() / n_ranks + cost.max() + 1e-6
    assert np.isclose(part.loads.sum(), cost.sum())
    for r, sh in enumerate(part.shards):
        assert np.isclose(part.loads[r], cost[sh].sum())


def test_partition_is_deterministic_and_tie_stable():
    lens = np.full(10, 500)
    a = dp.partition(lens, np.full(10, 64), 3)
    b = dp.partition(lens, np.full(10, 64), 3)
    assert all(np.array_equal(x, y) for x, y in zip(a.shards, b.shards))
    assert [len(s) for s in a.shards] == [4, 3, 3]


def test_request_cost_counts_prefill_and_decode_reads():
    c = dp.request_cost(np.array([100]), np.array([10]))
    assert c[0] == 100 + 10 * 100 + 45
    c2 = dp.request_cost(np.array([100]), np.array([10]), expected_new=np.array([3]))
    assert c2[0] == 100 + 3 * 100 + 3


def test_partition_rejects_bad_input():
    with pytest.raises(ValueError):
        dp.partition(np.array([1, 2]), np.array([1, 1]), 0)
    with pytest.raises(ValueError):
        dp.partition(np.ones((2, 2)), np.ones(2), 2)


def test_gather_single_process():
    out = dp.gather_results(None, 5, np.array([4, 0, 2, 1, 3]), ["e", "a", "c", "b", "d"])
    assert out == ["a", "b", "c", "d", "e"]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        lens, max_new, stops = _queue(n=n, seed=11)  # every rank builds the same queue
        part = dp.partition(lens, max_new, world, expected_new=stops)
        mine = part.shard(rank)
        # every rank must hold the same partition
        views = [None] * world
        dist.all_gather_object(views, [s.tolist() for s in part.shards])
        agree = all(v == views[0] for v in views)
        # a stand-in engine: the result of request i is (i, its prompt length)
        results = [(int(i), int(lens[i])) for i in mine]
        out = dp.gather_results(dist, n, mine, results)
        if rank == 0:
            q.put((agree, out == [(i, int(lens[i])) for i in range(n)], len(out)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_partition_and_gather():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    n = 97
    mp.start_processes(_rank_main, args=(2, _free_port(), n, q), nprocs=2, join=True, start_method="spawn")
    agree, ordered, count = q.get()
    assert agree, "ranks computed different partitions"
    assert ordered and count == n
