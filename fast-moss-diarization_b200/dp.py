"""Request-level data parallelism across GPUs (one process per GPU).

Requests are independent and the decoder is replicated on every GPU, so the
hot path needs no collective: the request queue is split once, each rank
runs its own continuous-batching engine over its share, and the results are
gathered on the host afterwards.

The reference runs one engine per process and micro-batches a sorted request
list (`Engine::transcribe`, crates/fmd-core/src/engine.rs:382-424: sort by
prompt length, `chunks(max_batch_size)`). Across GPUs the split balances
estimated work instead: greedy longest-processing-time (LPT) assignment by
`request_cost`. Within a rank's share the requests keep their queue order:
the reference sorts only to reduce padding inside static micro-batches, and
continuous batching over ragged attention has no padding. The partition is a
pure function of the request list and the rank count, so every rank computes
the same one and no message is needed to agree on it.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np


def request_cost(prompt_len: np.ndarray, max_new: np.ndarray, expected_new: np.ndarray | None = None,
                 prefill_weight: float = 1.0) -> np.ndarray:
    """Estimated device work of each request, in KV-position reads.

    A request prefills `prompt_len` positions (compute-bound, weighted by
    `prefill_weight` relative to a decode read of one position) and then
    decodes `n` tokens, the t-th of which reads `prompt_len + t` cached
    positions: n * prompt_len + n * (n - 1) / 2 in total. `n` is
    `expected_new` when the caller has an estimate of where the request
    stops, else the budget `max_new`.
    """
    p = np.asarray(prompt_len, dtype=np.float64)
    n = np.asarray(max_new if expected_new is None else np.minimum(expected_new, max_new), dtype=np.float64)
    return prefill_weight * p + n * p + n * (n - 1.0) / 2.0


@dataclass
class Partition:
    """`shards[r]`: request indices of rank r, in queue order."""

    shards: list[np.ndarray]
    loads: np.ndarray  # estimated cost per rank

    def shard(self, rank: int) -> np.ndarray:
        return self.shards[rank]


def partition(prompt_len, max_new, n_ranks: int, expected_new=None, prefill_weight: float = 1.0) -> Partition:
    """Greedy LPT: requests in decreasing cost, each to the least-loaded rank
    (ties to the lowest rank); deterministic for a given input."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    lens = np.asarray(prompt_len)
    if lens.ndim != 1:
        raise ValueError("prompt_len must be 1-D")
    cost = request_cost(lens, max_new, expected_new, prefill_weight)
    order = sorted(range(len(cost)), key=lambda i: (-cost[i], i))
    heap = [(0.0, r) for r in range(n_ranks)]
    buckets: list[list[int]] = [[] for _ in range(n_ranks)]
    loads = np.zeros(n_ranks)
    for i in order:
        load, r = heapq.heappop(heap)
        buckets[r].append(i)
        loads[r] = load + cost[i]
        heapq.heappush(heap, (loads[r], r))
    shards = [np.array(sorted(b), dtype=np.int64) for b in buckets]
    return Partition(shards, loads)


def gather_results(pg, n_total: int, local_indices: np.ndarray, local_results: list) -> list | None:
    """Host-side gather after the run: rank 0 gets every request's result in
    the original queue order, the other ranks get None. `pg` is
    `torch.distributed` (initialised), or None for a single process."""
    if pg is None:
        out = [None] * n_total
        for i, res in zip(local_indices.tolist(), local_results):
            out[i] = res
        return out
    payload = (local_indices.tolist(), local_results)
    gathered = [None] * pg.get_world_size() if pg.get_rank() == 0 else None
    pg.gather_object(payload, gathered, dst=0)
    if pg.get_rank() != 0:
        return None
    out = [None] * n_total
    for idx, res in gathered:
        for i, r in zip(idx, res):
            if out[i] is not None:
                raise RuntimeError(f"request {i} returned by two ranks")
            out[i] = r
    missing = [i for i, r in enumerate(out) if r is None]
    if missing:
        raise RuntimeError(f"{len(missing)} requests have no result (first: {missing[:5]})")
    return out
