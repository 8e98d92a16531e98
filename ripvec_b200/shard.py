"""Data-parallel sharding of the hot path across GPUs (one process per GPU).

* Encoder: chunks are independent units, so they are sharded with no collective on the forward
  path.  ``shard_by_tokens`` balances ranks by token count: chunks sorted by length
  (descending, ties by index) go one by one to the rank with the fewest tokens so far.
* Search: the embedding matrix is split into contiguous row ranges (``row_ranges``); every rank
  ranks its shard (global row numbers via the index base), the per-shard top-k lists are
  exchanged with one all-gather and merged by (score desc, row asc) — ``gather_and_merge``.

The reference has no multi-device path (``crates/ripvec-core/src/embed.rs:666-785`` distributes
batches over backends on one machine, at most one GPU, ``backend/driver/cuda.rs:1548``).
"""

from __future__ import annotations

import heapq

import numpy as np


def shard_by_tokens(lengths: np.ndarray, world: int) -> list[np.ndarray]:
    """Greedy longest-first assignment; returns the sorted chunk indices of every rank."""
    lengths = np.asarray(lengths, np.int64)
    order = np.lexsort((np.arange(len(lengths)), -lengths))
    heap = [(0, g) for g in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, g = heapq.heappop(heap)
        out[g].append(int(i))
        heapq.heappush(heap, (load + int(lengths[i]), g))
    return [np.asarray(sorted(o), np.int64) for o in out]


def row_ranges(n_rows: int, world: int) -> list[tuple[int, int]]:
    """Contiguous row range ``[lo, hi)`` of every rank (sizes differ by at most one)."""
    return [(r * n_rows // world, (r + 1) * n_rows // world) for r in range(world)]


def gather_and_merge(local_idx, local_score64, k: int, merge_fn, all_gather_fn):
    """Exchanges per-shard ``[nq, k]`` results with one all-gather and merges them.

    ``all_gather_fn(tensor) -> list[tensor]`` is the collective (NCCL on GPUs, gloo in tests);
    ``merge_fn(idx [n_lists, nq, k], score [n_lists, nq, k], k)`` is the merge (the device kernel
    on GPUs, the oracle in tests)."""
    gi = all_gather_fn(local_idx)
    gs = all_gather_fn(local_score64)
    return merge_fn(np.stack([np.asarray(x) for x in gi]) if isinstance(gi[0], np.ndarray) else gi,
                    np.stack([np.asarray(x) for x in gs]) if isinstance(gs[0], np.ndarray) else gs, k)
