"""Host-side logic of the N > 1 paths, run as world_size-2 gloo process groups on the CPU:
token-count sharding of the encoder chunks, the search protocol (row-range shards with global row
numbers, one all-gather of per-shard top-k lists, merge by (score desc, row asc)), and a rank that
leaves before the exchange (an error on the survivor within the process-group timeout)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import scan
from ripvec_b200 import shard, synth


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # search: each rank ranks its own row range
        n, dim, nq, k = 2000, 64, 4, 25
        db = synth.normalized_gaussian(n, dim, seed=31)
        qs = synth.normalized_gaussian(nq, dim, seed=32)
        lo, hi = shard.row_ranges(n, world)[rank]
        li, ls, _ = scan.topk_exact(db[lo:hi], qs, k)
        li = np.where(li >= 0, li + lo, -1)

        def all_gather(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            out = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(out, t)
            return [o.numpy() for o in out]

        mi, ms = shard.gather_and_merge(li, ls, k, scan.merge_topk, all_gather)
        gi, gs, _ = scan.topk_exact(db, qs, k)
        ok_search = bool((mi == gi).all() and (ms == gs).all())

        # encoder: the token-count shards partition the chunks; every rank agrees on them
        lengths = synth.lognormal_lengths(5000, 180.0, 0.8, 16, 1024, seed=33)
        mine = shard.shard_by_tokens(lengths, world)[rank]
        counts = all_gather(np.array([len(mine)], np.int64))
        tokens = all_gather(np.array([int(lengths[mine].sum())], np.int64))
        q.put((rank, ok_search, int(sum(c[0] for c in counts)), [int(t[0]) for t in tokens]))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_two_rank_search_merge_and_encoder_sharding():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=150) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, total, tokens in res:
        assert ok, f"rank {rank}: merged top-k differs from the global top-k"
        assert total == 5000
        assert abs(tokens[0] - tokens[1]) <= 1024  # greedy balance is within one chunk


def _failing_worker(rank, world, port, q):
    """Rank 1 leaves before the search exchange (as a rank that raised would); rank 0 must get an
    error from its all-gather within the process-group timeout, not wait forever."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush the message before the abrupt exit
        os._exit(0)  # no destroy_process_group: the rank is simply gone
    t0 = time.perf_counter()
    li = np.zeros((2, 5), np.int64)

    def all_gather(a):
        t = torch.from_numpy(np.ascontiguousarray(a))
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [o.numpy() for o in out]

    try:
        shard.gather_and_merge(li, li.astype(np.float64), 5, scan.merge_topk, all_gather)
        q.put((rank, "no error"))
    except Exception as e:  # gloo reports the missing peer or the timeout
        q.put((rank, f"error after {time.perf_counter() - t0:.1f} s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.timeout(120)
def test_missing_rank_surfaces_as_an_error_not_a_hang():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2]) < 60


def test_shard_by_tokens_partitions_and_balances():
    lengths = synth.lognormal_lengths(10_000, 180.0, 0.8, 16, 1024, seed=1)
    for world in (1, 2, 4, 8):
        parts = shard.shard_by_tokens(lengths, world)
        allidx = np.sort(np.concatenate(parts))
        np.testing.assert_array_equal(allidx, np.arange(len(lengths)))
        loads = [int(lengths[p].sum()) for p in parts]
        assert max(loads) - min(loads) <= int(lengths.max())


def test_row_ranges_cover_every_row_once():
    for n in (0, 1, 7, 10_000_001):
        for world in (1, 2, 3, 8):
            r = shard.row_ranges(n, world)
            assert r[0][0] == 0 and r[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
