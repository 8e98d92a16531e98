"""The library's own multi-device data plane through the C ABI:

* ``rv_embed_varlen_multi`` (``embed_distributed``, crates/ripvec-core/src/embed.rs:666-785):
  several contexts fed from one cursor by one host thread each; results in input order equal a
  single context's, and the first failure propagates.
* ``rv_index_topk_sharded``: row shards exchanging their top-k lists over NCCL and merging on
  the device.  With one GPU the communicator has one rank (the all-gather and merge still run);
  with two or more GPUs a two-process run checks the exchange itself.
"""

import multiprocessing as mp
import os

import numpy as np
import pytest

from helpers import TINY_MODERN
from oracle import scan
from ripvec_b200 import EmbedBackend, embed_distributed, synth
from ripvec_b200._lib import RvError
from ripvec_b200.index import SearchIndex, ShardComm, topk_sharded

pytestmark = pytest.mark.gpu


def test_embed_distributed_matches_one_context(cuda_device):
    w = synth.random_weights(TINY_MODERN, seed=8, qk_std=0.2)
    lengths = synth.uniform_lengths(300, 1, 900, seed=9)
    ids, cu = synth.packed_ids(lengths, TINY_MODERN.vocab, seed=10)
    one = EmbedBackend(TINY_MODERN, w, dtype="bf16", device=cuda_device)
    expect = one.embed_packed(ids, cu)
    one.close()
    # small token budgets so the cursor hands out many runs to the three workers
    many = [EmbedBackend(TINY_MODERN, w, dtype="bf16", device=cuda_device, max_batch_tokens=4096 * (i + 1))
            for i in range(3)]
    out = embed_distributed(many, ids, cu)
    np.testing.assert_array_equal(out, expect)
    # a token outside the vocabulary in the last chunk: the error reaches the caller
    bad = ids.copy()
    bad[-1] = TINY_MODERN.vocab + 5
    with pytest.raises(RvError):
        embed_distributed(many, bad, cu)
    # the contexts stay usable afterwards
    np.testing.assert_array_equal(embed_distributed(many[:2], ids, cu), expect)
    assert embed_distributed(many, np.zeros(0, np.int32), np.zeros(1, np.int32)).shape == (0, TINY_MODERN.hidden)
    for b in many:
        b.close()


def _sharded(torch, db, q, k, base, comm, threshold=float("-inf")):
    idx = SearchIndex(db, base=base, device=comm.device)
    qd = torch.from_numpy(q).cuda()
    oi = torch.empty(len(q), k, dtype=torch.int64, device="cuda")
    os_ = torch.empty(len(q), k, dtype=torch.float32, device="cuda")
    o64 = torch.empty(len(q), k, dtype=torch.float64, device="cuda")
    topk_sharded(idx, comm, qd, k, oi, os_, o64, threshold=threshold,
                 stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    idx.close()
    return oi.cpu().numpy(), o64.cpu().numpy()


def test_topk_sharded_single_rank(cuda_device):
    import torch

    db = synth.normalized_gaussian(40_000, 256, seed=30)
    q = synth.normalized_gaussian(12, 256, seed=31)
    ei, es, _ = scan.topk_exact(db, q, 64)
    comm = ShardComm(ShardComm.new_unique_id(), 0, 1, device=cuda_device, timeout_ms=30000)
    for _ in range(2):  # the communicator and its buffers are reused
        oi, o64 = _sharded(torch, db, q, 64, 0, comm)
        np.testing.assert_array_equal(oi, ei)
        np.testing.assert_array_equal(o64, es)
    comm.close()


def _rank_main(rank, world, uid, db, q, k, out_q):
    import torch

    torch.cuda.set_device(rank)
    try:
        comm = ShardComm(uid, rank, world, device=rank, timeout_ms=60000)
        bounds = np.linspace(0, len(db), world + 1).astype(int)
        lo, hi = bounds[rank], bounds[rank + 1]
        oi, o64 = _sharded(torch, db[lo:hi], q, k, int(lo), comm)
        comm.close()
        out_q.put((rank, oi, o64, None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out_q.put((rank, None, None, repr(e)))


def test_topk_sharded_two_ranks(cuda_device):
    """Two processes, one GPU each, one all-gather: every rank gets the oracle's global top-k."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    db = synth.normalized_gaussian(50_001, 128, seed=32)
    q = synth.normalized_gaussian(5, 128, seed=33)
    k = 100
    ei, es, _ = scan.topk_exact(db, q, k)
    uid = ShardComm.new_unique_id()
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    os.environ.update(env)
    ps = [ctx.Process(target=_rank_main, args=(r, 2, uid, db, q, k, out_q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [out_q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(timeout=120)
    for rank, oi, o64, err in res:
        assert err is None, (rank, err)
        np.testing.assert_array_equal(oi, ei)
        np.testing.assert_array_equal(o64, es)
