"""Exact top-k scan on the GPU through the C ABI: indices and f64 scores bit-exact against the
oracle when fed identical embeddings, with ties, thresholds, k > n, an empty index, ragged
sizes, row-sharded indexes merged on the device, and the reference's ``rank`` contract."""

from pathlib import Path

import numpy as np
import pytest

from helpers import scan_small_inputs
from oracle import scan
from ripvec_b200 import synth
from ripvec_b200.index import SearchIndex, merge_topk_device

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_golden_scan_bit_exact(cuda_device):
    g = np.load(GOLDEN / "scan_small.npz")
    db, q = scan_small_inputs()
    idx = SearchIndex(db)
    oi, os_, cnt, o64 = idx.topk(q, int(g["k"]), with_f64=True)
    np.testing.assert_array_equal(oi, g["idx"])
    np.testing.assert_array_equal(o64, g["s64"])
    assert list(oi[5, :2]) == [17, 2000]


@pytest.mark.parametrize("n,dim,nq,k", [(1, 64, 1, 1), (255, 128, 3, 10), (4097, 768, 5, 100),
                                        (200_000, 768, 4, 100), (20_000, 768, 130, 16), (50_000, 384, 2, 1000)])
def test_topk_bit_exact_vs_oracle(cuda_device, n, dim, nq, k):
    db = synth.normalized_gaussian(n, dim, seed=n + dim)
    q = synth.normalized_gaussian(nq, dim, seed=nq + 1)
    ei, es, ec = scan.topk_exact(db, q, k)
    oi, os_, cnt, o64 = SearchIndex(db).topk(q, k, with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(o64, es)
    np.testing.assert_array_equal(cnt, ec)


def test_fused_filter_many_queries_bit_exact(cuda_device):
    """Rows past the 65536-row prefix go through the filtering GEMM in growing blocks; 300 queries
    pad to 512 GEMM columns.  Result bit-exact against the oracle."""
    n, dim, nq, k = 200_000, 128, 300, 50
    db = synth.normalized_gaussian(n, dim, seed=11)
    q = synth.normalized_gaussian(nq, dim, seed=12)
    ei, es, ec = scan.topk_exact(db, q, k)
    oi, os_, cnt, o64 = SearchIndex(db).topk(q, k, with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(o64, es)
    np.testing.assert_array_equal(cnt, ec)


@pytest.mark.parametrize("n,dim,nq,k", [(300_000, 128, 1, 100), (30_000, 64, 128, 64), (30_000, 64, 129, 10)])
def test_fused_filter_small_batches_bit_exact(cuda_device, n, dim, nq, k):
    """Batches of at most 128 queries use 128-column filter tiles and blocks that grow 5x; 129
    queries take the 256-column tiles.  Bit-exact against the oracle either way."""
    db = synth.normalized_gaussian(n, dim, seed=17 + nq)
    q = synth.normalized_gaussian(nq, dim, seed=18 + nq)
    ei, es, ec = scan.topk_exact(db, q, k)
    oi, os_, cnt, o64 = SearchIndex(db).topk(q, k, with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(o64, es)
    np.testing.assert_array_equal(cnt, ec)


def test_fused_filter_overflow_falls_back(cuda_device):
    """Every row after the prefix is a near copy of the query, so each filter block keeps far more
    candidates than its buffer: the batch is redone on the chunked path and stays exact."""
    n, dim = 150_000, 128
    db = synth.normalized_gaussian(n, dim, seed=13)
    rng = np.random.default_rng(14)
    tail = db[0] + 0.01 * rng.standard_normal((n - 70_000, dim)).astype(np.float32)
    db[70_000:] = tail / np.linalg.norm(tail, axis=1, keepdims=True)
    q = db[0:2].copy()
    ei, es, ec = scan.topk_exact(db, q, 100)
    oi, os_, cnt, o64 = SearchIndex(db).topk(q, 100, with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(o64, es)


def test_fused_filter_matches_chunked_path(cuda_device, monkeypatch):
    """The same index answered with the filter and with RV_SCAN_FILTER=0 (every row through the
    chunked GEMM + select) gives identical indices and f64 scores."""
    db = synth.normalized_gaussian(300_000, 384, seed=15)
    q = synth.normalized_gaussian(64, 384, seed=16)
    a = SearchIndex(db).topk(q, 100, with_f64=True)
    monkeypatch.setenv("RV_SCAN_FILTER", "0")
    b = SearchIndex(db).topk(q, 100, with_f64=True)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_threshold_k_larger_than_n_and_empty_index(cuda_device):
    db = synth.normalized_gaussian(300, 64, seed=3)
    q = synth.normalized_gaussian(2, 64, seed=4)
    ei, es, ec = scan.topk_exact(db, q, 500, threshold=0.05)
    oi, os_, cnt, o64 = SearchIndex(db).topk(q, 500, threshold=0.05, with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(cnt, ec)
    empty = SearchIndex(np.zeros((0, 64), np.float32))
    oi, os_, cnt = empty.topk(q, 5)
    assert (oi == -1).all() and (cnt == 0).all()
    assert empty.rank(q[0], 0.0) == []


def test_many_duplicates_need_the_wide_pass(cuda_device):
    """300 identical rows tie at the top: the margin guard must widen the candidate list and the
    result must still be the lowest row indices."""
    db = synth.normalized_gaussian(5000, 128, seed=5)
    db[1000:1300] = db[7]
    q = db[7:8].copy()
    ei, es, _ = scan.topk_exact(db, q, 100)
    oi, _, _, o64 = SearchIndex(db).topk(q, 100, with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    assert oi[0, 0] == 7 and list(oi[0, 1:4]) == [1000, 1001, 1002]


def test_rank_contract(cuda_device):
    """``SearchIndex::rank`` cases of the reference (index.rs:414-464) on the GPU index."""
    e = np.zeros((3, 64), np.float32)
    e[0, :2] = [0.2, 0.8]
    e[1, :2] = [0.9, 0.1]
    e[2, :2] = [0.5, 0.5]
    idx = SearchIndex(e)
    qv = np.zeros(64, np.float32)
    qv[0] = 1.0
    res = idx.rank(qv, 0.3)
    assert [r for r, _ in res] == [1, 2] and res[0][1] > res[1][1]
    assert idx.rank(qv[:63], 0.0) == []
    assert idx.rank(np.zeros(0, np.float32), 0.0) == []


@pytest.mark.parametrize("threshold", [0.0, -1.0, 0.05])
def test_rank_returns_every_row_above_threshold(cuda_device, threshold):
    """``rank`` is not capped: 5000 rows at threshold 0.0 (about half of them), -1.0 (all 5000)
    and 0.05, in the oracle's (score desc, row asc) order with bit-identical f64 scores; two
    duplicated rows tie and must come out lowest row first.  MCP ``find_similar`` ranks at 0.0 and
    pages through the result (ripvec-mcp/src/tools.rs:563-570)."""
    db = synth.normalized_gaussian(5000, 768, seed=41)
    db[3000] = db[12]
    db[4999] = db[12]
    q = synth.normalized_gaussian(1, 768, seed=42)[0]
    ei, es = scan.rank_exact(db, q, threshold)
    idx = SearchIndex(db)
    oi, os_, o64 = idx.rank_arrays(q, threshold, with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(o64, es)
    if threshold == -1.0:
        assert len(oi) == 5000
    pos = {int(r): i for i, r in enumerate(oi)}
    if 12 in pos:
        assert pos[3000] == pos[12] + 1 and pos[4999] == pos[12] + 2
    res = idx.rank(q, threshold)
    assert [r for r, _ in res] == ei.tolist()
    # a capacity below the count returns the best ones and the total count
    oi2, _ = idx.rank_arrays(q, threshold, capacity=7)
    np.testing.assert_array_equal(oi2, ei[:7])
    assert [r for r, _ in idx.rank(q, threshold, top_k=3000)] == ei[:3000].tolist()


def test_rank_unfiltered_large_index(cuda_device):
    """threshold = -inf scores every row without the filter pass: 300k rows, order and scores
    against the oracle."""
    db = synth.normalized_gaussian(300_000, 128, seed=43)
    q = synth.normalized_gaussian(1, 128, seed=44)[0]
    ei, es = scan.rank_exact(db, q, -np.inf)
    oi, _, o64 = SearchIndex(db).rank_arrays(q, float("-inf"), with_f64=True)
    np.testing.assert_array_equal(oi, ei)
    np.testing.assert_array_equal(o64, es)


def test_sharded_indexes_merge_on_device(cuda_device):
    import torch

    n, dim, nq, k = 30_000, 768, 8, 50
    db = synth.normalized_gaussian(n, dim, seed=6)
    q = synth.normalized_gaussian(nq, dim, seed=7)
    ei, es, _ = scan.topk_exact(db, q, k)
    bounds = [0, 9_999, 20_000, n]
    qd = torch.from_numpy(q).cuda()
    idx_l, s64_l = [], []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        sh = SearchIndex(db[lo:hi], base=lo)
        oi = torch.empty(nq, k, dtype=torch.int64, device="cuda")
        os_ = torch.empty(nq, k, dtype=torch.float32, device="cuda")
        o64 = torch.empty(nq, k, dtype=torch.float64, device="cuda")
        sh.topk_device(qd, k, oi, os_, o64, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        idx_l.append(oi)
        s64_l.append(o64)
    mi, ms, m64 = merge_topk_device(torch.stack(idx_l), torch.stack(s64_l), k)
    np.testing.assert_array_equal(mi.cpu().numpy(), ei)
    np.testing.assert_array_equal(m64.cpu().numpy(), es)
