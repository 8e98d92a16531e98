"""PolarQuant ("TurboQuant") search on the GPU through the C ABI, bit-exact against the oracle
(``oracle/turbo_quant.py``, a restatement of ``turbo_quant.rs`` and ``index.rs:196-234``):
codes, approximate scores, and ``rank_turboquant`` results (indices and f64 scores), with ties
at the pre-filter boundary, every query-batch width of the scan, 2-bit angles, the all-rows
case, the fallback without a corpus and the argument checks."""

import numpy as np
import pytest

from oracle import turbo_quant as tq
from ripvec_b200 import _lib, synth
from ripvec_b200.index import SearchIndex, polar_rotation

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def corpus():
    n, dim = 4100, 256  # not a multiple of 32: the last row group is partial
    db = synth.normalized_gaussian(n, dim, seed=31)
    db[3000:3040] = db[11]  # 41 identical rows: equal approximate and exact scores
    rot = polar_rotation(dim, 7)
    return db, rot, tq.encode(db, rot)


@pytest.fixture(scope="module")
def queries(corpus):
    db = corpus[0]
    q = synth.normalized_gaussian(15, db.shape[1], seed=32)  # 15 = scan batches of 8 + 4 + 2 + 1
    q[4] = db[11]
    return q


def u32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_codes_bit_exact(cuda_device, corpus):
    db, rot, (radii, bins) = corpus
    idx = SearchIndex(db)
    idx.build_turboquant(rot)
    assert idx.has_turboquant
    r, b = idx.turboquant_codes()
    np.testing.assert_array_equal(b, bins)
    np.testing.assert_array_equal(u32(r), u32(radii))


def test_approximate_scores_bit_exact(cuda_device, corpus, queries):
    db, rot, (radii, bins) = corpus
    idx = SearchIndex(db)
    idx.build_turboquant(rot)
    s = idx.turboquant_scores(queries)
    for i in range(len(queries)):
        expect = tq.scan_corpus(radii, bins, tq.prepare_query(queries[i], rot))
        np.testing.assert_array_equal(u32(s[i]), u32(expect))


@pytest.mark.parametrize("top_k,threshold", [(2, -np.inf), (10, -np.inf), (100, 0.05)])
def test_rank_turboquant_bit_exact(cuda_device, corpus, queries, top_k, threshold):
    """top_k 2 keeps 20 of the 41 tied rows of query 4 (lowest rows first) before rescoring."""
    db, rot, codes = corpus
    idx = SearchIndex(db)
    idx.build_turboquant(rot)
    oi, os_, cnt, o64 = idx.topk_turboquant(queries, top_k, threshold, with_f64=True)
    for i in range(len(queries)):
        ei, es = tq.rank_turboquant(db, queries[i], top_k, threshold, rot, codes=codes)
        c = len(ei)
        assert cnt[i] == c
        np.testing.assert_array_equal(oi[i, :c], ei)
        np.testing.assert_array_equal(o64[i, :c], es)
        assert (oi[i, c:] == -1).all()
    assert list(oi[4, :2]) == [11, 3000]


def test_dim_768_and_two_bit_angles(cuda_device):
    n, dim = 4096, 768
    db = synth.normalized_gaussian(n, dim, seed=33)
    q = synth.normalized_gaussian(2, dim, seed=34)
    rot = polar_rotation(dim, 42)
    idx = SearchIndex(db)
    idx.build_turboquant(rot)
    codes = tq.encode(db, rot)
    r, b = idx.turboquant_codes()
    np.testing.assert_array_equal(b, codes[1])
    np.testing.assert_array_equal(u32(r), u32(codes[0]))
    oi, _, cnt, o64 = idx.topk_turboquant(q, 100, with_f64=True)
    for i in range(2):
        ei, es = tq.rank_turboquant(db, q[i], 100, -np.inf, rot, codes=codes)
        np.testing.assert_array_equal(oi[i], ei)
        np.testing.assert_array_equal(o64[i], es)
    # 2-bit angles (4 levels): same radii, coarser bins.
    idx.build_turboquant(rot, bits=2)
    codes2 = tq.encode(db, rot, bits=2)
    r2, b2 = idx.turboquant_codes()
    np.testing.assert_array_equal(b2, codes2[1])
    s2 = idx.turboquant_scores(q[:1])
    np.testing.assert_array_equal(u32(s2[0]), u32(tq.scan_corpus(*codes2, tq.prepare_query(q[0], rot, bits=2))))


def test_all_rows_candidates_fallback_and_limits(cuda_device, corpus, queries):
    db, rot, _ = corpus
    idx = SearchIndex(db)
    exact = idx.topk(queries, 500, with_f64=True)
    # Without a corpus rank_turboquant is the exact top-k.
    nocorp = idx.topk_turboquant(queries, 500, with_f64=True)
    for x, y in zip(exact, nocorp):
        np.testing.assert_array_equal(x, y)
    # With one, 10 * 500 >= n rows makes every row a candidate: the same exact top-k.
    idx.build_turboquant(rot)
    allrows = idx.topk_turboquant(queries, 500, with_f64=True)
    for x, y in zip(exact, allrows):
        np.testing.assert_array_equal(x, y)
    with pytest.raises(_lib.RvError):
        idx.topk_turboquant(queries, 801)
    with pytest.raises(ValueError):
        idx.rank_turboquant(queries[0][:-1], 10, 0.0)
    res = idx.rank_turboquant(queries[0], 5, 0.0)
    ei, es = tq.rank_turboquant(db, queries[0], 5, 0.0, rot)
    assert [r for r, _ in res] == ei.tolist()
    assert SearchIndex(db[:4096], turboquant="auto").has_turboquant
    assert not SearchIndex(db[:2], turboquant="auto").has_turboquant


def test_device_entry_point_matches_host(cuda_device, corpus, queries):
    import torch

    db, rot, _ = corpus
    idx = SearchIndex(db)
    idx.build_turboquant(rot)
    hi, hs, _, h64 = idx.topk_turboquant(queries, 10, with_f64=True)
    qd = torch.from_numpy(queries).cuda()
    oi = torch.empty(len(queries), 10, dtype=torch.int64, device="cuda")
    os_ = torch.empty(len(queries), 10, dtype=torch.float32, device="cuda")
    o64 = torch.empty(len(queries), 10, dtype=torch.float64, device="cuda")
    idx.topk_turboquant_device(qd, 10, oi, os_, o64, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(oi.cpu().numpy(), hi)
    np.testing.assert_array_equal(o64.cpu().numpy(), h64)
