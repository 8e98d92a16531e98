"""MRL cascade search on the GPU through the C ABI, bit-exact against the oracle
(``oracle/scan.py`` ``ln_truncate`` / ``rank_cascade``, restating ``index.rs:99-132`` and
``:245-297``): the truncated matrix, results (indices and f64 scores) with thresholds and a
row offset, the clamp of the truncated dimension, and the fallback without a truncated matrix."""

import numpy as np
import pytest

from oracle import ops, scan
from ripvec_b200 import _lib, synth
from ripvec_b200.index import SearchIndex

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def data():
    n, dim = 5000, 256
    db = synth.normalized_gaussian(n, dim, seed=41)
    db[2000:2010] = db[5]  # duplicates: ties in both phases
    q = synth.normalized_gaussian(4, dim, seed=42)
    q[3] = db[5]
    return db, q


def test_truncated_rows_bit_exact(cuda_device, data):
    db, _ = data
    idx = SearchIndex(db, cascade_dim=64)
    assert idx.truncated_dim() == 64
    expect = ops.to_bf16(scan.ln_truncate(ops.to_bf16(db), 64))
    np.testing.assert_array_equal(idx.truncated_rows().view(np.uint32), expect.view(np.uint32))


@pytest.mark.parametrize("top_k,threshold", [(10, -np.inf), (50, 0.1)])
def test_rank_cascade_bit_exact(cuda_device, data, top_k, threshold):
    db, q = data
    idx = SearchIndex(db, cascade_dim=64)
    oi, _, cnt, o64 = idx.topk_cascade(q, top_k, threshold, with_f64=True)
    for i in range(len(q)):
        ei, es = scan.rank_cascade(db, q[i], top_k, threshold, 64)
        c = len(ei)
        assert cnt[i] == c
        np.testing.assert_array_equal(oi[i, :c], ei)
        np.testing.assert_array_equal(o64[i, :c], es)
        assert (oi[i, c:] == -1).all()
    assert list(oi[3, :3]) == [5, 2000, 2001]


def test_dim_768_truncated_256_with_row_offset(cuda_device):
    n, dim = 4096, 768
    db = synth.normalized_gaussian(n, dim, seed=43)
    q = synth.normalized_gaussian(1, dim, seed=44)
    idx = SearchIndex(db, base=1000, cascade_dim=256)
    oi, _, cnt, o64 = idx.topk_cascade(q, 20, with_f64=True)
    ei, es = scan.rank_cascade(db, q[0], 20, -np.inf, 256)
    np.testing.assert_array_equal(oi[0], ei + 1000)
    np.testing.assert_array_equal(o64[0], es)


def test_clamp_fallback_and_errors(cuda_device, data):
    db, q = data
    idx = SearchIndex(db)
    assert idx.truncated_dim() is None
    exact = idx.topk(q, 30, with_f64=True)
    fallback = idx.topk_cascade(q, 30, with_f64=True)
    for x, y in zip(exact, fallback):
        np.testing.assert_array_equal(x, y)
    assert SearchIndex(db, cascade_dim=1000).truncated_dim() == 256  # clamped to the row dimension
    with pytest.raises(_lib.RvError):
        SearchIndex(db, cascade_dim=100)  # not a multiple of 64
    idx2 = SearchIndex(db, cascade_dim=64)
    assert idx2.rank_cascade(q[0][:-1], 10, 0.0) == []
    with pytest.raises(_lib.RvError):
        idx2.topk_cascade(q, 683)
    res = idx2.rank_cascade(q[0], 5, 0.0)
    ei, _ = scan.rank_cascade(db, q[0], 5, 0.0, 64)
    assert [r for r, _ in res] == ei.tolist()
