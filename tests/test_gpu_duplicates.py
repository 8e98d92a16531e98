"""All-pairs near-duplicate search (``SearchIndex::find_duplicates``, ``index.rs:325-348``) on the
GPU through the C ABI, bit-exact against the oracle (``oracle/scan.py:find_duplicates``): pairs,
order and f64 scores, at the reference's default threshold and at a low threshold with thousands of
pairs, across strip boundaries of the tensor-core GEMM, with a row offset, and the empty cases.
When more candidates reach the threshold than one pass keeps, the cut is raised until the best
max_pairs fit (checked with a small test capacity, ``RV_DUP_CAP_RECORDS``)."""

import numpy as np
import pytest

from oracle import scan
from ripvec_b200 import synth
from ripvec_b200._lib import RvError
from ripvec_b200.index import SearchIndex

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rows():
    n, dim = 3000, 128
    db = synth.normalized_gaussian(n, dim, seed=51)
    rng = np.random.default_rng(52)
    near = db[5] + 0.05 * rng.standard_normal((20, dim)).astype(np.float32)
    db[100:120] = near / np.linalg.norm(near, axis=1, keepdims=True)
    db[2999] = db[0]  # exact copy across the last strip
    return db


def check(got, want):
    a, b, s, s64 = got
    ea, eb, es = want
    np.testing.assert_array_equal(a, ea)
    np.testing.assert_array_equal(b, eb)
    np.testing.assert_array_equal(s64, es)
    np.testing.assert_array_equal(s, es.astype(np.float32))


@pytest.mark.parametrize("threshold,max_pairs", [(0.85, 20), (0.85, 1000), (0.25, 10**6)])
def test_find_duplicates_bit_exact(cuda_device, rows, threshold, max_pairs):
    got = SearchIndex(rows).duplicate_pairs(threshold, max_pairs)
    want = scan.find_duplicates(rows, threshold, max_pairs)
    check(got, want)
    if threshold == 0.25:
        assert len(got[0]) > 1000  # many candidates near the threshold
    else:
        assert (got[0][0], got[1][0]) == (0, 2999)


def test_strip_boundaries_and_row_offset(cuda_device, rows, monkeypatch):
    want = scan.find_duplicates(rows, 0.3, 10**6)
    monkeypatch.setenv("RV_DUP_STRIP_ROWS", "512")  # six GEMM strips instead of one
    check(SearchIndex(rows).duplicate_pairs(0.3, 10**6), want)
    a, b, s, s64 = SearchIndex(rows, base=7).duplicate_pairs(0.3, 10**6)
    np.testing.assert_array_equal(a, want[0] + 7)
    np.testing.assert_array_equal(b, want[1] + 7)
    np.testing.assert_array_equal(s64, want[2])


def test_dim_768_and_empty_cases(cuda_device):
    db = synth.normalized_gaussian(1500, 768, seed=53)
    db[700] = db[3]
    db[701] = db[3] * 0.9 + db[4] * 0.1
    db[701] /= np.linalg.norm(db[701])
    idx = SearchIndex(db)
    check(idx.duplicate_pairs(0.8, 20), scan.find_duplicates(db, 0.8, 20))
    res = idx.find_duplicates(0.8, 20)
    assert res[0][:2] == (3, 700) and all(x < y for x, y, _ in res)
    assert SearchIndex(db[:1]).find_duplicates(0.0, 10) == []
    assert idx.find_duplicates(0.5, 0) == []


@pytest.fixture(scope="module")
def crowded():
    """600 rows: 300 noisy copies of one direction (44,850 pairs between 0.9 and 1) and 300
    unrelated rows."""
    dim = 128
    rng = np.random.default_rng(60)
    c = rng.standard_normal(dim).astype(np.float32)
    near = c + 0.25 * rng.standard_normal((300, dim)).astype(np.float32)
    db = np.concatenate([near, synth.normalized_gaussian(300, dim, seed=61)])
    return (db / np.linalg.norm(db, axis=1, keepdims=True)).astype(np.float32)


@pytest.mark.parametrize("max_pairs", [20, 1000])
def test_overflowing_threshold_raises_the_cut(cuda_device, crowded, monkeypatch, max_pairs):
    monkeypatch.setenv("RV_DUP_CAP_RECORDS", "2048")  # far fewer than the 44,850 crowded pairs
    want = scan.find_duplicates(crowded, 0.5, max_pairs)
    assert len(want[0]) == max_pairs
    check(SearchIndex(crowded).duplicate_pairs(0.5, max_pairs), want)


def test_no_cut_fits_is_an_error(cuda_device, monkeypatch):
    monkeypatch.setenv("RV_DUP_CAP_RECORDS", "2048")
    db = np.repeat(synth.normalized_gaussian(1, 128, seed=62), 300, axis=0)  # 44,850 pairs at 1.0
    idx = SearchIndex(db)
    with pytest.raises(RvError):
        idx.duplicate_pairs(0.5, 20)
    monkeypatch.setenv("RV_DUP_CAP_RECORDS", "65536")  # the same index, with room for every pair
    a, b, s, _ = idx.duplicate_pairs(0.5, 20)
    assert len(a) == 20 and (a[0], b[0]) == (0, 1)
