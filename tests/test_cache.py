"""The embedding store's import side on the CPU (``rv_cache_decode``, host-only C++): the
reference's own FileCache tests (``crates/ripvec-core/src/cache/file_cache.rs:113-190``: a one-chunk
round trip, an empty cache, garbage bytes) plus the formats around them (zstd with and without a
content size, the bare legacy archive, the portable "BC" form, truncated and inconsistent objects)
and ``load_all_from_store``'s skipping of corrupt objects (``cache/reindex.rs:537-603``).  The
archives are built by ``file_cache_objects`` from rkyv 0.8's default layout; see its notes."""

import numpy as np
import pytest

from file_cache_objects import archive, file_cache, zstd_frame
from ripvec_b200 import _lib as L
from ripvec_b200.cache import decode_file_cache, load_file_caches, read_shard


def test_round_trip_like_the_reference():
    obj = file_cache(["foo"], [1.0, 2.0, 3.0, 4.0], 4)
    assert obj[:4] == bytes([0x28, 0xB5, 0x2F, 0xFD])
    e = decode_file_cache(obj)
    np.testing.assert_array_equal(e, [[1.0, 2.0, 3.0, 4.0]])


def test_empty_cache_keeps_hidden_dim():
    e = decode_file_cache(file_cache([], np.zeros(0, np.float32), 384))
    assert e.shape == (0, 384)


def test_garbage_is_an_error():
    with pytest.raises(L.RvError) as ex:
        decode_file_cache(b"garbage data")
    assert ex.value.code == L.RV_E_IO


@pytest.mark.parametrize("form", ["stream", "frame", "bare"])
def test_forms_decode_bit_exact(form):
    rng = np.random.default_rng(3)
    emb = rng.standard_normal((7, 768)).astype(np.float32)
    names = [f"chunk{i}" for i in range(7)]
    if form == "bare":
        obj = archive(names, emb, 768)
    else:
        obj = file_cache(names, emb, 768, stream=form == "stream")
    np.testing.assert_array_equal(decode_file_cache(obj), emb)


def test_portable_form_is_refused():
    obj = b"BC" + zstd_frame(archive(["a"], np.ones(64, np.float32), 64))
    with pytest.raises(L.RvError) as ex:
        decode_file_cache(obj)
    assert ex.value.code == L.RV_E_IO


def test_malformed_objects():
    good = archive(["a", "b"], np.ones((2, 64), np.float32), 64)
    with pytest.raises(L.RvError):
        decode_file_cache(file_cache(["a"], np.ones(64, np.float32), 64)[:-5])  # truncated frame
    with pytest.raises(L.RvError):
        decode_file_cache(good[:-1])  # not a whole archive
    with pytest.raises(L.RvError):
        decode_file_cache(archive(["a"], np.ones(64, np.float32), 64, n_floats=10**6))  # past the end
    with pytest.raises(L.RvError):
        decode_file_cache(archive(["a"], np.ones(64, np.float32), 0))  # hidden_dim 0


def test_rows_are_the_chunks_with_a_whole_slice():
    # Three chunks but only 2.5 rows of floats: chunk 2 is dropped, as load_all_from_store does.
    emb = np.arange(160, dtype=np.float32)
    e = decode_file_cache(file_cache(["a", "b", "c"], emb, 64))
    np.testing.assert_array_equal(e, emb[:128].reshape(2, 64))


def test_size_query_and_capacity():
    import ctypes as C

    lib = L.lib()
    obj = file_cache(["a", "b"], np.ones((2, 64), np.float32), 64)
    buf = (C.c_uint8 * len(obj)).from_buffer_copy(obj)
    rows, dim = C.c_int64(), C.c_int32()
    assert lib.rv_cache_decode(buf, len(obj), None, 0, C.byref(rows), C.byref(dim)) == L.RV_OK
    assert (rows.value, dim.value) == (2, 64)
    small = np.empty(100, np.float32)
    assert lib.rv_cache_decode(buf, len(obj), small.ctypes.data, 100, C.byref(rows), C.byref(dim)) == L.RV_E_INVALID
    assert b"need 128" in lib.rv_cache_last_error()


def test_load_skips_corrupt_objects_in_order():
    rng = np.random.default_rng(4)
    a, b = rng.standard_normal((3, 64)).astype(np.float32), rng.standard_normal((2, 64)).astype(np.float32)
    other_dim = file_cache(["x"], np.ones(128, np.float32), 128)
    objs = [file_cache(["1", "2", "3"], a, 64), b"garbage data", other_dim, file_cache(["4", "5"], b, 64)]
    emb, counts, skipped = load_file_caches(objs)
    np.testing.assert_array_equal(emb, np.concatenate([a, b]))
    assert counts == [3, 0, 0, 2] and skipped == [1, 2]


def test_shard_file_errors(tmp_path):
    p = tmp_path / "bad.shard"
    p.write_bytes(b"RVSHARD1" + b"\0" * 4)
    with pytest.raises(ValueError):
        read_shard(p)
