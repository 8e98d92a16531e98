"""The embedding store end to end on the GPU: per-file cache objects decoded into one matrix,
searched exactly (``cache/reindex.rs:274-302`` builds the index from them), and a device index
shard exported (``rv_index_export``) to a file and loaded back bit for bit."""

import ctypes as C

import numpy as np
import pytest

from file_cache_objects import file_cache
from oracle import scan
from ripvec_b200 import _lib as L
from ripvec_b200 import synth
from ripvec_b200.cache import load_file_caches, load_shard, read_shard, save_shard
from ripvec_b200.index import SearchIndex

pytestmark = pytest.mark.gpu


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bf16 of f32 values, as uint16."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def test_cache_objects_to_exact_search(cuda_device):
    rng = np.random.default_rng(70)
    sizes = rng.integers(1, 40, 50)
    db = synth.normalized_gaussian(int(sizes.sum()), 768, seed=71)
    objs, at = [], 0
    for s in sizes:
        objs.append(file_cache([f"c{i}" for i in range(s)], db[at:at + s], 768))
        at += s
    emb, counts, skipped = load_file_caches(objs)
    assert skipped == [] and counts == list(sizes)
    np.testing.assert_array_equal(emb, db)
    q = synth.normalized_gaussian(9, 768, seed=72)
    idx = SearchIndex(emb)
    got = idx.topk(q, 25, with_f64=True)
    ei, es, _ = scan.topk_exact(emb, q, 25)
    np.testing.assert_array_equal(got[0], ei)
    np.testing.assert_array_equal(got[3], es)


def test_shard_round_trip(cuda_device, tmp_path):
    import torch

    db = synth.normalized_gaussian(3001, 384, seed=73)
    idx = SearchIndex(db, base=500)
    bits = idx.export_rows(bf16_bits=True)
    np.testing.assert_array_equal(bits, bf16_bits(db))
    np.testing.assert_array_equal(idx.export_rows(10, 5), (bits[10:15].astype(np.uint32) << 16).view(np.float32))
    path = tmp_path / "part0.shard"
    save_shard(idx, path, base=500)
    rows, base = read_shard(path)
    assert base == 500 and rows.shape == (3001, 384)
    back = load_shard(path)
    np.testing.assert_array_equal(back.export_rows(bf16_bits=True), bits)
    q = synth.normalized_gaussian(4, 384, seed=74)
    a, b = idx.topk(q, 10), back.topk(q, 10)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)
    assert a[0].min() >= 500
    # device destinations, both dtypes
    lib = L.lib()
    d16 = torch.empty(7, 384, dtype=torch.bfloat16, device="cuda")
    d32 = torch.empty(7, 384, dtype=torch.float32, device="cuda")
    assert lib.rv_index_export(idx._h, 100, 7, L.RV_DTYPE_BF16, C.c_void_p(d16.data_ptr()), 1) == L.RV_OK
    assert lib.rv_index_export(idx._h, 100, 7, L.RV_DTYPE_F32, C.c_void_p(d32.data_ptr()), 1) == L.RV_OK
    np.testing.assert_array_equal(d16.view(torch.int16).cpu().numpy().view(np.uint16), bits[100:107])
    np.testing.assert_array_equal(d32.cpu().numpy(), (bits[100:107].astype(np.uint32) << 16).view(np.float32))
    assert lib.rv_index_export(idx._h, 3000, 2, L.RV_DTYPE_F32, C.c_void_p(d32.data_ptr()), 1) == L.RV_E_INVALID
    idx.close()
    back.close()
