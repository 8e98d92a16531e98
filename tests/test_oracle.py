"""The CPU oracle against the reference's own known answers, its committed golden fixtures, an
independent float64 evaluation and the invariants the reference relies on (no GPU needed)."""

import json
from pathlib import Path

import numpy as np
import pytest

from helpers import TINY_CLASSIC, TINY_MODERN, classic_cfg, modern_cfg, row_cosines, scan_small_inputs
from oracle import classic_bert, modern_bert, ops, scan
from ripvec_b200 import synth

GOLDEN = Path(__file__).resolve().parent / "golden"
KA = json.loads((GOLDEN / "reference_known_answers.json").read_text())["cases"]


def _query(spec):
    if spec == "zeros384":
        return np.zeros(384, np.float32)
    if spec == "ones384":
        return np.ones(384, np.float32)
    return np.asarray(spec, np.float32)


def _embeddings(case):
    if "embeddings_shape" in case:
        return np.zeros(case["embeddings_shape"], np.float32)
    return np.asarray(case["embeddings"], np.float32)


@pytest.mark.parametrize("case", [c for c in KA if c["op"] != "invariant"], ids=lambda c: c["id"])
def test_reference_known_answer(case):
    op = case["op"]
    if op == "gelu":
        out = ops.gelu_tanh(np.asarray(case["input"], np.float32))
        for chk in case["checks"]:
            assert abs(out[chk["index"]] - chk["expect"]) < chk["tol"]
    elif op == "layer_norm":
        out = ops.layer_norm(np.asarray(case["input"], np.float32), np.asarray(case["weight"], np.float32),
                             np.asarray(case["bias"], np.float32), case["eps"])
        for chk in case["checks"]:
            assert abs(out[chk["row_mean"]].mean()) < chk["tol"]
    elif op == "gemm":
        out = ops.gemm(np.asarray(case["a"], np.float32), np.asarray(case["b"], np.float32), case["transpose_b"])
        np.testing.assert_allclose(out, case["expect"], atol=case["tol"])
    elif op == "embedding_lookup":
        out = ops.embedding_lookup(case["ids"], np.asarray(case["table"], np.float32))
        np.testing.assert_array_equal(out, np.asarray(case["expect"], np.float32))
    elif op == "cls_pool":
        out = ops.cls_pool(np.asarray(case["hidden"], np.float32), case["batch"], case["seq"])
        np.testing.assert_array_equal(out, np.asarray(case["expect"], np.float32))
    elif op == "dot":
        assert abs(scan.dot_product(case["a"], case["b"]) - case["expect"]) < case["tol"]
    elif op == "rank_all_vs_dot":
        e = _embeddings(case)
        s = scan.rank_all(e, case["query"])
        for i, row in enumerate(e):
            assert abs(s[i] - scan.dot_product(row, case["query"])) < case["tol"]
    elif op == "rank_all":
        s = scan.rank_all(_embeddings(case), _query(case["query"]))
        np.testing.assert_allclose(s, np.asarray(case["expect"], np.float32), atol=case.get("tol", 0))
    elif op == "rank":
        res = scan.rank(_embeddings(case), _query(case["query"]), case["threshold"])
        assert [r for r, _ in res] == case["expect_rows"]
        assert all(res[i][1] >= res[i + 1][1] for i in range(len(res) - 1))
    else:
        raise AssertionError(op)


def test_rope_table_matches_reference_formula():
    cos, sin = ops.rope_tables(64, 8192, 160000.0)
    assert cos.shape == (8192, 32) and cos.dtype == np.float32
    assert cos[0].tolist() == [1.0] * 32 and sin[0].tolist() == [0.0] * 32
    # freq = pos / theta^(2d/64); spot-check in float64 (the table itself is float32 libm)
    p, d = 5000, 3
    f = np.float32(p) / np.float32(160000.0 ** (2 * d / 64))
    assert abs(cos[p, d] - np.cos(np.float64(f))) < 1e-6


def test_golden_modernbert_fixture_reproduces():
    g = np.load(GOLDEN / "modernbert_tiny.npz")
    w = synth.random_weights(TINY_MODERN, seed=int(g["weight_seed"]), qk_std=float(g["qk_std"]))
    emb = modern_bert.embed_batch(w, modern_cfg(TINY_MODERN), g["ids"], g["cu"])
    np.testing.assert_allclose(emb, g["emb"], atol=1e-5)


def test_golden_classic_fixture_reproduces():
    g = np.load(GOLDEN / "classicbert_tiny.npz")
    w = synth.random_weights(TINY_CLASSIC, seed=int(g["weight_seed"]), qk_std=float(g["qk_std"]))
    cfg = classic_cfg(TINY_CLASSIC)
    np.testing.assert_allclose(classic_bert.embed_batch(w, cfg, g["ids"], g["cu"], "cls"), g["emb_cls"], atol=1e-5)
    np.testing.assert_allclose(classic_bert.embed_batch(w, cfg, g["ids"], g["cu"], "mean"), g["emb_mean"], atol=1e-5)


def test_golden_scan_fixture_reproduces():
    g = np.load(GOLDEN / "scan_small.npz")
    db, q = scan_small_inputs()
    idx, s64, _ = scan.topk_exact(db, q, int(g["k"]))
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_array_equal(s64, g["s64"])
    # the duplicated row ties with its original and loses on row index
    assert list(idx[5, :2]) == [17, 2000]


def test_modernbert_fp32_matches_fp64():
    w = synth.random_weights(TINY_MODERN, seed=3, qk_std=0.2)
    ids, cu = synth.packed_ids(np.array([7, 70, 150], np.int32), TINY_MODERN.vocab, seed=4)
    cfg = modern_cfg(TINY_MODERN)
    a = modern_bert.embed_batch(w, cfg, ids, cu, np.float32)
    b = modern_bert.embed_batch(w, cfg, ids, cu, np.float64)
    assert row_cosines(a, b).min() > 0.999999


def test_classic_fp32_matches_fp64():
    w = synth.random_weights(TINY_CLASSIC, seed=3, qk_std=0.2)
    ids, cu = synth.packed_ids(np.array([3, 40, 128], np.int32), TINY_CLASSIC.vocab, seed=4)
    cfg = classic_cfg(TINY_CLASSIC)
    a = classic_bert.embed_batch(w, cfg, ids, cu, "cls", np.float32)
    b = classic_bert.embed_batch(w, cfg, ids, cu, "cls", np.float64)
    assert row_cosines(a, b).min() > 0.999999


def test_embeddings_are_unit_norm_batch_independent_and_distinct():
    w = synth.random_weights(TINY_MODERN, seed=5)
    cfg = modern_cfg(TINY_MODERN)
    ids, cu = synth.packed_ids(np.array([12, 33, 80], np.int32), TINY_MODERN.vocab, seed=6)
    e = modern_bert.embed_batch(w, cfg, ids, cu)
    np.testing.assert_allclose(np.linalg.norm(e, axis=1), 1.0, atol=1e-4)  # backend/cpu.rs:865
    # batch independence: a chunk's embedding does not depend on its neighbours (catches the
    # reference CPU driver's multi-sequence gather quirk)
    alone = modern_bert.embed_sequence(w, cfg, ids[cu[1]:cu[2]])
    np.testing.assert_allclose(alone, e[1], atol=1e-6)
    cs = e @ e.T
    assert cs[0, 1] < 0.99 and cs[1, 2] < 0.99  # backend/cpu.rs:881
    assert modern_bert.embed_batch(w, cfg, ids[:0], np.zeros(1, np.int32)).shape == (0, cfg.hidden)


def test_local_window_ignores_far_keys():
    rng = np.random.default_rng(0)
    L, nh, d = 300, 2, 64
    q = rng.standard_normal((L, nh, d)).astype(np.float32)
    k = rng.standard_normal((L, nh, d)).astype(np.float32)
    v = rng.standard_normal((L, nh, d)).astype(np.float32)
    a = modern_bert._attention(q, k, v, 0.125, 64, np.float32)
    k2, v2 = k.copy(), v.copy()
    k2[200:] += 5.0
    v2[200:] -= 3.0
    b = modern_bert._attention(q, k2, v2, 0.125, 64, np.float32)
    np.testing.assert_array_equal(a[:136], b[:136])  # queries < 136 never see keys >= 200
    assert not np.allclose(a[136:], b[136:])


def test_scan_oracle_threshold_and_k_larger_than_n():
    db = synth.normalized_gaussian(50, 64, seed=1)
    q = synth.normalized_gaussian(2, 64, seed=2)
    idx, s64, cnt = scan.topk_exact(db, q, 80, threshold=0.1)
    for r in range(2):
        c = int(cnt[r])
        assert (s64[r, :c] >= 0.1).all() and (idx[r, c:] == -1).all()
        assert all(s64[r, i] >= s64[r, i + 1] for i in range(c - 1))


def test_scan_merge_equals_global_topk():
    db = synth.normalized_gaussian(1000, 64, seed=9)
    q = synth.normalized_gaussian(3, 64, seed=10)
    gi, gs, _ = scan.topk_exact(db, q, 20)
    parts = []
    for s in range(4):
        lo, hi = s * 250, (s + 1) * 250
        i, sc, _ = scan.topk_exact(db[lo:hi], q, 20)
        parts.append((np.where(i >= 0, i + lo, -1), sc))
    mi, ms = scan.merge_topk(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]), 20)
    np.testing.assert_array_equal(mi, gi)
    np.testing.assert_array_equal(ms, gs)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf], np.float32)
    r = ops.to_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == 1.015625 and r[3] == -2.5 and np.isinf(r[5])


@pytest.mark.parametrize("window_half", [-1, 64])
def test_threaded_oracle_attention_is_bit_identical_to_the_sequential_loop(monkeypatch, window_half):
    """The oracle runs the attention heads of long chunks on a thread pool, with one BLAS thread
    per call; every head must come out exactly as the sequential loop computes it with the same
    BLAS setting.  (The BLAS thread count itself can change the last bits of a GEMM, as for any
    BLAS caller: with several BLAS threads the sequential loop differs by about 1e-7 here.)"""
    from oracle import modern_bert

    rng = np.random.default_rng(11)
    L, nh, d = 1100, 4, 64
    q, k, v = (rng.standard_normal((L, nh, d)).astype(np.float32) for _ in range(3))
    threaded = modern_bert._attention(q, k, v, 0.125, window_half, np.float32)
    monkeypatch.setattr(modern_bert.os, "cpu_count", lambda: 1)
    with modern_bert._single_threaded_blas():
        sequential = modern_bert._attention(q, k, v, 0.125, window_half, np.float32)
    np.testing.assert_array_equal(threaded, sequential)
    np.testing.assert_allclose(threaded, modern_bert._attention(q, k, v, 0.125, window_half, np.float32), atol=1e-6)
