"""Exact cosine ranking — restatement of the reference search path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``rank`` follows ``SearchIndex::rank`` (``crates/ripvec-core/src/index.rs:172-186``): a dimension
check (wrong or empty query -> no results), scores ``embeddings @ query`` (``similarity.rs:24-26``),
``score >= threshold`` filter, sort by descending score.  The reference's ``sort_unstable_by``
leaves the order of equal scores unspecified; this build fixes it to (score desc, row asc), the
order ``rrf_fuse`` uses (``hybrid.rs:198-200``).

``ln_truncate`` / ``rank_cascade`` restate the MRL cascade (``index.rs:99-132``, ``:245-297``) and
``find_duplicates`` the all-pairs search (``index.rs:325-348``).

``topk_exact`` is the bit-exact definition the GPU scan is checked against: rows and query are
bf16 values, each score is the sequential sum over d = 0..dim-1 in float64 of the (exact)
bf16 x bf16 products, results are ordered by (score desc, row asc), the best k are kept, and
rows scoring below ``threshold`` are dropped after selection.
"""

from __future__ import annotations

import numpy as np

from . import ops


def dot_product(a, b) -> float:
    """``similarity::dot_product`` (``similarity.rs:12-15``)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    s = np.float32(0.0)
    for x, y in zip(a, b):
        s = np.float32(s + np.float32(x * y))
    return float(s)


def rank_all(embeddings: np.ndarray, query: np.ndarray) -> np.ndarray:
    """``similarity::rank_all``: ``embeddings @ query`` in f32 (``similarity.rs:24-26``)."""
    embeddings = np.asarray(embeddings, np.float32)
    if embeddings.shape[0] == 0:
        return np.zeros(0, np.float32)
    return embeddings @ np.asarray(query, np.float32)


def rank(embeddings: np.ndarray, query, threshold: float) -> list[tuple[int, float]]:
    """``SearchIndex::rank`` (``index.rs:172-186``) with the (score desc, row asc) tie order."""
    embeddings = np.asarray(embeddings, np.float32)
    query = np.asarray(query, np.float32)
    if embeddings.ndim != 2 or query.shape != (embeddings.shape[1],) or embeddings.shape[0] == 0:
        return []
    s = rank_all(embeddings, query)
    keep = np.nonzero(s >= np.float32(threshold))[0]
    order = np.lexsort((keep, -s[keep].astype(np.float64)))
    return [(int(keep[i]), float(s[keep[i]])) for i in order]


def scores_exact(db_bf16: np.ndarray, q_bf16: np.ndarray) -> np.ndarray:
    """Float64 scores of every row, summing d = 0..dim-1 in order (products are exact in f64)."""
    db = np.asarray(db_bf16, np.float64)
    q = np.asarray(q_bf16, np.float64)
    acc = np.zeros(db.shape[0], np.float64)
    for d in range(db.shape[1]):
        acc += db[:, d] * q[d]
    return acc


def rank_exact(db: np.ndarray, query: np.ndarray, threshold: float):
    """``SearchIndex::rank`` (``index.rs:172-186``) under the exact score definition of
    ``topk_exact``: every row whose f64 score is ``>= threshold``, ordered by (score desc, row
    asc).  Returns ``(idx int64 [m], score64 [m])``."""
    dbb = ops.to_bf16(np.asarray(db, np.float32))
    qb = ops.to_bf16(np.asarray(query, np.float32).reshape(-1))
    s = scores_exact(dbb, qb)
    keep = np.nonzero(s >= np.float64(np.float32(threshold)))[0]
    order = np.lexsort((keep, -s[keep]))
    return keep[order].astype(np.int64), s[keep[order]]


def topk_exact(db: np.ndarray, queries: np.ndarray, k: int, threshold: float = -np.inf):
    """Reference top-k of every query: returns ``(idx int64 [nq,k], score64 [nq,k], count [nq])``.

    ``db`` and ``queries`` are rounded to bf16 first (the GPU index stores bf16 rows and rounds
    the f32 queries the same way).  Missing entries are ``-1`` / ``-inf``.
    """
    dbb = ops.to_bf16(np.asarray(db, np.float32))
    qb = ops.to_bf16(np.asarray(queries, np.float32).reshape(-1, dbb.shape[1]))
    nq, n = qb.shape[0], dbb.shape[0]
    out_i = np.full((nq, k), -1, np.int64)
    out_s = np.full((nq, k), -np.inf, np.float64)
    cnt = np.zeros(nq, np.int32)
    kk = min(k, n)
    if kk == 0 or nq == 0:
        return out_i, out_s, cnt
    # Sequential f64 sums over d for all queries at once, in row blocks (the order of the
    # additions per (query, row) is d = 0, 1, ..., dim-1, as in scores_exact).
    q64 = qb.astype(np.float64)
    best_i = [np.zeros(0, np.int64) for _ in range(nq)]
    best_s = [np.zeros(0, np.float64) for _ in range(nq)]
    step = max(1, (1 << 22) // max(nq, 1))
    for r0 in range(0, n, step):
        blk = dbb[r0:r0 + step].astype(np.float64)
        acc = np.zeros((nq, blk.shape[0]), np.float64)
        for d in range(blk.shape[1]):
            acc += q64[:, d:d + 1] * blk[None, :, d]
        rows = np.arange(r0, r0 + blk.shape[0], dtype=np.int64)
        for qi in range(nq):
            ii = np.concatenate([best_i[qi], rows])
            ss = np.concatenate([best_s[qi], acc[qi]])
            order = np.lexsort((ii, -ss))[:kk]
            best_i[qi], best_s[qi] = ii[order], ss[order]
    for qi in range(nq):
        sel = best_s[qi] >= threshold
        c = int(sel.sum())
        out_i[qi, :c] = best_i[qi][sel]
        out_s[qi, :c] = best_s[qi][sel]
        cnt[qi] = c
    return out_i, out_s, cnt


def ln_truncate(x: np.ndarray, t: int) -> np.ndarray:
    """MRL cascade transform of ``SearchIndex::new`` (``index.rs:99-132``) and of the query in
    ``rank_cascade`` (``index.rs:262-283``): LayerNorm over the full vector (mean, biased
    variance, ``1 / sqrt(var + 1e-5)``), the first ``t`` values, divided by their L2 norm floored
    at 1e-12.  Every sum runs over the dimensions in order in f32 (``iter().sum()``)."""
    x = np.asarray(x, np.float32)
    m, dim = x.shape
    t = min(t, dim)
    s = np.zeros(m, np.float32)
    for d in range(dim):
        s += x[:, d]
    mean = (s / np.float32(dim)).astype(np.float32)
    v = np.zeros(m, np.float32)
    for d in range(dim):
        c = (x[:, d] - mean).astype(np.float32)
        v += c * c
    var = (v / np.float32(dim)).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(var + np.float32(1e-5))).astype(np.float32)
    nn = np.zeros(m, np.float32)
    for j in range(t):
        ln = ((x[:, j] - mean) * inv).astype(np.float32)
        nn += ln * ln
    norm = np.maximum(np.sqrt(nn), np.float32(1e-12)).astype(np.float32)
    ln = ((x[:, :t] - mean[:, None]) * inv[:, None]).astype(np.float32)
    return (ln / norm[:, None]).astype(np.float32)


def rank_cascade(rows: np.ndarray, query, top_k: int, threshold: float, cascade_dim: int | None):
    """``SearchIndex::rank_cascade`` (``index.rs:245-297``) for one query: ``(idx int64 [m],
    score f64 [m])``, m <= top_k.  Phase 1 is the exact top ``max(100, 3 top_k)`` of the
    truncated rows (stored in bf16) against the truncated query; phase 2 re-scores those rows
    with the full rows (``scores_exact``), keeps ``score >= threshold`` and the best ``top_k`` by
    (score desc, row asc).  ``cascade_dim=None``: no truncated matrix, the exact top-k (the
    reference's ``rank`` fallback, truncated by its callers)."""
    rows = np.asarray(rows, np.float32)
    q = np.asarray(query, np.float32).reshape(1, -1)
    if cascade_dim is None:
        ei, es, ec = topk_exact(rows, q, top_k, threshold)
        return ei[0, :ec[0]], es[0, :ec[0]]
    rb = ops.to_bf16(rows)
    tr = ops.to_bf16(ln_truncate(rb, cascade_dim))
    return rank_cascade_prepared(rb, tr, q[0], top_k, threshold, cascade_dim)


def rank_cascade_prepared(rb: np.ndarray, tr: np.ndarray, query, top_k: int, threshold: float, cascade_dim: int):
    """``rank_cascade``'s query work on an index already built: ``rb`` the bf16 rows (as f32),
    ``tr`` their bf16 truncated LayerNorm rows (``ln_truncate``)."""
    q = np.asarray(query, np.float32).reshape(1, -1)
    tq = ln_truncate(q, cascade_dim)
    pre = max(100, 3 * top_k)
    ci, _, cc = topk_exact(tr, tq, pre)
    cand = ci[0, :cc[0]]
    exact = scores_exact(rb[cand], ops.to_bf16(q[0]))
    keep = exact >= threshold
    cand, exact = cand[keep], exact[keep]
    order = np.lexsort((cand, -exact))[:top_k]
    return cand[order].astype(np.int64), exact[order]


def find_duplicates(rows: np.ndarray, threshold: float, max_pairs: int):
    """``SearchIndex::find_duplicates`` (``index.rs:325-348``): pairs (a, b), a < b, of the
    bf16-rounded rows whose exact score (sequential f64 sum over d of the bf16 products) is
    ``>= threshold``, ordered by (score desc, a asc, b asc), at most ``max_pairs``.  Returns
    ``(a int64 [m], b int64 [m], score f64 [m])``.  The reference scores with one f32 BLAS GEMM
    and leaves the order of equal scores to ``sort_unstable_by``."""
    rb = ops.to_bf16(np.asarray(rows, np.float32)).astype(np.float64)
    n = rb.shape[0]
    if n < 2 or max_pairs <= 0:
        e = np.zeros(0, np.int64)
        return e, e, np.zeros(0, np.float64)
    thr = np.float64(np.float32(threshold))
    rt = np.ascontiguousarray(rb.T)
    aa, bb, ss = [], [], []
    for r0 in range(0, n - 1, 128):  # upper-triangle row blocks whose accumulators stay in cache
        r1 = min(n, r0 + 128)
        acc = np.zeros((r1 - r0, n - r0), np.float64)
        prod = np.empty_like(acc)
        for d in range(rb.shape[1]):
            np.multiply(rt[d, r0:r1, None], rt[d, None, r0:], out=prod)
            np.add(acc, prod, out=acc)
        i, j = np.nonzero(acc >= thr)
        up = (j + r0) > (i + r0)
        aa.append(i[up] + r0)
        bb.append(j[up] + r0)
        ss.append(acc[i[up], j[up]])
    a, b, sc = np.concatenate(aa), np.concatenate(bb), np.concatenate(ss)
    order = np.lexsort((b, a, -sc))[:max_pairs]
    return a[order].astype(np.int64), b[order].astype(np.int64), sc[order]


def rank_cascade_f32(rows: np.ndarray, tr: np.ndarray, query, top_k: int, threshold: float, cascade_dim: int):
    """The reference's own arithmetic for ``rank_cascade`` (``index.rs:245-297``) on a built index
    (``tr`` = ``ln_truncate(rows, cascade_dim)``): the truncated query, an f32 GEMV over ``tr``, a
    full sort of the scores, the first ``max(100, 3 top_k)``, full-dimension f32 dot products for
    those, threshold, sort, ``top_k``.  Used as the timed CPU baseline; parity uses
    ``rank_cascade``."""
    q = np.asarray(query, np.float32).reshape(1, -1)
    tq = ln_truncate(q, cascade_dim)[0]
    s = np.asarray(tr, np.float32) @ tq
    cand = np.argsort(-s, kind="stable")[:max(100, 3 * top_k)]
    full = np.asarray(rows, np.float32)[cand] @ q[0]
    keep = full >= np.float32(threshold)
    cand, full = cand[keep], full[keep]
    order = np.argsort(-full, kind="stable")[:top_k]
    return cand[order], full[order]


def find_duplicates_f32(rows: np.ndarray, threshold: float, max_pairs: int, block: int = 4096):
    """The reference's own arithmetic for ``find_duplicates`` (``index.rs:325-348``): the f32
    similarity matrix E Eᵀ by BLAS (here in row blocks of the upper triangle), pairs a < b with
    score >= threshold, sorted by descending score, the first ``max_pairs``.  Ties are left as
    the sort leaves them (the reference uses ``sort_unstable_by``).  Used as the timed CPU
    baseline; parity uses ``find_duplicates``."""
    e = np.ascontiguousarray(rows, np.float32)
    n = e.shape[0]
    aa, bb, ss = [], [], []
    for r0 in range(0, n, block):
        r1 = min(n, r0 + block)
        s = e[r0:r1] @ e[r0:].T
        i, j = np.nonzero(s >= np.float32(threshold))
        up = j > i
        aa.append(i[up] + r0)
        bb.append(j[up] + r0)
        ss.append(s[i[up], j[up]])
    a, b, sc = np.concatenate(aa), np.concatenate(bb), np.concatenate(ss)
    order = np.argsort(-sc, kind="stable")[:max_pairs]
    return a[order], b[order], sc[order]


def merge_topk(idx_lists: np.ndarray, score_lists: np.ndarray, k: int, threshold: float = -np.inf):
    """Merge per-shard results ``[n_lists, nq, k]`` into the global best k by (score desc, idx asc)."""
    n_lists, nq, kk = idx_lists.shape
    out_i = np.full((nq, k), -1, np.int64)
    out_s = np.full((nq, k), -np.inf, np.float64)
    for q in range(nq):
        ii = idx_lists[:, q, :].reshape(-1)
        ss = score_lists[:, q, :].reshape(-1)
        valid = ii >= 0
        ii, ss = ii[valid], ss[valid]
        order = np.lexsort((ii, -ss))[:k]
        order = order[ss[order] >= threshold]
        out_i[q, :len(order)] = ii[order]
        out_s[q, :len(order)] = ss[order]
    return out_i, out_s
