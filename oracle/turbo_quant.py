"""PolarQuant ("TurboQuant") compressed scan — restatement of the reference's approximate ranking.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``crates/ripvec-core/src/turbo_quant.rs`` and ``SearchIndex::rank_turboquant``
(``crates/ripvec-core/src/index.rs:196-234``):

* ``gram_schmidt_qr`` — modified Gram-Schmidt over the columns (``turbo_quant.rs:346-367``);
* ``angle_tables`` — ``theta_j = (j / levels) * 2 * PI - PI`` in f32 and its cos / sin
  (``turbo_quant.rs:104-109``);
* ``encode`` — rotation ``rotated = x R^T`` then, per pair (a, b), ``r = sqrt(a*a + b*b)`` and
  the angle bin ``min(trunc((atan2(b, a) + PI) / (2 PI) * levels), levels - 1)``
  (``turbo_quant.rs:161-188``, ``:311-318``);
* ``prepare_query`` — the rotated query's centroid table ``q_a cos_j + q_b sin_j``
  (``turbo_quant.rs:212-241``);
* ``scan_corpus`` — ``score = sum_i r_i * table[i, idx_i]`` accumulated pair by pair in f32
  (``turbo_quant.rs:248-289``);
* ``rank_turboquant`` — approximate scores of every row, the best ``min(10 top_k, n)`` kept,
  re-scored exactly, ``score >= threshold`` kept, sorted, truncated to ``top_k``
  (``index.rs:196-234``); without a compressed corpus it is ``rank`` (``index.rs:202-204``).

Order of operations fixed here (the reference leaves it to BLAS / libm):

* the rotation of a row or query sums ``x_d * R[j, d]`` sequentially over d = 0..dim-1 in f32,
  each product and each sum rounded (no fused multiply-add) — the reference's ``vectors.dot
  (&rotation.t())`` runs through OpenBLAS sgemm, whose accumulation order is its own;
* the angle is ``atan2`` evaluated in f64 and rounded to f32 (the correctly rounded f32 angle;
  the reference calls the platform's f32 ``atan2f``); the cos / sin tables likewise come from
  the f64 functions rounded to f32;
* rows are the bf16 values the GPU index stores (the reference encodes f32 rows); the LUT query
  is the f32 query, as in the reference;
* the exact re-rank is the sequential f64 sum of the bf16 products of row and bf16-rounded query
  (``scan.scores_exact``, the exact path's definition), ordered by (score desc, row asc); the
  approximate pre-filter is ordered by (approximate score desc, row asc) — the reference's
  ``sort_unstable_by`` leaves ties unordered.
"""

from __future__ import annotations

import math

import numpy as np

from . import ops
from . import scan

PI32 = np.float32(math.pi)  # the f32 nearest to pi, = Rust's std::f32::consts::PI
TURBOQUANT_MIN_CHUNKS = 4096  # index.rs:22


def gram_schmidt_qr(a: np.ndarray) -> np.ndarray:
    """Modified Gram-Schmidt on the columns of ``a`` in f32 (``turbo_quant.rs:346-367``): each
    column is normalised (skipped when its norm is below 1e-10), then removed from the later ones."""
    q = np.array(a, dtype=np.float32, copy=True)
    n = q.shape[1]
    for i in range(n):
        norm = np.float32(np.sqrt(np.sum(q[:, i] * q[:, i], dtype=np.float32)))
        if norm < 1e-10:
            continue
        q[:, i] = q[:, i] * np.float32(np.float32(1.0) / norm)
        if i + 1 < n:
            dots = (q[:, i][None, :] @ q[:, i + 1:]).astype(np.float32)
            q[:, i + 1:] -= dots * q[:, i][:, None]
    return q


def generate_rotation(dim: int, seed: int) -> np.ndarray:
    """A seeded orthogonal [dim, dim] f32 matrix: MGS of a standard-normal matrix
    (``turbo_quant.rs:335-343``).  The Gaussian source is numpy's generator, not the
    reference's ChaCha8 stream, so the matrix differs from the reference's for the same seed."""
    rng = np.random.default_rng(seed)
    return gram_schmidt_qr(rng.standard_normal((dim, dim)).astype(np.float32))


def angle_tables(levels: int) -> tuple[np.ndarray, np.ndarray]:
    """f32 cos / sin of ``theta_j = (j / levels) * 2 * PI - PI`` (``turbo_quant.rs:104-109``)."""
    cos_t = np.empty(levels, np.float32)
    sin_t = np.empty(levels, np.float32)
    for j in range(levels):
        theta = np.float32(np.float32(np.float32(np.float32(j) / np.float32(levels)) * np.float32(2.0)) * PI32)
        theta = np.float32(theta - PI32)
        cos_t[j] = np.float32(math.cos(float(theta)))
        sin_t[j] = np.float32(math.sin(float(theta)))
    return cos_t, sin_t


def rotate(x: np.ndarray, rotation: np.ndarray) -> np.ndarray:
    """``x R^T`` in f32, each output summed over d = 0..dim-1 in order with rounded products and
    sums (no fused multiply-add)."""
    x = np.asarray(x, np.float32)
    rt = np.ascontiguousarray(np.asarray(rotation, np.float32).T)  # rt[d] = column d of R
    out = np.zeros((x.shape[0], rt.shape[1]), np.float32)
    for r0 in range(0, x.shape[0], 256):  # row blocks whose accumulators stay in cache
        xb = x[r0:r0 + 256]
        acc = out[r0:r0 + 256]
        prod = np.empty_like(acc)
        for d in range(x.shape[1]):
            np.multiply(xb[:, d:d + 1], rt[d][None, :], out=prod)
            np.add(acc, prod, out=acc)
    return out


def encode_pairs(rotated: np.ndarray, levels: int) -> tuple[np.ndarray, np.ndarray]:
    """``encode_pair`` over every pair of the rotated rows (``turbo_quant.rs:311-318``): radii
    f32 [n, pairs] and angle bins u8 [n, pairs]."""
    a = np.ascontiguousarray(rotated[:, 0::2], np.float32)
    b = np.ascontiguousarray(rotated[:, 1::2], np.float32)
    radii = np.sqrt(a * a + b * b).astype(np.float32)
    theta = np.arctan2(b.astype(np.float64), a.astype(np.float64)).astype(np.float32)
    normalized = ((theta + PI32) / np.float32(np.float32(2.0) * PI32)).astype(np.float32)
    scaled = (normalized * np.float32(levels)).astype(np.float32)
    idx = np.clip(np.trunc(scaled), 0, None).astype(np.int64)
    idx = np.minimum(idx, levels - 1).astype(np.uint8)
    return radii, idx


def encode(rows: np.ndarray, rotation: np.ndarray, bits: int = 4) -> tuple[np.ndarray, np.ndarray]:
    """``PolarCodec::encode_batch`` of the bf16-rounded rows."""
    rows_bf16 = ops.to_bf16(np.asarray(rows, np.float32))
    return encode_pairs(rotate(rows_bf16, rotation), 1 << bits)


def prepare_query(query: np.ndarray, rotation: np.ndarray, bits: int = 4) -> np.ndarray:
    """``PolarCodec::prepare_query``: centroid table [pairs, levels] f32 of the f32 query."""
    levels = 1 << bits
    rq = rotate(np.asarray(query, np.float32).reshape(1, -1), rotation)[0]
    cos_t, sin_t = angle_tables(levels)
    qa = rq[0::2][:, None]
    qb = rq[1::2][:, None]
    return (qa * cos_t[None, :] + qb * sin_t[None, :]).astype(np.float32)


def scan_corpus(radii: np.ndarray, idx: np.ndarray, table: np.ndarray) -> np.ndarray:
    """``PolarCodec::scan_corpus``: approximate score of every row, pair by pair in f32."""
    n, pairs = radii.shape
    score = np.zeros(n, np.float32)
    for i in range(pairs):
        score += radii[:, i] * table[i, idx[:, i].astype(np.int64)]
    return score


def rank_turboquant(rows: np.ndarray, query: np.ndarray, top_k: int, threshold: float,
                    rotation: np.ndarray | None, bits: int = 4, codes=None):
    """``SearchIndex::rank_turboquant`` for one query: ``(idx int64 [m], score f64 [m])`` with
    m <= top_k.  ``rotation=None`` means no compressed corpus: the exact ranking truncated to
    top_k (the reference returns every row above the threshold; its callers truncate).
    ``codes`` = ``encode(rows, rotation, bits)`` when already computed."""
    rows = np.asarray(rows, np.float32)
    n = rows.shape[0]
    q = np.asarray(query, np.float32).reshape(1, -1)
    if rotation is None:
        ei, es, ec = scan.topk_exact(rows, q, top_k, threshold)
        c = int(ec[0])
        return ei[0, :c], es[0, :c]
    radii, idx = encode(rows, rotation, bits) if codes is None else codes
    approx = scan_corpus(radii, idx, prepare_query(q[0], rotation, bits))
    pre = min(top_k * 10, n)
    cand = np.lexsort((np.arange(n), -approx.astype(np.float64)))[:pre]
    exact = scan.scores_exact(ops.to_bf16(rows[cand]), ops.to_bf16(q[0]))
    keep = exact >= threshold
    cand, exact = cand[keep], exact[keep]
    order = np.lexsort((cand, -exact))[:top_k]
    return cand[order].astype(np.int64), exact[order]
