"""ModernBERT encoder forward — numpy restatement of the reference FP32 path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``crates/ripvec-core/src/backend/arch/modern_bert.rs``: embedding + LayerNorm
(:901-912), per layer pre-attention LayerNorm (identity for layer 0, :141-157), fused QKV
projection (:159-170), split into heads (``driver/cpu.rs:1089-1125``), RoPE with the global or
local table (:200-219, ``driver/cpu.rs:1155-1186``), scores ``q.k`` scaled by ``1/sqrt(d)`` with the
additive ``-1e9`` window mask on local layers (:250-284, ``driver/cpu.rs:1016-1074``), ``P V`` and
head merge (:286-322), output projection + residual (:324-344), pre-MLP LayerNorm (:362-372),
``Wi`` projection, split into value / gate and GeGLU (:374-401), ``Wo`` + residual (:403-423),
then final LayerNorm, mean pool and L2 normalisation (:1071-1111).

Each sequence is run on its own (batch of one): the reference CPU driver has no
``prepare_batch_unpadded`` override, so for multi-sequence batches its embedding gather takes
the first ``total_tokens`` ids of the padded array (``modern_bert.rs:901-902``,
``driver/cpu.rs:863``); running per sequence is the intended, batch-independent semantics.
"""

from __future__ import annotations

import contextlib
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

from . import ops


@dataclass(frozen=True)
class ModernBertConfig:
    """Mirrors ``ModernBertConfig`` (``driver/cpu.rs:620-667``)."""

    hidden: int = 768
    num_layers: int = 22
    num_heads: int = 12
    intermediate: int = 1152
    vocab: int = 50368
    max_position: int = 8192
    global_every_n: int = 3
    local_window: int = 128
    global_rope_theta: float = 160000.0
    local_rope_theta: float = 10000.0
    norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.num_heads


def weight_names(cfg: ModernBertConfig) -> list[str]:
    """Tensor names the reference loader reads (``driver/cpu.rs:521-616``)."""
    names = ["embeddings.tok_embeddings.weight", "embeddings.norm.weight", "final_norm.weight"]
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        names += [p + "attn.Wqkv.weight", p + "attn.Wo.weight"]
        if i > 0:
            names.append(p + "attn_norm.weight")
        names += [p + "mlp.Wi.weight", p + "mlp.Wo.weight", p + "mlp_norm.weight"]
    return names


_Q_BLOCK = 512  # query rows per score block: keeps [block, L] f32 small at L = 8192


@contextlib.contextmanager
def _single_threaded_blas():
    """One BLAS thread per call while the attention heads run on their own threads (the small
    per-block GEMMs gain nothing from more, and nested pools would oversubscribe the cores)."""
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:
        yield
        return
    with threadpool_limits(limits=1, user_api="blas"):
        yield


def _attention(q, k, v, scale, window_half, dt):
    """``q,k,v [L, heads, d]`` -> context ``[L, heads*d]``.  ``window_half < 0`` means global.

    Per head, the scores ``q k^T`` are BLAS GEMMs like the reference's ``gemm_batched``
    (``modern_bert.rs:250-263``), scaled and masked row by row (``s * scale + mask``,
    ``driver/cpu.rs:1016-1074``), soft-maxed and multiplied by V (``:286-300``).  Rows are
    processed in blocks of ``_Q_BLOCK`` queries so that an 8192-token chunk never materialises
    ``[heads, L, L]``.  On windowed layers a block only forms scores for keys within
    ``window_half`` of its rows: every other key carries the additive ``-1e9`` mask, whose
    ``exp(s - max)`` is exactly 0 in f32, so leaving it out changes no softmax weight and adds
    only exact zeros to ``P V``.
    """
    L, nh, d = q.shape
    ctx = np.empty((L, nh, d), dtype=q.dtype)
    sc = dt(scale)

    def head(h):
        qh = np.ascontiguousarray(q[:, h, :])
        kh = np.ascontiguousarray(k[:, h, :])
        vh = np.ascontiguousarray(v[:, h, :])
        for i0 in range(0, L, _Q_BLOCK):
            i1 = min(L, i0 + _Q_BLOCK)
            j0, j1 = (0, L) if window_half < 0 else (max(0, i0 - window_half), min(L, i1 + window_half))
            s = (qh[i0:i1] @ kh[j0:j1].T) * sc
            if window_half >= 0:
                far = np.abs(np.arange(i0, i1)[:, None] - np.arange(j0, j1)[None, :]) > window_half
                s = s + np.where(far, dt(-1e9), dt(0.0))
            ctx[i0:i1, h, :] = ops.softmax_rows(s) @ vh[j0:j1]

    # The heads are independent and write disjoint slices of ctx, so they run on a thread pool
    # (numpy releases the GIL inside these array operations); each head's arithmetic is that of a
    # sequential loop with one BLAS thread per call (the BLAS thread count can change the last
    # bits of a GEMM, as for any BLAS caller).  Long chunks only: short ones are not worth it.
    workers = min(nh, os.cpu_count() or 1) if L >= 1024 else 1
    if workers <= 1:
        for h in range(nh):
            head(h)
    else:
        with _single_threaded_blas(), ThreadPoolExecutor(max_workers=workers) as pool:
            list(pool.map(head, range(nh)))
    return ctx.reshape(L, nh * d)


def forward_hidden(w: dict, cfg: ModernBertConfig, ids: np.ndarray, dtype=np.float32) -> np.ndarray:
    """Hidden states after the last layer, before the final LayerNorm: ``[L, hidden]``."""
    dt = np.dtype(dtype).type
    W = {k: v.astype(dtype, copy=False) for k, v in w.items()}
    H, nh, hd, I = cfg.hidden, cfg.num_heads, cfg.head_dim, cfg.intermediate
    L = len(ids)
    x = ops.layer_norm(ops.embedding_lookup(ids, W["embeddings.tok_embeddings.weight"]),
                       W["embeddings.norm.weight"], None, cfg.norm_eps)
    tables = {
        True: tuple(t.astype(dtype) for t in ops.rope_tables(hd, cfg.max_position, cfg.global_rope_theta)),
        False: tuple(t.astype(dtype) for t in ops.rope_tables(hd, cfg.max_position, cfg.local_rope_theta)),
    }
    scale = 1.0 / np.sqrt(np.float32(hd))
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        is_global = i % cfg.global_every_n == 0
        h = x if i == 0 else ops.layer_norm(x, W[p + "attn_norm.weight"], None, cfg.norm_eps)
        qkv = ops.gemm_bt(h, W[p + "attn.Wqkv.weight"])
        q = qkv[:, :H].reshape(L, nh, hd)
        k = qkv[:, H:2 * H].reshape(L, nh, hd)
        v = qkv[:, 2 * H:].reshape(L, nh, hd)
        cos, sin = tables[is_global]
        q = ops.apply_rope(q, cos, sin)
        k = ops.apply_rope(k, cos, sin)
        ctx = _attention(q, k, v, scale, -1 if is_global else cfg.local_window // 2, dt)
        x = ops.gemm_bt(ctx, W[p + "attn.Wo.weight"]) + x
        y = ops.layer_norm(x, W[p + "mlp_norm.weight"], None, cfg.norm_eps)
        u = ops.gemm_bt(y, W[p + "mlp.Wi.weight"])
        a = ops.gelu_tanh(u[:, :I]) * u[:, I:]
        x = ops.gemm_bt(a, W[p + "mlp.Wo.weight"]) + x
    return x


def embed_sequence(w: dict, cfg: ModernBertConfig, ids, dtype=np.float32) -> np.ndarray:
    """L2-normalised mean-pooled embedding of one sequence (``modern_bert.rs:1071-1111``)."""
    ids = np.asarray(ids, dtype=np.int64)
    if len(ids) == 0:
        return np.zeros(cfg.hidden, dtype)
    x = forward_hidden(w, cfg, ids, dtype)
    x = ops.layer_norm(x, w["final_norm.weight"].astype(dtype), None, cfg.norm_eps)
    return ops.l2_normalize(ops.mean_pool(x))


def embed_batch(w: dict, cfg: ModernBertConfig, ids: np.ndarray, cu_seqlens: np.ndarray,
                dtype=np.float32) -> np.ndarray:
    """``EmbedBackend::embed_batch`` over packed ids: ``[n_seqs, hidden]``, input order."""
    n = len(cu_seqlens) - 1
    out = np.zeros((n, cfg.hidden), dtype)
    for b in range(n):
        out[b] = embed_sequence(w, cfg, ids[cu_seqlens[b]:cu_seqlens[b + 1]], dtype)
    return out
