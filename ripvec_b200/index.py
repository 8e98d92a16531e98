"""Host-side mirror of ripvec's ``SearchIndex`` over the C ABI (exact cosine top-k on the GPU).

``SearchIndex(embeddings)`` corresponds to ``SearchIndex::new`` (``crates/ripvec-core/src/
index.rs:76-165``) for the embedding matrix, and ``rank(query, threshold)`` to
``SearchIndex::rank`` (``index.rs:172-186``): a query of the wrong dimension or an empty index
gives no results, rows scoring below ``threshold`` are dropped, results are sorted by descending
score.  Differences, by design: rows are stored in bf16 and queries are rounded to bf16, scores
are exact sums of the bf16 products (so equal inputs give bit-identical rankings), ties are
ordered by row index, and one call returns at most 2048 rows per query (``top_k``).
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L

MAX_K = 2048


class SearchIndex:
    def __init__(self, embeddings, device: int = 0, base: int = 0):
        self._lib = L.lib()
        h = C.c_void_p()
        if hasattr(embeddings, "data_ptr"):  # device tensor (torch): f32 or bf16
            import torch

            t = embeddings.contiguous()
            dt = {torch.float32: L.RV_DTYPE_F32, torch.bfloat16: L.RV_DTYPE_BF16}[t.dtype]
            n, dim = t.shape
            rc = self._lib.rv_index_create(device, t.data_ptr(), n, dim, dt, 1, C.byref(h))
        else:
            e = np.ascontiguousarray(embeddings, np.float32)
            if e.ndim != 2:
                e = e.reshape(0, 384) if e.size == 0 else e
            n, dim = e.shape
            rc = self._lib.rv_index_create(device, e.ctypes.data if e.size else None, n, dim,
                                           L.RV_DTYPE_F32, 0, C.byref(h))
        if rc != L.RV_OK:
            raise L.RvError(rc, "rv_index_create failed (dimension must be a multiple of 64)")
        self._h = h
        self.hidden_dim = int(dim)
        self.device = device
        if base:
            self._check(self._lib.rv_index_set_base(self._h, base))

    def _check(self, rc: int) -> None:
        if rc != L.RV_OK:
            raise L.RvError(rc, self._lib.rv_index_last_error(self._h).decode())

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.rv_index_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return int(self._lib.rv_index_size(self._h))

    def is_empty(self) -> bool:
        return len(self) == 0

    def topk(self, queries, k: int, threshold: float = float("-inf"), with_f64: bool = False):
        """Best ``k`` rows per query: ``(idx int64 [nq,k], score f32 [nq,k], count int32 [nq])``
        (plus the f64 scores when ``with_f64``); missing entries are ``-1`` / ``-inf``."""
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.hidden_dim)
        nq = q.shape[0]
        oi = np.empty((nq, k), np.int64)
        os_ = np.empty((nq, k), np.float32)
        o64 = np.empty((nq, k), np.float64) if with_f64 else None
        cnt = np.empty(nq, np.int32)
        self._check(self._lib.rv_index_topk(self._h, q.ctypes.data, nq, k, threshold, oi.ctypes.data,
                                            os_.ctypes.data, o64.ctypes.data if with_f64 else None,
                                            cnt.ctypes.data))
        return (oi, os_, cnt, o64) if with_f64 else (oi, os_, cnt)

    def topk_device(self, queries_dev, k: int, out_idx, out_score, out_score64=None,
                    threshold: float = float("-inf"), stream: int = 0) -> None:
        nq = queries_dev.shape[0]
        self._check(self._lib.rv_index_topk_device(self._h, L.ptr(queries_dev), nq, k, threshold,
                                                   L.ptr(out_idx), L.ptr(out_score), L.ptr(out_score64),
                                                   stream or None))

    def rank(self, query, threshold: float, top_k: int | None = None) -> list[tuple[int, float]]:
        """``SearchIndex::rank``: ``(row, score)`` pairs sorted by descending score, ``>= threshold``."""
        q = np.asarray(query, np.float32).reshape(-1)
        n = len(self)
        if q.shape[0] != self.hidden_dim or n == 0:
            return []
        k = min(n, MAX_K) if top_k is None else min(top_k, n, MAX_K)
        if k <= 0:
            return []
        oi, os_, cnt = self.topk(q[None, :], k, threshold)
        return [(int(oi[0, i]), float(os_[0, i])) for i in range(int(cnt[0]))]


def merge_topk_device(idx_lists, score64_lists, k: int, threshold: float = float("-inf"), device: int = 0,
                      stream: int = 0):
    """Merges per-shard device results ``[n_lists, nq, k]`` (int64 idx, f64 scores) on the GPU;
    returns ``(idx, score f32, score f64)`` device tensors ``[nq, k]``."""
    import torch

    n_lists, nq, kk = idx_lists.shape
    oi = torch.empty((nq, k), dtype=torch.int64, device=idx_lists.device)
    os_ = torch.empty((nq, k), dtype=torch.float32, device=idx_lists.device)
    o64 = torch.empty((nq, k), dtype=torch.float64, device=idx_lists.device)
    rc = L.lib().rv_topk_merge_device(device, idx_lists.data_ptr(), score64_lists.data_ptr(), n_lists, nq, kk,
                                      threshold, oi.data_ptr(), os_.data_ptr(), o64.data_ptr(), stream or None)
    if rc != L.RV_OK:
        raise L.RvError(rc, "rv_topk_merge_device failed")
    return oi[:, :k], os_[:, :k], o64[:, :k]
