"""Host-side mirror of ripvec's ``SearchIndex`` over the C ABI (exact cosine top-k on the GPU).

``SearchIndex(embeddings)`` corresponds to ``SearchIndex::new`` (``crates/ripvec-core/src/
index.rs:76-165``) for the embedding matrix, and ``rank(query, threshold)`` to
``SearchIndex::rank`` (``index.rs:172-186``): a query of the wrong dimension or an empty index
gives no results, rows scoring below ``threshold`` are dropped, results are sorted by descending
score.  Differences, by design: rows are stored in bf16 and queries are rounded to bf16, scores
are exact sums of the bf16 products (so equal inputs give bit-identical rankings), and ties are
ordered by row index.  ``rank`` returns every row at or above the threshold, like the
reference; ``topk`` returns the best ``k <= 2048`` rows of a batch of queries.

``rank_turboquant`` mirrors ``SearchIndex::rank_turboquant`` (``index.rs:196-234``) over the
PolarQuant codes of ``turbo_quant.rs``, built on the GPU by ``build_turboquant``.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L

MAX_K = 2048
TURBOQUANT_MIN_CHUNKS = 4096  # index.rs:22
TURBOQUANT_MAX_TOP_K = 800


def turboquant_eligible(n: int, dim: int) -> bool:
    """``SearchIndex::new`` builds the compressed corpus only for at least 4096 rows of an even
    dimension of at least 64 (``index.rs:136-140``)."""
    return n >= TURBOQUANT_MIN_CHUNKS and dim >= 64 and dim % 2 == 0


def polar_rotation(dim: int, seed: int = 42) -> np.ndarray:
    """A seeded orthogonal [dim, dim] f32 rotation: modified Gram-Schmidt over the columns of a
    standard-normal matrix, as ``generate_rotation`` / ``gram_schmidt_qr`` do
    (``turbo_quant.rs:335-367``).  The normal samples come from numpy's generator, so the matrix
    is not the reference's ChaCha8-seeded one; pass that matrix to ``build_turboquant`` to get
    the reference's codes."""
    q = np.random.default_rng(seed).standard_normal((dim, dim)).astype(np.float32)
    for i in range(dim):
        norm = np.float32(np.sqrt(np.sum(q[:, i] * q[:, i], dtype=np.float32)))
        if norm < 1e-10:
            continue
        q[:, i] *= np.float32(1.0) / norm
        if i + 1 < dim:
            q[:, i + 1:] -= (q[:, i][None, :] @ q[:, i + 1:]).astype(np.float32) * q[:, i][:, None]
    return q


class SearchIndex:
    def __init__(self, embeddings, device: int = 0, base: int = 0, turboquant: bool | str = False,
                 turboquant_seed: int = 42, cascade_dim: int | None = None):
        """``turboquant``: ``False`` (default) keeps only the exact index; ``"auto"`` builds the
        PolarQuant corpus when ``SearchIndex::new`` would (``turboquant_eligible``); ``True``
        builds it for any size.  ``cascade_dim``: builds the truncated matrix of the MRL cascade
        (``SearchIndex::new``'s ``cascade_dim``, clamped to the row dimension)."""
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
        if turboquant is True or (turboquant == "auto" and turboquant_eligible(int(n), int(dim))):
            self.build_turboquant(polar_rotation(int(dim), turboquant_seed))
        if cascade_dim is not None:
            self._check(self._lib.rv_index_build_cascade(self._h, cascade_dim))

    def _check(self, rc: int) -> None:
        if rc != L.RV_OK:
            raise L.RvError(rc, self._lib.rv_index_last_error(self._h).decode())

    def __len__(self) -> int:
        return int(self._lib.rv_index_size(self._h))

    def kernel_launches(self) -> int:
        """Kernels launched by this index so far."""
        return int(self._lib.rv_index_kernel_launches(self._h))

    def export_rows(self, row0: int = 0, n: int | None = None, bf16_bits: bool = False) -> np.ndarray:
        """Rows ``[row0, row0 + n)`` as stored on the device (``rv_index_export``): widened to f32
        (exact), or with ``bf16_bits`` the raw bf16 values as uint16."""
        n = len(self) - row0 if n is None else n
        out = np.empty((max(n, 0), self.hidden_dim), np.uint16 if bf16_bits else np.float32)
        dt = L.RV_DTYPE_BF16 if bf16_bits else L.RV_DTYPE_F32
        self._check(self._lib.rv_index_export(self._h, row0, n, dt, out.ctypes.data if out.size else None, 0))
        return out

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

    def kernel_launches(self) -> int:
        """Kernels launched by this index so far."""
        return int(self._lib.rv_index_kernel_launches(self._h))

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

    def rank_arrays(self, query, threshold: float, capacity: int | None = None, with_f64: bool = False):
        """Every row with exact score ``>= threshold`` ordered by (score desc, row asc), as arrays
        ``(idx int64 [m], score f32 [m])`` (plus f64 scores), ``m = min(count, capacity)``; the
        total count is the length when ``capacity`` is None."""
        q = np.ascontiguousarray(query, np.float32).reshape(-1)
        if q.shape[0] != self.hidden_dim:
            raise ValueError(f"query has {q.shape[0]} dimensions, the index {self.hidden_dim}")
        cap = len(self) if capacity is None else max(0, min(int(capacity), len(self)))
        oi = np.empty(max(cap, 1), np.int64)
        os_ = np.empty(max(cap, 1), np.float32)
        o64 = np.empty(max(cap, 1), np.float64) if with_f64 else None
        cnt = C.c_int64(0)
        self._check(self._lib.rv_index_rank(self._h, q.ctypes.data, threshold, cap, oi.ctypes.data,
                                            os_.ctypes.data, o64.ctypes.data if with_f64 else None, C.byref(cnt)))
        m = min(int(cnt.value), cap)
        return (oi[:m], os_[:m], o64[:m]) if with_f64 else (oi[:m], os_[:m])

    def rank(self, query, threshold: float, top_k: int | None = None) -> list[tuple[int, float]]:
        """``SearchIndex::rank``: every ``(row, score)`` pair with score ``>= threshold``, sorted by
        descending score (ties by row); ``top_k`` keeps only the first ``top_k``.  A query of the
        wrong dimension or an empty index gives no results."""
        q = np.asarray(query, np.float32).reshape(-1)
        n = len(self)
        if q.shape[0] != self.hidden_dim or n == 0:
            return []
        if top_k is not None and top_k <= 0:
            return []
        if top_k is not None and top_k <= MAX_K:
            oi, os_, cnt = self.topk(q[None, :], min(top_k, n), threshold)
            return [(int(oi[0, i]), float(os_[0, i])) for i in range(int(cnt[0]))]
        oi, os_ = self.rank_arrays(q, threshold, top_k)
        return list(zip(oi.tolist(), os_.astype(np.float64).tolist()))

    # ------------------------------------------------------------ PolarQuant ("TurboQuant")
    def build_turboquant(self, rotation: np.ndarray, bits: int = 4) -> None:
        """``PolarCodec::new`` + ``encode_batch`` of the stored rows under ``rotation``."""
        r = np.ascontiguousarray(rotation, np.float32)
        if r.shape != (self.hidden_dim, self.hidden_dim):
            raise ValueError(f"rotation must be [{self.hidden_dim}, {self.hidden_dim}]")
        self._check(self._lib.rv_index_build_polar(self._h, r.ctypes.data, bits))

    @property
    def has_turboquant(self) -> bool:
        return bool(self._lib.rv_index_has_polar(self._h))

    def turboquant_codes(self) -> tuple[np.ndarray, np.ndarray]:
        """The compressed corpus as ``(radii f32 [n, dim/2], bins u8 [n, dim/2])``."""
        n, pairs = len(self), self.hidden_dim // 2
        radii = np.empty((n, pairs), np.float32)
        bins = np.empty((n, pairs), np.uint8)
        self._check(self._lib.rv_index_polar_export(self._h, radii.ctypes.data, bins.ctypes.data))
        return radii, bins

    def turboquant_scores(self, queries) -> np.ndarray:
        """``scan_corpus`` of each query: approximate scores ``[nq, n]`` f32."""
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.hidden_dim)
        out = np.empty((q.shape[0], len(self)), np.float32)
        self._check(self._lib.rv_index_polar_scores(self._h, q.ctypes.data, q.shape[0], out.ctypes.data))
        return out

    def topk_turboquant(self, queries, top_k: int, threshold: float = float("-inf"), with_f64: bool = False):
        """``rank_turboquant`` for a batch of queries, as arrays like ``topk``."""
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.hidden_dim)
        nq = q.shape[0]
        oi = np.empty((nq, top_k), np.int64)
        os_ = np.empty((nq, top_k), np.float32)
        o64 = np.empty((nq, top_k), np.float64) if with_f64 else None
        cnt = np.empty(nq, np.int32)
        self._check(self._lib.rv_index_rank_turboquant(self._h, q.ctypes.data, nq, top_k, threshold, oi.ctypes.data,
                                                       os_.ctypes.data, o64.ctypes.data if with_f64 else None,
                                                       cnt.ctypes.data))
        return (oi, os_, cnt, o64) if with_f64 else (oi, os_, cnt)

    def topk_turboquant_device(self, queries_dev, top_k: int, out_idx, out_score, out_score64=None,
                               threshold: float = float("-inf"), stream: int = 0) -> None:
        nq = queries_dev.shape[0]
        self._check(self._lib.rv_index_rank_turboquant_device(self._h, L.ptr(queries_dev), nq, top_k, threshold,
                                                              L.ptr(out_idx), L.ptr(out_score),
                                                              L.ptr(out_score64), stream or None))

    def rank_turboquant(self, query, top_k: int, threshold: float) -> list[tuple[int, float]]:
        """``SearchIndex::rank_turboquant`` (``index.rs:196-234``): ``(row, score)`` pairs, at
        most ``top_k``, sorted by descending exact score.  A query of the wrong dimension is an
        error (the reference's ``prepare_query`` asserts the length)."""
        q = np.asarray(query, np.float32).reshape(-1)
        if q.shape[0] != self.hidden_dim:
            raise ValueError(f"query has {q.shape[0]} dimensions, the index {self.hidden_dim}")
        n = len(self)
        if n == 0 or top_k <= 0:
            return []
        oi, os_, cnt = self.topk_turboquant(q[None, :], min(top_k, TURBOQUANT_MAX_TOP_K), threshold)
        return [(int(oi[0, i]), float(os_[0, i])) for i in range(int(cnt[0]))]


    # ------------------------------------------------------------ MRL cascade
    def truncated_dim(self) -> int | None:
        """``SearchIndex::truncated_dim``."""
        t = int(self._lib.rv_index_cascade_dim(self._h))
        return t or None

    def truncated_rows(self) -> np.ndarray:
        """The truncated, re-normalised matrix ``[n, truncated_dim]`` (bf16 values as f32)."""
        out = np.empty((len(self), self.truncated_dim() or 0), np.float32)
        self._check(self._lib.rv_index_cascade_rows(self._h, out.ctypes.data))
        return out

    def topk_cascade(self, queries, top_k: int, threshold: float = float("-inf"), with_f64: bool = False):
        """``rank_cascade`` for a batch of queries, as arrays like ``topk``."""
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.hidden_dim)
        nq = q.shape[0]
        oi = np.empty((nq, top_k), np.int64)
        os_ = np.empty((nq, top_k), np.float32)
        o64 = np.empty((nq, top_k), np.float64) if with_f64 else None
        cnt = np.empty(nq, np.int32)
        self._check(self._lib.rv_index_rank_cascade(self._h, q.ctypes.data, nq, top_k, threshold, oi.ctypes.data,
                                                    os_.ctypes.data, o64.ctypes.data if with_f64 else None,
                                                    cnt.ctypes.data))
        return (oi, os_, cnt, o64) if with_f64 else (oi, os_, cnt)

    def rank_cascade(self, query, top_k: int, threshold: float) -> list[tuple[int, float]]:
        """``SearchIndex::rank_cascade`` (``index.rs:245-297``): a query of the wrong dimension or
        an empty index gives no results."""
        q = np.asarray(query, np.float32).reshape(-1)
        if q.shape[0] != self.hidden_dim or len(self) == 0 or top_k <= 0:
            return []
        oi, os_, cnt = self.topk_cascade(q[None, :], top_k, threshold)
        return [(int(oi[0, i]), float(os_[0, i])) for i in range(int(cnt[0]))]


    # ------------------------------------------------------------ near-duplicate pairs
    def duplicate_pairs(self, threshold: float, max_pairs: int):
        """``find_duplicates`` as arrays: ``(a int64 [m], b int64 [m], score f32 [m], score f64 [m])``."""
        mp = max(int(max_pairs), 0)
        a = np.empty(max(mp, 1), np.int64)
        b = np.empty(max(mp, 1), np.int64)
        s = np.empty(max(mp, 1), np.float32)
        s64 = np.empty(max(mp, 1), np.float64)
        cnt = C.c_int64(0)
        self._check(self._lib.rv_index_find_duplicates(self._h, threshold, mp, a.ctypes.data, b.ctypes.data,
                                                       s.ctypes.data, s64.ctypes.data, C.byref(cnt)))
        m = int(cnt.value)
        return a[:m], b[:m], s[:m], s64[:m]

    def find_duplicates(self, threshold: float, max_pairs: int) -> list[tuple[int, int, float]]:
        """``SearchIndex::find_duplicates`` (``index.rs:325-348``): ``(a, b, similarity)`` with
        a < b and similarity >= threshold, sorted by descending similarity, at most ``max_pairs``."""
        a, b, s, _ = self.duplicate_pairs(threshold, max_pairs)
        return [(int(x), int(y), float(z)) for x, y, z in zip(a, b, s)]


class ShardComm:
    """NCCL communicator of a row-sharded search (``rv_comm_*``): rank ``rank`` of ``world`` on
    CUDA device ``device``.  ``unique_id`` (``RV_COMM_ID_BYTES`` bytes from ``new_unique_id`` on
    rank 0) reaches every rank through the caller's own channel.  Every wait gives up after
    ``timeout_ms`` with an error instead of hanging."""

    def __init__(self, unique_id: bytes, rank: int, world: int, device: int = 0, timeout_ms: int = 60000):
        self._lib = L.lib()
        if len(unique_id) != L.RV_COMM_ID_BYTES:
            raise ValueError(f"unique id must be {L.RV_COMM_ID_BYTES} bytes")
        buf = (C.c_uint8 * L.RV_COMM_ID_BYTES).from_buffer_copy(unique_id)
        h = C.c_void_p()
        rc = self._lib.rv_comm_create(device, buf, rank, world, timeout_ms, C.byref(h))
        if rc != L.RV_OK:
            raise L.RvError(rc, "rv_comm_create failed (NCCL missing, bad id, or a rank did not join in time)")
        self._h = h
        self.rank, self.world, self.device = rank, world, device

    @staticmethod
    def new_unique_id() -> bytes:
        buf = (C.c_uint8 * L.RV_COMM_ID_BYTES)()
        rc = L.lib().rv_comm_get_unique_id(buf)
        if rc != L.RV_OK:
            raise L.RvError(rc, "rv_comm_get_unique_id failed (NCCL could not be loaded)")
        return bytes(buf)

    def last_error(self) -> str:
        return self._lib.rv_comm_last_error(self._h).decode()

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.rv_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def topk_sharded(index: "SearchIndex", comm: ShardComm, queries_dev, k: int, out_idx, out_score,
                 out_score64=None, threshold: float = float("-inf"), stream: int = 0) -> None:
    """``rv_index_topk_sharded``: the global top ``k`` over every rank's shard (same queries on
    every rank, same results on every rank; device tensors)."""
    nq = queries_dev.shape[0]
    rc = L.lib().rv_index_topk_sharded(index._h, comm._h, L.ptr(queries_dev), nq, k, threshold, L.ptr(out_idx),
                                       L.ptr(out_score), L.ptr(out_score64), stream or None)
    if rc != L.RV_OK:
        raise L.RvError(rc, index._lib.rv_index_last_error(index._h).decode())


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
