"""Host-side mirror of ripvec's embedding-backend interface over the C ABI.

``Encoding`` and ``EmbedBackend`` keep the names, argument meaning and error behaviour of
``crates/ripvec-core/src/backend/mod.rs:27-94``: ``embed_batch`` takes pre-tokenised encodings
and returns one L2-normalised vector per encoding in input order, errors propagate as exceptions
(never silent defaults), an empty batch returns an empty list, and GPU backends do not support
cloning.  ``load_backend`` plays the role of ``backend::load_backend`` (``mod.rs:152-235``) for
the two architectures of this library.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Iterable, Sequence

import numpy as np

from . import _lib as L
from .synth import ModelSpec


@dataclass
class Encoding:
    """``backend::Encoding``: token ids, attention mask (all 1 for tokenizer output) and type ids."""

    input_ids: Sequence[int]
    attention_mask: Sequence[int] = field(default=None)  # type: ignore[assignment]
    token_type_ids: Sequence[int] = field(default=None)  # type: ignore[assignment]

    def __post_init__(self):
        n = len(self.input_ids)
        if self.attention_mask is None:
            self.attention_mask = [1] * n
        if self.token_type_ids is None:
            self.token_type_ids = [0] * n
        if len(self.attention_mask) != n or len(self.token_type_ids) != n:
            raise ValueError("input_ids, attention_mask and token_type_ids must have equal lengths")


def pack_encodings(encodings: Iterable[Encoding]) -> tuple[np.ndarray, np.ndarray]:
    """Packs encodings into int32 ids + cu_seqlens (only tokens with attention_mask == 1)."""
    ids, cu = [], [0]
    for e in encodings:
        m = np.asarray(e.attention_mask, np.int64)
        t = np.asarray(e.input_ids, np.int64)[m == 1]
        if t.size and (t.min() < np.iinfo(np.int32).min or t.max() > np.iinfo(np.int32).max):
            raise ValueError("token id does not fit in int32")
        ids.append(t.astype(np.int32))
        cu.append(cu[-1] + len(t))
    flat = np.concatenate(ids) if ids else np.zeros(0, np.int32)
    return np.ascontiguousarray(flat, np.int32), np.asarray(cu, np.int32)


class EmbedBackend:
    """GPU embedding backend (``trait EmbedBackend``) on one CUDA device."""

    def __init__(self, spec: ModelSpec, weights: dict | None = None, *, dtype: str = "bf16",
                 device: int = 0, pooling: str | None = None, max_batch_tokens: int = 0,
                 safetensors: str | None = None):
        self._lib = L.lib()
        self.spec = spec
        d = L.ModelDesc()
        d.arch = L.RV_ARCH_MODERNBERT if spec.arch == "modernbert" else L.RV_ARCH_CLASSICBERT
        d.dtype = {"bf16": L.RV_DTYPE_BF16, "f16": L.RV_DTYPE_F16, "fp16": L.RV_DTYPE_F16}[dtype]
        d.hidden, d.num_layers, d.num_heads = spec.hidden, spec.num_layers, spec.num_heads
        d.intermediate, d.vocab, d.max_position = spec.intermediate, spec.vocab, spec.max_position
        d.global_every_n, d.local_window = spec.global_every_n, spec.local_window
        d.global_rope_theta, d.local_rope_theta = spec.global_rope_theta, spec.local_rope_theta
        d.norm_eps, d.type_vocab = spec.norm_eps, spec.type_vocab
        if pooling is None:
            pooling = "mean" if spec.arch == "modernbert" else "cls"
        d.pooling = L.RV_POOL_MEAN if pooling == "mean" else L.RV_POOL_CLS
        d.max_batch_tokens = max_batch_tokens
        h = C.c_void_p()
        rc = self._lib.rv_create(C.byref(d), device, C.byref(h))
        if rc != L.RV_OK:
            raise L.RvError(rc, "rv_create failed (invalid model description or CUDA device)")
        self._h = h
        self.device = device
        if safetensors is not None:
            self._check(self._lib.rv_load_safetensors(self._h, safetensors.encode()))
        if weights is not None:
            for name, arr in weights.items():
                a = np.ascontiguousarray(arr, np.float32)
                self._check(self._lib.rv_set_weight(self._h, name.encode(), a.ctypes.data, a.size))
        self._check(self._lib.rv_finalize(self._h))

    def _check(self, rc: int) -> None:
        if rc != L.RV_OK:
            raise L.RvError(rc, self._lib.rv_last_error(self._h).decode())

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.rv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------------ EmbedBackend
    def embed_batch(self, encodings: Sequence[Encoding]) -> list[list[float]]:
        """L2-normalised embeddings, one per encoding, in input order."""
        if len(encodings) == 0:
            return []
        ids, cu = pack_encodings(encodings)
        return self.embed_packed(ids, cu).tolist()

    def supports_clone(self) -> bool:
        return False

    def clone_backend(self):
        raise RuntimeError("GPU backends do not support clone_backend (supports_clone() is false)")

    def is_gpu(self) -> bool:
        return bool(self._lib.rv_is_gpu(self._h))

    def max_tokens(self) -> int:
        return int(self._lib.rv_max_tokens(self._h))

    def name(self) -> str:
        return self._lib.rv_name(self._h).decode()

    # ------------------------------------------------------------------ packed entry points
    def embed_packed(self, ids: np.ndarray, cu_seqlens: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """``rv_embed_varlen``: host ids / cu_seqlens -> host ``[n, hidden]`` f32."""
        ids = np.ascontiguousarray(ids, np.int32)
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        n = len(cu) - 1
        if out is None:
            out = np.empty((max(n, 0), self.spec.hidden), np.float32)
        self._check(self._lib.rv_embed_varlen(self._h, ids.ctypes.data if ids.size else None,
                                              cu.ctypes.data, n, out.ctypes.data))
        return out

    def embed_device(self, ids_dev, cu_seqlens: np.ndarray, out_dev, out_dtype: int = L.RV_DTYPE_F32,
                     stream: int = 0) -> None:
        """``rv_embed_varlen_device``: ids and output are device tensors (anything with ``data_ptr``)."""
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        self._check(self._lib.rv_embed_varlen_device(self._h, L.ptr(ids_dev), cu.ctypes.data, len(cu) - 1,
                                                     L.ptr(out_dev), out_dtype, stream or None))

    def submit(self, ids: np.ndarray, cu_seqlens: np.ndarray, out: np.ndarray | None = None):
        """``rv_embed_submit``: queues the packed chunks and returns ``(ticket, out)`` at once; ``out``
        ([n, hidden] f32) is filled when ``wait(ticket)`` returns and must be kept until then."""
        ids = np.ascontiguousarray(ids, np.int32)
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        n = len(cu) - 1
        if out is None:
            out = np.empty((max(n, 0), self.spec.hidden), np.float32)
        t = C.c_int64(0)
        self._check(self._lib.rv_embed_submit(self._h, ids.ctypes.data if ids.size else None, cu.ctypes.data, n,
                                              out.ctypes.data, C.byref(t)))
        self._pending = getattr(self, "_pending", {})
        self._pending[t.value] = out  # the library writes into it until the wait
        return t.value, out

    def wait(self, ticket: int) -> None:
        """``rv_embed_wait``: returns when the ticket's embeddings (and every earlier ticket's) are in
        their output arrays."""
        try:
            self._check(self._lib.rv_embed_wait(self._h, ticket))
        finally:
            pend = getattr(self, "_pending", {})
            for t in [t for t in pend if t <= ticket]:
                pend.pop(t)

    def kernel_launches(self) -> int:
        return int(self._lib.rv_kernel_launches(self._h))


def embed_distributed(backends: Sequence[EmbedBackend], ids: np.ndarray, cu_seqlens: np.ndarray,
                      out: np.ndarray | None = None) -> np.ndarray:
    """``embed_distributed`` over several backends (``embed.rs:666-785``) through
    ``rv_embed_varlen_multi``: one host thread per backend, runs of consecutive chunks taken from
    one cursor, results in input order; the first failure is raised."""
    if not backends:
        raise ValueError("no backends")
    ids = np.ascontiguousarray(ids, np.int32)
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    n = len(cu) - 1
    hidden = backends[0].spec.hidden
    if out is None:
        out = np.empty((max(n, 0), hidden), np.float32)
    handles = (C.c_void_p * len(backends))(*[b._h.value for b in backends])
    lib = L.lib()
    rc = lib.rv_embed_varlen_multi(handles, len(backends), ids.ctypes.data if ids.size else None, cu.ctypes.data,
                                   n, out.ctypes.data)
    if rc != L.RV_OK:
        msgs = [lib.rv_last_error(b._h).decode() for b in backends]
        raise L.RvError(rc, "; ".join(m for m in msgs if m) or "rv_embed_varlen_multi failed")
    return out


def load_backend(spec: ModelSpec, weights: dict | None = None, **kw) -> EmbedBackend:
    """``backend::load_backend`` for this library (CUDA only; no CPU fallback)."""
    return EmbedBackend(spec, weights, **kw)
