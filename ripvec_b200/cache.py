"""Embedding store: the reference's per-file cache objects into a search index, and device index
shards out to a file and back.

* ``decode_file_cache(obj)``: the embeddings of one object written by ``FileCache::to_bytes``
  (``crates/ripvec-core/src/cache/file_cache.rs:43-70``: zstd around an rkyv 0.8 archive, or the
  bare archive), through ``rv_cache_decode``.  Objects in the portable bitcode form are refused.
* ``load_file_caches(objs)``: ``load_all_from_store`` (``cache/reindex.rs:537-603``): every
  object's rows in the given order, one row per chunk whose whole embedding slice exists; corrupt
  or unsupported objects are skipped and reported, so the caller re-embeds those files.
* ``save_shard`` / ``load_shard``: a device index shard as a file (a 32-byte header, then the
  bf16 rows as stored on the device) and back, bit for bit.
"""

from __future__ import annotations

import ctypes as C
import os
import struct
from typing import Iterable

import numpy as np

from . import _lib as L

SHARD_MAGIC = b"RVSHARD1"
_HEADER = struct.Struct("<8sQIIQ")  # magic, rows, dim, dtype code (bf16), base


def decode_file_cache(obj: bytes) -> np.ndarray:
    """The ``[rows, hidden_dim]`` f32 embeddings of one cache object; raises ``RvError`` (code
    ``RV_E_IO``) for malformed or portable-form objects."""
    lib = L.lib()
    buf = (C.c_uint8 * len(obj)).from_buffer_copy(obj) if obj else None
    rows, dim = C.c_int64(), C.c_int32()
    rc = lib.rv_cache_decode(buf, len(obj), None, 0, C.byref(rows), C.byref(dim))
    if rc != L.RV_OK:
        raise L.RvError(rc, lib.rv_cache_last_error().decode())
    out = np.empty((rows.value, dim.value), np.float32)
    rc = lib.rv_cache_decode(buf, len(obj), out.ctypes.data if out.size else None, out.size, C.byref(rows),
                             C.byref(dim))
    if rc != L.RV_OK:
        raise L.RvError(rc, lib.rv_cache_last_error().decode())
    return out


def load_file_caches(objs: Iterable[bytes]) -> tuple[np.ndarray, list[int], list[int]]:
    """All objects' rows concatenated in order.  Returns ``(embeddings [n, dim] f32, rows per
    object, indices of the skipped objects)``; an object whose hidden_dim differs from the first
    readable one is skipped too."""
    parts, counts, skipped, dim = [], [], [], None
    for i, obj in enumerate(objs):
        try:
            e = decode_file_cache(obj)
        except L.RvError:
            skipped.append(i)
            counts.append(0)
            continue
        if dim is None:
            dim = e.shape[1]
        if e.shape[1] != dim:
            skipped.append(i)
            counts.append(0)
            continue
        parts.append(e)
        counts.append(e.shape[0])
    emb = np.concatenate(parts) if parts else np.zeros((0, dim or 0), np.float32)
    return emb, counts, skipped


def save_shard(index, path: str | os.PathLike, base: int = 0) -> None:
    """Writes every row of ``index`` (a ``SearchIndex``) as stored (bf16) after a header."""
    rows = index.export_rows(bf16_bits=True)
    with open(path, "wb") as f:
        f.write(_HEADER.pack(SHARD_MAGIC, rows.shape[0], index.hidden_dim, L.RV_DTYPE_BF16, base))
        f.write(rows.tobytes())


def read_shard(path: str | os.PathLike) -> tuple[np.ndarray, int]:
    """``(rows [n, dim] f32, base)`` of a shard file; the bf16 values widen exactly."""
    with open(path, "rb") as f:
        head = f.read(_HEADER.size)
        if len(head) != _HEADER.size:
            raise ValueError(f"{path}: not a shard file (short header)")
        magic, n, dim, dt, base = _HEADER.unpack(head)
        if magic != SHARD_MAGIC or dt != L.RV_DTYPE_BF16 or dim == 0:
            raise ValueError(f"{path}: not a bf16 shard file")
        raw = np.frombuffer(f.read(n * dim * 2), np.uint16)
    if raw.size != n * dim:
        raise ValueError(f"{path}: truncated ({raw.size} of {n * dim} values)")
    rows = (raw.astype(np.uint32) << 16).view(np.float32).reshape(n, dim)
    return rows, int(base)


def load_shard(path: str | os.PathLike, device: int = 0):
    """A ``SearchIndex`` on ``device`` holding the shard's rows (bit-identical to the saved ones)."""
    from .index import SearchIndex

    rows, base = read_shard(path)
    return SearchIndex(rows, device=device, base=base)
