"""Test fixtures: per-file cache objects laid out as ``FileCache::to_bytes`` writes them
(``crates/ripvec-core/src/cache/file_cache.rs:43-49``), built here without the Rust crates.

An rkyv 0.8 archive with the crate's default format (little-endian, 32-bit relative pointers and
lengths) puts every out-of-line object first and the 20-byte root last:
``chunks {i32 offset, u32 len}, embeddings {i32 offset, u32 len}, hidden_dim u32``, each offset
relative to the position of its own pointer field.  The chunk records are written as opaque
48-byte entries followed by their strings: the reader under test only uses the chunk count, the
embeddings and hidden_dim.  These bytes follow that layout; they are not a byte-for-byte copy of
what rkyv writes for ``CodeChunk``, and no object written by the reference was available to
compare against.

zstd frames come from the system's libzstd (public API): ``zstd_frame`` with the content size in
the header (``ZSTD_compress``) and ``zstd_stream`` without it, as the streaming encoder behind
``zstd::encode_all`` writes them.
"""

import ctypes as C
import struct

import numpy as np

_Z = None


def _zstd():
    global _Z
    if _Z is None:
        z = C.CDLL("libzstd.so.1")
        z.ZSTD_compressBound.restype = C.c_size_t
        z.ZSTD_compressBound.argtypes = [C.c_size_t]
        z.ZSTD_compress.restype = C.c_size_t
        z.ZSTD_compress.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_int]
        z.ZSTD_isError.restype = C.c_uint
        z.ZSTD_isError.argtypes = [C.c_size_t]
        z.ZSTD_createCStream.restype = C.c_void_p
        z.ZSTD_freeCStream.argtypes = [C.c_void_p]
        z.ZSTD_initCStream.restype = C.c_size_t
        z.ZSTD_initCStream.argtypes = [C.c_void_p, C.c_int]
        z.ZSTD_compressStream.restype = C.c_size_t
        z.ZSTD_compressStream.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        z.ZSTD_endStream.restype = C.c_size_t
        z.ZSTD_endStream.argtypes = [C.c_void_p, C.c_void_p]
        _Z = z
    return _Z


def zstd_frame(data: bytes, level: int = 1) -> bytes:
    z = _zstd()
    cap = z.ZSTD_compressBound(len(data))
    out = C.create_string_buffer(cap)
    src = C.create_string_buffer(data, len(data))
    n = z.ZSTD_compress(out, cap, src, len(data), level)
    assert not z.ZSTD_isError(n)
    return out.raw[:n]


class _In(C.Structure):
    _fields_ = [("src", C.c_void_p), ("size", C.c_size_t), ("pos", C.c_size_t)]


class _Out(C.Structure):
    _fields_ = [("dst", C.c_void_p), ("size", C.c_size_t), ("pos", C.c_size_t)]


def zstd_stream(data: bytes, level: int = 1) -> bytes:
    """One frame from the streaming encoder (no content size in the frame header)."""
    z = _zstd()
    cs = z.ZSTD_createCStream()
    assert not z.ZSTD_isError(z.ZSTD_initCStream(cs, level))
    src = C.create_string_buffer(data, len(data))
    cap = z.ZSTD_compressBound(len(data)) + 1024
    dst = C.create_string_buffer(cap)
    inb = _In(C.cast(src, C.c_void_p), len(data), 0)
    outb = _Out(C.cast(dst, C.c_void_p), cap, 0)
    while inb.pos < inb.size:
        assert not z.ZSTD_isError(z.ZSTD_compressStream(cs, C.byref(outb), C.byref(inb)))
    while True:
        left = z.ZSTD_endStream(cs, C.byref(outb))
        assert not z.ZSTD_isError(left)
        if left == 0:
            break
    z.ZSTD_freeCStream(cs)
    return dst.raw[:outb.pos]


def _pad4(b: bytearray) -> None:
    b.extend(b"\0" * (-len(b) % 4))


def archive(chunk_names: list[str], embeddings: np.ndarray, hidden_dim: int,
            n_floats: int | None = None) -> bytes:
    """The bare archive of ``FileCache { chunks, embeddings, hidden_dim }`` (one chunk per name).
    ``n_floats`` overrides the stored embeddings length (for malformed cases)."""
    emb = np.ascontiguousarray(embeddings, np.float32).reshape(-1)
    b = bytearray()
    for name in chunk_names:  # out-of-line strings first, like rkyv's depth-first writer
        b.extend(name.encode())
    _pad4(b)
    chunks_at = len(b)
    for i, name in enumerate(chunk_names):
        b.extend(struct.pack("<IIII", i, len(name), 1, 10) + b"\0" * 32)  # opaque 48-byte record
    _pad4(b)
    emb_at = len(b)
    b.extend(emb.astype("<f4").tobytes())
    _pad4(b)
    root = len(b)
    nf = emb.size if n_floats is None else n_floats
    b.extend(struct.pack("<iI", chunks_at - root, len(chunk_names)))
    b.extend(struct.pack("<iI", emb_at - (root + 8), nf))
    b.extend(struct.pack("<I", hidden_dim))
    return bytes(b)


def file_cache(chunk_names, embeddings, hidden_dim, stream: bool = True, **kw) -> bytes:
    """``FileCache::to_bytes``: zstd level 1 around the archive."""
    raw = archive(chunk_names, embeddings, hidden_dim, **kw)
    return zstd_stream(raw) if stream else zstd_frame(raw)
