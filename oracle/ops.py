"""Op-level restatement of the reference CPU driver (``crates/ripvec-core/src/backend/driver/cpu.rs``).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Every function takes numpy arrays and
computes in the arrays' dtype (float32 to follow the reference, float64 for the cross-check).
"""

from __future__ import annotations

import ctypes
import ctypes.util
import functools

import numpy as np


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None, eps: float) -> np.ndarray:
    """Row-wise LayerNorm: mean, biased variance, ``1/sqrt(var+eps)``, ``*weight + bias``.

    Follows ``driver/cpu.rs:892-916`` (and ``backend/cpu.rs:166-176`` for ClassicBert).
    """
    dt = x.dtype
    n = dt.type(x.shape[-1])
    mean = x.sum(axis=-1, keepdims=True, dtype=dt) / n
    d = x - mean
    var = (d * d).sum(axis=-1, keepdims=True, dtype=dt) / n
    inv_std = dt.type(1.0) / np.sqrt(var + dt.type(eps))
    out = d * inv_std * weight.astype(dt)
    if bias is not None:
        out = out + bias.astype(dt)
    return out


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """tanh-approximation GELU, ``x*0.5*(1+tanh(sqrt(2/pi)*(x+0.044715 x^3)))`` (``driver/cpu.rs:697-699``)."""
    dt = x.dtype.type
    k = dt(np.sqrt(2.0 / np.pi))
    return x * dt(0.5) * (dt(1.0) + np.tanh(k * (x + dt(0.044715) * x * x * x)))


def softmax_rows(s: np.ndarray) -> np.ndarray:
    """Max-subtracted softmax along the last axis, ``exp(v-max) * (1/sum)`` (``driver/cpu.rs:704-715``)."""
    dt = s.dtype.type
    e = np.exp(s - s.max(axis=-1, keepdims=True))
    return e * (dt(1.0) / e.sum(axis=-1, keepdims=True))


def gemm_bt(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """``a @ b^T`` — the reference ``Driver::gemm`` with ``transpose_b = true`` (``driver/cpu.rs:922-957``)."""
    return a @ b.T


def gemm(a: np.ndarray, b: np.ndarray, transpose_b: bool) -> np.ndarray:
    """``Driver::gemm`` with either orientation of B (``driver/cpu.rs:922-957``)."""
    return a @ (b.T if transpose_b else b)


@functools.lru_cache(maxsize=1)
def _libm():
    lib = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
    for name in ("powf", "cosf", "sinf"):
        f = getattr(lib, name)
        f.restype = ctypes.c_float
        f.argtypes = [ctypes.c_float] * (2 if name == "powf" else 1)
    return lib


@functools.lru_cache(maxsize=8)
def rope_tables(head_dim: int, max_seq: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """RoPE cos/sin tables ``[max_seq, head_dim/2]`` built in f32 with libm like the reference.

    ``freq = (pos as f32) / theta.powf(2d/head_dim)``; ``cos/sin`` in f32
    (``driver/cpu.rs:670-688``).  The libm single-precision functions are called directly so
    that the table matches the one the reference computes on Linux bit for bit.
    """
    m = _libm()
    half = head_dim // 2
    th = float(np.float32(theta))
    denom = [m.powf(th, float(np.float32(2.0 * d) / np.float32(head_dim))) for d in range(half)]
    cos = np.empty((max_seq, half), np.float32)
    sin = np.empty((max_seq, half), np.float32)
    for p in range(max_seq):
        pf = np.float32(p)
        for d in range(half):
            f = float(pf / np.float32(denom[d]))
            cos[p, d] = m.cosf(f)
            sin[p, d] = m.sinf(f)
    return cos, sin


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE on ``x[L, heads, head_dim]`` with position = row index (``driver/cpu.rs:1155-1186``)."""
    half = x.shape[-1] // 2
    L = x.shape[0]
    c = cos[:L, None, :].astype(x.dtype)
    s = sin[:L, None, :].astype(x.dtype)
    first, second = x[..., :half], x[..., half:]
    return np.concatenate([first * c - second * s, first * s + second * c], axis=-1)


def mean_pool(h: np.ndarray) -> np.ndarray:
    """Mean over the sequence with ``sum * (1/len)`` (``driver/cpu.rs:1366-1390``); zero for an empty sequence."""
    if h.shape[0] == 0:
        return np.zeros(h.shape[1], h.dtype)
    return h.sum(axis=0, dtype=h.dtype) * (h.dtype.type(1.0) / h.dtype.type(h.shape[0]))


def l2_normalize(v: np.ndarray) -> np.ndarray:
    """``v * (1/norm)`` when ``norm > 0`` else zeros (``driver/cpu.rs:1392-1403``)."""
    n = np.sqrt((v * v).sum(dtype=v.dtype))
    return v * (v.dtype.type(1.0) / n) if n > 0 else np.zeros_like(v)


def l2_normalize_floor(v: np.ndarray, floor: float = 1e-12) -> np.ndarray:
    """``v / max(norm, 1e-12)`` — the ClassicBert backend's normalisation (``backend/cpu.rs:740-743``)."""
    n = max(np.sqrt((v * v).sum(dtype=v.dtype)), v.dtype.type(floor))
    return v / n


def embedding_lookup(ids: np.ndarray, table: np.ndarray) -> np.ndarray:
    """Row gather ``table[ids]`` (``driver/cpu.rs:855-871``)."""
    return table[np.asarray(ids, dtype=np.int64)]


def cls_pool(hidden: np.ndarray, batch: int, seq: int) -> np.ndarray:
    """First row of each ``[seq, hidden]`` block of a padded batch (``driver/cpu.rs:1346-1364``)."""
    return hidden.reshape(batch, seq, -1)[:, 0, :].copy()


def to_bf16(x: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 (nearest even) and return the values as f32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, r)
    return (r.astype(np.uint32) << 16).view(np.float32).reshape(np.shape(x))


def to_f16(x: np.ndarray) -> np.ndarray:
    """Round f32 to IEEE half (nearest even) and return the values as f32."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
