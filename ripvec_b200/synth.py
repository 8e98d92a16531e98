"""Seeded synthetic inputs and random-init weights for the benchmark configurations.

There is no network for checkpoints or corpora, so every run uses weights drawn from N(0, 0.02)
(LayerNorm gains 1, LayerNorm biases 0) and token ids drawn uniformly over the vocabulary, with
the chunk-length distributions of the benchmark configurations.  All draws come from
``numpy.random.default_rng(seed)`` in a fixed order, so the GPU run and the CPU oracle see the
same numbers.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import numpy as np


@dataclass(frozen=True)
class ModelSpec:
    arch: str  # "modernbert" | "classicbert"
    hidden: int
    num_layers: int
    num_heads: int
    intermediate: int
    vocab: int
    max_position: int
    global_every_n: int = 3
    local_window: int = 128
    global_rope_theta: float = 160000.0
    local_rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    type_vocab: int = 2

    def as_dict(self) -> dict:
        return asdict(self)


MODERNBERT_BASE = ModelSpec("modernbert", 768, 22, 12, 1152, 50368, 8192)
BERT_SMALL = ModelSpec("classicbert", 384, 12, 12, 1536, 30522, 512, norm_eps=1e-12)


def modernbert_weight_shapes(s: ModelSpec) -> list[tuple[str, tuple[int, ...]]]:
    H, I = s.hidden, s.intermediate
    out = [("embeddings.tok_embeddings.weight", (s.vocab, H)), ("embeddings.norm.weight", (H,)),
           ("final_norm.weight", (H,))]
    for i in range(s.num_layers):
        p = f"layers.{i}."
        out += [(p + "attn.Wqkv.weight", (3 * H, H)), (p + "attn.Wo.weight", (H, H))]
        if i > 0:
            out.append((p + "attn_norm.weight", (H,)))
        out += [(p + "mlp.Wi.weight", (2 * I, H)), (p + "mlp.Wo.weight", (H, I)), (p + "mlp_norm.weight", (H,))]
    return out


def classicbert_weight_shapes(s: ModelSpec) -> list[tuple[str, tuple[int, ...]]]:
    H, I = s.hidden, s.intermediate
    out = [("embeddings.word_embeddings.weight", (s.vocab, H)),
           ("embeddings.position_embeddings.weight", (s.max_position, H)),
           ("embeddings.token_type_embeddings.weight", (s.type_vocab, H)),
           ("embeddings.LayerNorm.weight", (H,)), ("embeddings.LayerNorm.bias", (H,))]
    for i in range(s.num_layers):
        p = f"encoder.layer.{i}."
        for m in ("query", "key", "value"):
            out += [(p + f"attention.self.{m}.weight", (H, H)), (p + f"attention.self.{m}.bias", (H,))]
        out += [(p + "attention.output.dense.weight", (H, H)), (p + "attention.output.dense.bias", (H,)),
                (p + "attention.output.LayerNorm.weight", (H,)), (p + "attention.output.LayerNorm.bias", (H,)),
                (p + "intermediate.dense.weight", (I, H)), (p + "intermediate.dense.bias", (I,)),
                (p + "output.dense.weight", (H, I)), (p + "output.dense.bias", (H,)),
                (p + "output.LayerNorm.weight", (H,)), (p + "output.LayerNorm.bias", (H,))]
    return out


def random_weights(spec: ModelSpec, seed: int, std: float = 0.02, qk_std: float | None = None) -> dict:
    """Random-init weights: matrices, embedding tables and dense biases ~ N(0, std); LayerNorm
    gains = 1 and LayerNorm biases = 0.  ``qk_std`` (stress variant) redraws the query / key
    projection rows with a larger spread so attention is far from uniform."""
    rng = np.random.default_rng(seed)
    shapes = modernbert_weight_shapes(spec) if spec.arch == "modernbert" else classicbert_weight_shapes(spec)
    w = {}
    for name, shape in shapes:
        if "norm" in name.lower() and name.endswith(".weight") and len(shape) == 1:
            w[name] = np.ones(shape, np.float32)
        elif "LayerNorm.bias" in name:
            w[name] = np.zeros(shape, np.float32)
        else:
            w[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
    if qk_std is not None:
        H = spec.hidden
        for name in list(w):
            if name.endswith("attn.Wqkv.weight"):
                w[name][: 2 * H] = rng.standard_normal((2 * H, H), dtype=np.float32) * np.float32(qk_std)
            if name.endswith("attention.self.query.weight") or name.endswith("attention.self.key.weight"):
                w[name][:] = rng.standard_normal(w[name].shape, dtype=np.float32) * np.float32(qk_std)
    return w


def uniform_lengths(n: int, lo: int, hi: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n).astype(np.int32)


def lognormal_lengths(n: int, median: float, sigma: float, lo: int, hi: int, seed: int) -> np.ndarray:
    """``clip(round(exp(N(ln median, sigma^2))), lo, hi)``."""
    r = np.random.default_rng(seed).normal(np.log(median), sigma, size=n)
    return np.clip(np.rint(np.exp(r)), lo, hi).astype(np.int32)


def packed_ids(lengths: np.ndarray, vocab: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Token ids uniform over the vocabulary, packed; returns ``(ids int32 [T], cu_seqlens int32 [n+1])``."""
    cu = np.zeros(len(lengths) + 1, np.int64)
    np.cumsum(lengths, out=cu[1:])
    ids = np.random.default_rng(seed).integers(0, vocab, size=int(cu[-1])).astype(np.int32)
    return ids, cu.astype(np.int32)


def normalized_gaussian(n: int, dim: int, seed: int, chunk: int = 1 << 20) -> np.ndarray:
    """Gaussian rows L2-normalised in f32 (the search database / query distribution)."""
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        x = rng.standard_normal((e - s, dim), dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        out[s:e] = x
    return out
