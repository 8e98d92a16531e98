"""ClassicBert (BERT / BGE) encoder forward — numpy restatement of ``backend/cpu.rs``.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Per sequence (``backend/cpu.rs:722-748``): word + learned position + token-type embeddings then
LayerNorm with bias (:232-272); per layer post-LN attention with biases, scores scaled by
``1/sqrt(head_dim)`` plus the additive mask (all real tokens here), softmax, ``P V``, output
projection + bias, residual, LayerNorm (:318-394); FFN ``Linear -> tanh-GELU -> Linear``,
residual, LayerNorm (:426-462).  Pooling: the reference pools the first (CLS) token and divides
by ``max(norm, 1e-12)`` (:736-745); the benchmark configuration asks for mean pooling, which is
offered as ``pooling="mean"`` with the same normalisation.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import ops


@dataclass(frozen=True)
class ClassicBertConfig:
    """Mirrors ``BertConfig`` (``backend/cpu.rs:52-92``) plus the sizes the loader reads."""

    hidden: int = 384
    num_layers: int = 12
    num_heads: int = 12
    intermediate: int = 1536
    vocab: int = 30522
    max_position: int = 512
    type_vocab: int = 2
    norm_eps: float = 1e-12

    @property
    def head_dim(self) -> int:
        return self.hidden // self.num_heads


def weight_names(cfg: ClassicBertConfig) -> list[str]:
    """Tensor names of ``CpuBertModel::from_safetensors`` / ``load_classic_layer`` (``backend/cpu.rs:519-612``)."""
    names = [
        "embeddings.word_embeddings.weight",
        "embeddings.position_embeddings.weight",
        "embeddings.token_type_embeddings.weight",
        "embeddings.LayerNorm.weight",
        "embeddings.LayerNorm.bias",
    ]
    for i in range(cfg.num_layers):
        p = f"encoder.layer.{i}."
        for m in ("query", "key", "value"):
            names += [p + f"attention.self.{m}.weight", p + f"attention.self.{m}.bias"]
        names += [
            p + "attention.output.dense.weight", p + "attention.output.dense.bias",
            p + "attention.output.LayerNorm.weight", p + "attention.output.LayerNorm.bias",
            p + "intermediate.dense.weight", p + "intermediate.dense.bias",
            p + "output.dense.weight", p + "output.dense.bias",
            p + "output.LayerNorm.weight", p + "output.LayerNorm.bias",
        ]
    return names


def forward_hidden(w: dict, cfg: ClassicBertConfig, ids, dtype=np.float32) -> np.ndarray:
    """Final hidden states ``[L, hidden]`` of one sequence (token type 0 everywhere)."""
    dt = np.dtype(dtype).type
    W = {k: v.astype(dtype, copy=False) for k, v in w.items()}
    ids = np.asarray(ids, dtype=np.int64)
    L = len(ids)
    H, nh, hd = cfg.hidden, cfg.num_heads, cfg.head_dim
    x = (W["embeddings.word_embeddings.weight"][ids]
         + W["embeddings.position_embeddings.weight"][:L]
         + W["embeddings.token_type_embeddings.weight"][0][None, :])
    x = ops.layer_norm(x, W["embeddings.LayerNorm.weight"], W["embeddings.LayerNorm.bias"], cfg.norm_eps)
    scale = dt(1.0) / np.sqrt(dt(hd))
    mask = np.zeros(L, dtype)  # attention_mask is all ones for tokenizer output
    for i in range(cfg.num_layers):
        p = f"encoder.layer.{i}."
        wqkv = np.concatenate([W[p + f"attention.self.{m}.weight"] for m in ("query", "key", "value")], 0)
        bqkv = np.concatenate([W[p + f"attention.self.{m}.bias"] for m in ("query", "key", "value")], 0)
        qkv = ops.gemm_bt(x, wqkv) + bqkv
        q = qkv[:, :H].reshape(L, nh, hd)
        k = qkv[:, H:2 * H].reshape(L, nh, hd)
        v = qkv[:, 2 * H:].reshape(L, nh, hd)
        s = np.einsum("ihd,jhd->hij", q, k, optimize=False) * scale + mask[None, None, :]
        pr = ops.softmax_rows(s)
        ctx = np.einsum("hij,jhd->ihd", pr, v, optimize=False).reshape(L, H)
        proj = ops.gemm_bt(ctx, W[p + "attention.output.dense.weight"]) + W[p + "attention.output.dense.bias"]
        x = ops.layer_norm(x + proj, W[p + "attention.output.LayerNorm.weight"],
                           W[p + "attention.output.LayerNorm.bias"], cfg.norm_eps)
        inter = ops.gelu_tanh(ops.gemm_bt(x, W[p + "intermediate.dense.weight"]) + W[p + "intermediate.dense.bias"])
        out = ops.gemm_bt(inter, W[p + "output.dense.weight"]) + W[p + "output.dense.bias"]
        x = ops.layer_norm(x + out, W[p + "output.LayerNorm.weight"], W[p + "output.LayerNorm.bias"],
                           cfg.norm_eps)
    return x


def embed_sequence(w: dict, cfg: ClassicBertConfig, ids, pooling: str = "cls", dtype=np.float32) -> np.ndarray:
    ids = np.asarray(ids, dtype=np.int64)
    if len(ids) == 0:
        return np.zeros(cfg.hidden, dtype)
    h = forward_hidden(w, cfg, ids, dtype)
    v = h[0] if pooling == "cls" else ops.mean_pool(h)
    return ops.l2_normalize_floor(v)


def embed_batch(w: dict, cfg: ClassicBertConfig, ids, cu_seqlens, pooling: str = "cls",
                dtype=np.float32) -> np.ndarray:
    n = len(cu_seqlens) - 1
    out = np.zeros((n, cfg.hidden), dtype)
    for b in range(n):
        out[b] = embed_sequence(w, cfg, ids[cu_seqlens[b]:cu_seqlens[b + 1]], pooling, dtype)
    return out
