"""Shared test configurations and comparison helpers."""

from __future__ import annotations

import numpy as np

from oracle.classic_bert import ClassicBertConfig
from oracle.modern_bert import ModernBertConfig
from ripvec_b200 import synth
from ripvec_b200.synth import ModelSpec

# Small models with the real head dimensions (64 for ModernBERT, 32 for BERT-small) so the same
# kernels run; the full-size configurations are used where the oracle stays fast enough.
TINY_MODERN = ModelSpec("modernbert", hidden=256, num_layers=4, num_heads=4, intermediate=384, vocab=1000,
                        max_position=1024)
TINY_CLASSIC = ModelSpec("classicbert", hidden=128, num_layers=2, num_heads=4, intermediate=256, vocab=500,
                         max_position=128, norm_eps=1e-12)


def modern_cfg(spec: ModelSpec) -> ModernBertConfig:
    return ModernBertConfig(hidden=spec.hidden, num_layers=spec.num_layers, num_heads=spec.num_heads,
                            intermediate=spec.intermediate, vocab=spec.vocab, max_position=spec.max_position,
                            global_every_n=spec.global_every_n, local_window=spec.local_window,
                            global_rope_theta=spec.global_rope_theta, local_rope_theta=spec.local_rope_theta,
                            norm_eps=spec.norm_eps)


def classic_cfg(spec: ModelSpec) -> ClassicBertConfig:
    return ClassicBertConfig(hidden=spec.hidden, num_layers=spec.num_layers, num_heads=spec.num_heads,
                             intermediate=spec.intermediate, vocab=spec.vocab, max_position=spec.max_position,
                             type_vocab=spec.type_vocab, norm_eps=spec.norm_eps)


def row_cosines(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    na = np.linalg.norm(a, axis=1)
    nb = np.linalg.norm(b, axis=1)
    return (a * b).sum(1) / np.maximum(na * nb, 1e-300)


def scan_small_inputs():
    """3000 x 128 normalised Gaussian rows with one exact duplicate (row 2000 = row 17) and six
    queries, the last equal to row 17, so that ties must break by row index."""
    db = synth.normalized_gaussian(3000, 128, seed=21)
    db[2000] = db[17]
    q = synth.normalized_gaussian(6, 128, seed=22)
    q[5] = db[17]
    return db, q
