"""ripvec_b200 — B200-native (sm_100a) embedding backend and exact cosine top-k scan for ripvec.

The compute path is ``librv_b200.so`` (hand-written CUDA for sm_100a behind a C ABI, declared in
``include/ripvec_b200.h``); this package is its host-side mirror of the reference interfaces:
``EmbedBackend`` / ``Encoding`` / ``load_backend`` (``backend.py``) and ``SearchIndex``
(``index.py``).
"""

from .backend import EmbedBackend, Encoding, embed_distributed, load_backend, pack_encodings  # noqa: F401
from .synth import BERT_SMALL, MODERNBERT_BASE, ModelSpec  # noqa: F401

__all__ = ["EmbedBackend", "Encoding", "embed_distributed", "load_backend", "pack_encodings", "ModelSpec", "MODERNBERT_BASE",
           "BERT_SMALL"]
