"""Generates the model-level golden fixtures from the CPU oracle (seeded weights and inputs).

The reference has no model-level golden vectors (its model tests download checkpoints), so
these fixtures pin the oracle's own output on fixed seeds: the CPU tests check that the oracle
still reproduces them, and the GPU tests compare the CUDA path against them.  Weights are not
stored; they are regenerated from the seed by ``ripvec_b200.synth.random_weights``.

Run from the repository root: ``python tests/golden/make_golden.py``.
"""

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from helpers import TINY_CLASSIC, TINY_MODERN, classic_cfg, modern_cfg, scan_small_inputs  # noqa: E402
from oracle import classic_bert, modern_bert, scan  # noqa: E402
from ripvec_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def main():
    # ModernBERT (tiny, stress variant so attention is not uniform); lengths cover the 64-token
    # tile edges and the +-64 window edges.
    lengths = np.array([1, 5, 63, 64, 65, 129, 200, 300], np.int32)
    ids, cu = synth.packed_ids(lengths, TINY_MODERN.vocab, seed=11)
    w = synth.random_weights(TINY_MODERN, seed=7, qk_std=0.2)
    emb = modern_bert.embed_batch(w, modern_cfg(TINY_MODERN), ids, cu)
    np.savez_compressed(OUT / "modernbert_tiny.npz", ids=ids, cu=cu, emb=emb, weight_seed=7, qk_std=0.2)

    lengths = np.array([1, 2, 17, 64, 100, 128], np.int32)
    ids, cu = synth.packed_ids(lengths, TINY_CLASSIC.vocab, seed=12)
    w = synth.random_weights(TINY_CLASSIC, seed=8, qk_std=0.2)
    cfg = classic_cfg(TINY_CLASSIC)
    np.savez_compressed(OUT / "classicbert_tiny.npz", ids=ids, cu=cu,
                        emb_cls=classic_bert.embed_batch(w, cfg, ids, cu, "cls"),
                        emb_mean=classic_bert.embed_batch(w, cfg, ids, cu, "mean"), weight_seed=8, qk_std=0.2)

    db, q = scan_small_inputs()
    idx, s64, cnt = scan.topk_exact(db, q, 10)
    np.savez_compressed(OUT / "scan_small.npz", idx=idx, s64=s64, k=10)
    print("written to", OUT)


if __name__ == "__main__":
    main()
