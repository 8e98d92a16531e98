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

    np.savez_compressed(OUT / "approx_search_small.npz", **approx_search_fixture())
    print("written to", OUT)


def approx_search_inputs():
    """600 x 128 normalised Gaussian rows (row 400 = row 9) and three queries (the last = row 9)."""
    db = synth.normalized_gaussian(600, 128, seed=61)
    db[400] = db[9]
    q = synth.normalized_gaussian(3, 128, seed=62)
    q[2] = db[9]
    return db, q


def approx_search_fixture() -> dict:
    """PolarQuant codes (bins, and radii as a checksum of their bits), approximate scores and
    rank_turboquant results; rank_cascade results; find_duplicates pairs."""
    from oracle import turbo_quant as tq

    db, q = approx_search_inputs()
    rot = tq.generate_rotation(128, 42)
    radii, bins = tq.encode(db, rot)
    out = {"bins": bins, "radii_bits_sum": np.uint64(radii.view(np.uint32).astype(np.uint64).sum()),
           "approx": np.stack([tq.scan_corpus(radii, bins, tq.prepare_query(x, rot)) for x in q])}
    for name, fn in (("tq", lambda x: tq.rank_turboquant(db, x, 5, -np.inf, rot, codes=(radii, bins))),
                     ("cascade", lambda x: scan.rank_cascade(db, x, 5, -np.inf, 64))):
        res = [fn(x) for x in q]
        out[f"{name}_idx"] = np.stack([r[0] for r in res])
        out[f"{name}_s64"] = np.stack([r[1] for r in res])
    a, b, s = scan.find_duplicates(db, 0.3, 50)
    out.update(dup_a=a, dup_b=b, dup_s64=s)
    return out


if __name__ == "__main__":
    main()
