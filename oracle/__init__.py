"""CPU oracle for the ripvec hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's own CPU path for the functions the B200
library replaces, so that the parity tests can check the CUDA kernels against it:

* ``modern_bert`` — ModernBERT encoder forward of ``crates/ripvec-core/src/backend/arch/
  modern_bert.rs`` (FP32 branch) over the ops of ``backend/driver/cpu.rs``;
* ``classic_bert`` — the ClassicBert (BGE / BERT) CPU backend ``backend/cpu.rs``;
* ``scan`` — exact cosine ranking (``similarity.rs::rank_all`` + ``index.rs::SearchIndex::rank``)
  plus the bit-exact top-k definition used by the GPU scan.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
this package, and only as the checker or the timed CPU baseline.  The product path
(``ripvec_b200``) never imports it and has no CPU fallback.

Pinning: the op-level functions are checked against every known-answer test the reference
holds for this path (``tests/golden/reference_known_answers.json``, produced by
``tests/golden/make_known_answers.py``), and the fp32 forward is cross-checked against an
independent fp64 evaluation of the same equations.  The reference has no model-level golden
vectors (its ModernBERT / BGE tests need downloaded checkpoints), so model-level parity is
pinned only through those op-level answers.
"""
