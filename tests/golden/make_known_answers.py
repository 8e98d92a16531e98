"""Writes ``reference_known_answers.json``: the known-answer tests the reference holds for the
hot path, transcribed from its test modules (inputs, expected outputs and tolerances as the
reference asserts them), each with the file:line of the reference test it comes from.

Run from the repository root: ``python tests/golden/make_known_answers.py``.
"""

import json
from pathlib import Path

CASES = [
    {"id": "gelu_smoke", "ref": "crates/ripvec-core/src/backend/driver/cpu.rs:1541",
     "op": "gelu", "input": [0.0, 1.0, -1.0, 2.0],
     "checks": [{"index": 0, "expect": 0.0, "tol": 1e-4}, {"index": 1, "expect": 0.8412, "tol": 0.01},
                {"index": 2, "expect": -0.1588, "tol": 0.01}]},
    {"id": "layer_norm_smoke", "ref": "crates/ripvec-core/src/backend/driver/cpu.rs:1568",
     "op": "layer_norm", "input": [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]], "weight": [1.0, 1.0, 1.0],
     "bias": [0.0, 0.0, 0.0], "eps": 1e-5, "checks": [{"row_mean": 0, "expect": 0.0, "tol": 1e-5}]},
    {"id": "gemm_smoke", "ref": "crates/ripvec-core/src/backend/driver/cpu.rs:1589",
     "op": "gemm", "a": [[1.0, 2.0], [3.0, 4.0]], "b": [[5.0, 6.0], [7.0, 8.0]], "transpose_b": False,
     "expect": [[19.0, 22.0], [43.0, 50.0]], "tol": 1e-4},
    {"id": "gemm_transpose_b", "ref": "crates/ripvec-core/src/backend/driver/cpu.rs:1608",
     "op": "gemm", "a": [[1.0, 2.0], [3.0, 4.0]], "b": [[5.0, 6.0], [7.0, 8.0]], "transpose_b": True,
     "expect": [[17.0, 23.0], [39.0, 53.0]], "tol": 1e-4},
    {"id": "embedding_lookup", "ref": "crates/ripvec-core/src/backend/driver/cpu.rs:1627",
     "op": "embedding_lookup", "table": [[0.1, 0.2], [0.3, 0.4], [0.5, 0.6], [0.7, 0.8], [0.9, 1.0]],
     "ids": [2, 0, 4], "expect": [[0.5, 0.6], [0.1, 0.2], [0.9, 1.0]], "tol": 0.0},
    {"id": "cls_pool", "ref": "crates/ripvec-core/src/backend/driver/cpu.rs:1646",
     "op": "cls_pool", "hidden": [[1.0, 2.0], [3.0, 4.0], [5.0, 6.0], [7.0, 8.0], [9.0, 10.0], [11.0, 12.0]],
     "batch": 2, "seq": 3, "expect": [[1.0, 2.0], [7.0, 8.0]], "tol": 0.0},
    {"id": "dot_identical_normalized", "ref": "crates/ripvec-core/src/similarity.rs:34",
     "op": "dot", "a": [0.5773, 0.5773, 0.5773], "b": [0.5773, 0.5773, 0.5773], "expect": 1.0, "tol": 0.01},
    {"id": "dot_orthogonal", "ref": "crates/ripvec-core/src/similarity.rs:41",
     "op": "dot", "a": [1.0, 0.0, 0.0], "b": [0.0, 1.0, 0.0], "expect": 0.0, "tol": 1e-6},
    {"id": "dot_opposite", "ref": "crates/ripvec-core/src/similarity.rs:49",
     "op": "dot", "a": [1.0, 0.0], "b": [-1.0, 0.0], "expect": -1.0, "tol": 1e-6},
    {"id": "rank_all_matches_scalar", "ref": "crates/ripvec-core/src/similarity.rs:57",
     "op": "rank_all_vs_dot",
     "embeddings": [[1.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.5773, 0.5773, 0.5773], [-1.0, 0.0, 0.0]],
     "query": [1.0, 0.0, 0.0], "tol": 1e-6},
    {"id": "rank_all_empty", "ref": "crates/ripvec-core/src/similarity.rs:82",
     "op": "rank_all", "embeddings_shape": [0, 384], "query": "zeros384", "expect": []},
    {"id": "rank_all_known_values_1", "ref": "crates/ripvec-core/src/similarity.rs:90",
     "op": "rank_all", "embeddings": [[1.0, 2.0], [3.0, 4.0]], "query": [1.0, 0.0], "expect": [1.0, 3.0], "tol": 1e-6},
    {"id": "rank_all_known_values_2", "ref": "crates/ripvec-core/src/similarity.rs:90",
     "op": "rank_all", "embeddings": [[1.0, 2.0], [3.0, 4.0]], "query": [0.0, 1.0], "expect": [2.0, 4.0], "tol": 1e-6},
    {"id": "rank_sorted_threshold", "ref": "crates/ripvec-core/src/index.rs:414",
     "op": "rank", "embeddings": [[0.2, 0.8], [0.9, 0.1], [0.5, 0.5]], "query": [1.0, 0.0], "threshold": 0.3,
     "expect_rows": [1, 2]},
    {"id": "rank_wrong_dimension", "ref": "crates/ripvec-core/src/index.rs:432",
     "op": "rank", "embeddings": [[1.0, 0.0, 0.0]], "query": [1.0, 0.0], "threshold": 0.0, "expect_rows": []},
    {"id": "rank_empty_query", "ref": "crates/ripvec-core/src/index.rs:444",
     "op": "rank", "embeddings": [[1.0, 0.0, 0.0]], "query": [], "threshold": 0.0, "expect_rows": []},
    {"id": "rank_empty_index", "ref": "crates/ripvec-core/src/index.rs:455",
     "op": "rank", "embeddings_shape": [0, 384], "query": "ones384", "threshold": 0.0, "expect_rows": []},
    {"id": "embed_l2_norm", "ref": "crates/ripvec-core/src/backend/cpu.rs:865",
     "op": "invariant", "what": "every embedding has L2 norm 1 within 1e-4"},
    {"id": "embed_inputs_differ", "ref": "crates/ripvec-core/src/backend/cpu.rs:881",
     "op": "invariant", "what": "different inputs give embeddings with cosine < 0.99"},
    {"id": "embed_empty_batch", "ref": "crates/ripvec-core/src/backend/cpu.rs:909",
     "op": "invariant", "what": "an empty batch returns an empty result"},
]

if __name__ == "__main__":
    out = Path(__file__).resolve().parent / "reference_known_answers.json"
    out.write_text(json.dumps({"source": "fnordpig/ripvec v0.13.21 test modules", "cases": CASES}, indent=1) + "\n")
    print(out)
