/*
 * ripvec_b200 — C ABI of the B200 (sm_100a) embedding backend and cosine top-k scan.
 *
 * The library replaces, behind a thin FFI shim, the hot path of fnordpig/ripvec:
 *   - the embedding backend (`EmbedBackend`, crates/ripvec-core/src/backend/mod.rs:49-94,
 *     implemented for GPUs by `GenericBackend<CudaDriver, ModernBertArch>`,
 *     backend/generic.rs:147-184, and for ClassicBert by backend/cpu.rs:722-748), and
 *   - the exact search (`SearchIndex::new` / `SearchIndex::rank`,
 *     crates/ripvec-core/src/index.rs:76-186, scoring `similarity::rank_all`,
 *     similarity.rs:24-26), and
 *   - its two approximate rankings, `SearchIndex::rank_turboquant` over PolarQuant codes
 *     (index.rs:196-234, turbo_quant.rs) and the MRL cascade `SearchIndex::rank_cascade`
 *     (index.rs:245-297), and its all-pairs `SearchIndex::find_duplicates` (index.rs:325-348).
 *
 * Conventions: every entry point returns 0 (RV_OK) on success or a negative RV_E* code; the
 * message of the last failure on a handle is returned by rv_last_error / rv_index_last_error.
 * Nothing aborts or exits.  Input pointers are not retained after a call returns.  Host buffers
 * are plain CPU memory (pinned or not); "device" buffers are CUDA device pointers on the
 * handle's device.  A context or index may be used from several threads: calls on one handle
 * are serialised internally.
 */
#ifndef RIPVEC_B200_H
#define RIPVEC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define RV_OK 0
#define RV_E_INVALID -1     /* bad argument (null pointer, size, shape, unsupported option) */
#define RV_E_CUDA -2        /* CUDA runtime error */
#define RV_E_NOT_READY -3   /* weights missing / model not finalised */
#define RV_E_IO -4          /* file could not be read or parsed */
#define RV_E_DEVICE -5      /* a kernel reported an error (bounded wait expired, bad token) */
#define RV_E_NOMEM -6       /* device allocation failed */
#define RV_E_COMM -7        /* NCCL unavailable, a collective failed, or a rank did not answer in time */

/* ---------------------------------------------------------------- model description */
#define RV_ARCH_MODERNBERT 1  /* backend/arch/modern_bert.rs */
#define RV_ARCH_CLASSICBERT 2 /* backend/cpu.rs (BGE / BERT) */

#define RV_DTYPE_F32 0
#define RV_DTYPE_BF16 1
#define RV_DTYPE_F16 2

#define RV_POOL_MEAN 0 /* mean over the sequence (ModernBERT; BASELINE ClassicBert config) */
#define RV_POOL_CLS 1  /* first token (the reference ClassicBert CPU backend) */

/* Mirrors ModernBertConfig (backend/driver/cpu.rs:620-667) and BertConfig (backend/cpu.rs:52-92). */
typedef struct rv_model_desc {
  int32_t arch;                /* RV_ARCH_* */
  int32_t dtype;               /* RV_DTYPE_BF16 or RV_DTYPE_F16: device storage of weights and activations */
  int32_t hidden;              /* 768 (ModernBERT-base) / 384 (BERT-small) */
  int32_t num_layers;          /* 22 / 12 */
  int32_t num_heads;           /* 12 / 12 */
  int32_t intermediate;        /* 1152 (GeGLU half width) / 1536 */
  int32_t vocab;               /* 50368 / 30522 */
  int32_t max_position;        /* 8192 / 512 */
  int32_t global_every_n;      /* ModernBERT: layer i is global iff i % n == 0 (3) */
  int32_t local_window;        /* ModernBERT: 128 (keys with |i-j| <= 64 are visible) */
  float global_rope_theta;     /* 160000 */
  float local_rope_theta;      /* 10000 */
  float norm_eps;              /* 1e-5 / 1e-12 */
  int32_t type_vocab;          /* ClassicBert token-type rows (2) */
  int32_t pooling;             /* RV_POOL_MEAN / RV_POOL_CLS */
  int64_t max_batch_tokens;    /* device workspace: packed tokens per forward (0 = 262144) */
} rv_model_desc;

typedef struct rv_ctx rv_ctx;

/* Creates a context on CUDA device `device` for the model described by *desc.  Weights are then
 * supplied with rv_set_weight (or rv_load_safetensors) and the model is frozen by rv_finalize. */
int rv_create(const rv_model_desc* desc, int device, rv_ctx** out);
void rv_destroy(rv_ctx* ctx);

/* Uploads one named f32 host tensor (names as in the reference's safetensors files, e.g.
 * "layers.3.attn.Wqkv.weight", "embeddings.tok_embeddings.weight", "final_norm.weight";
 * ClassicBert: "encoder.layer.0.attention.self.query.weight", ...).  numel must match. */
int rv_set_weight(rv_ctx* ctx, const char* name, const float* host, int64_t numel);
/* Reads every tensor of a safetensors file (F32, BF16 or F16) through rv_set_weight. */
int rv_load_safetensors(rv_ctx* ctx, const char* path);
/* Checks that every weight is present and builds the device layouts (interleaved Wi, RoPE
 * tables, TMA descriptors).  Required before rv_embed_*. */
int rv_finalize(rv_ctx* ctx);

/* EmbedBackend::embed_batch.  ids: packed int32 token ids of n_seqs sequences, sequence b being
 * ids[cu_seqlens[b] .. cu_seqlens[b+1]); cu_seqlens has n_seqs+1 entries, cu_seqlens[0] = 0,
 * non-decreasing, every length <= rv_max_tokens.  out_host: [n_seqs, hidden] f32 L2-normalised
 * embeddings in input order.  Host buffers; the copies are part of the call. */
int rv_embed_varlen(rv_ctx* ctx, const int32_t* ids, const int32_t* cu_seqlens, int32_t n_seqs,
                    float* out_host);
/* Same with device-resident ids and output (out_dev: [n_seqs, hidden] of out_dtype f32/bf16/f16);
 * cu_seqlens stays on the host (it drives the token-budget packing).  stream may be 0. */
int rv_embed_varlen_device(rv_ctx* ctx, const int32_t* ids_dev, const int32_t* cu_seqlens_host,
                           int32_t n_seqs, void* out_dev, int32_t out_dtype, void* stream);

/* Asynchronous form of rv_embed_varlen, for a caller that keeps the GPU fed while it tokenises the
 * next chunks (the reference's bounded pipeline of tokeniser threads feeding the embedding stage,
 * crates/ripvec-core/src/embed.rs:273-463).  rv_embed_submit copies the ids into the context's
 * pinned staging, queues the copies and the forward of every packed batch on the context's
 * stream and returns at once with a ticket; out_host must stay valid until rv_embed_wait on that
 * ticket returns.  At most two batches are in flight: a submission whose batches need a busy
 * staging slot first completes the oldest batch (moving its embeddings to its caller's buffer).
 * Input errors (bad cu_seqlens, token ids outside the vocabulary) are returned by the submit;
 * device errors of a job are returned by its wait.  rv_embed_wait returns when the embeddings of
 * the ticket (and of every earlier ticket) are in their buffers; waiting on a ticket twice
 * returns RV_OK. */
int rv_embed_submit(rv_ctx* ctx, const int32_t* ids, const int32_t* cu_seqlens, int32_t n_seqs, float* out_host,
                    int64_t* ticket);
int rv_embed_wait(rv_ctx* ctx, int64_t ticket);

/* embed_distributed over several backends (crates/ripvec-core/src/embed.rs:666-785): one host
 * thread per context (each context on its own GPU, or several on one), all taking runs of
 * consecutive chunks from one cursor in input order, each run sized to its context's token
 * budget and embedded with rv_embed_varlen straight into out_host ([n_seqs, hidden] f32, input
 * order).  Contexts must share the hidden size.  The first failure stops the other workers from
 * taking new runs and is returned; its message is on the failing context (rv_last_error). */
int rv_embed_varlen_multi(rv_ctx* const* ctxs, int32_t n_ctx, const int32_t* ids, const int32_t* cu_seqlens,
                          int32_t n_seqs, float* out_host);

int rv_max_tokens(const rv_ctx* ctx);   /* EmbedBackend::max_tokens */
int rv_hidden_dim(const rv_ctx* ctx);
const char* rv_name(const rv_ctx* ctx); /* EmbedBackend::name */
int rv_is_gpu(const rv_ctx* ctx);       /* EmbedBackend::is_gpu (1) */
const char* rv_last_error(const rv_ctx* ctx);
/* Number of kernels this context launched since creation (for launch accounting). */
int64_t rv_kernel_launches(const rv_ctx* ctx);

/* Per-kernel timing: when enabled, every kernel launch of rv_embed_* is bracketed by CUDA events
 * on the context's stream and its device time is accumulated per kernel kind. */
#define RV_KIND_GEMM 0      /* tcgen05 projection GEMMs (all four per layer) */
#define RV_KIND_ATTENTION 1 /* varlen attention */
#define RV_KIND_NORM 2      /* LayerNorm */
#define RV_KIND_EMBED 3     /* embedding gather + LayerNorm, positions */
#define RV_KIND_POOL 4      /* final LayerNorm + mean pool + L2 */
#define RV_KIND_COUNT 5
int rv_set_profiling(rv_ctx* ctx, int enable);
/* Totals since the last reset: device milliseconds, launches and algorithmic FLOPs (GEMM: 2MNK;
 * attention: 4 * head_dim * heads * visible query-key pairs; others 0). */
int rv_get_profile(rv_ctx* ctx, int kind, double* total_ms, int64_t* launches, double* flops);
int rv_reset_profile(rv_ctx* ctx);

/* ---------------------------------------------------------------- search */
typedef struct rv_index rv_index;

/* SearchIndex::new: a bf16 device copy of n rows of dimension dim.  src is f32, bf16 or f16
 * (src_dtype); src_on_device selects a device or host source.  Rows are stored as given (the
 * reference stores embed_batch output, already L2-normalised). */
int rv_index_create(int device, const void* src, int64_t n, int32_t dim, int32_t src_dtype,
                    int32_t src_on_device, rv_index** out);
void rv_index_destroy(rv_index* idx);
const char* rv_index_last_error(const rv_index* idx);
int64_t rv_index_size(const rv_index* idx);
/* Kernels this index has launched so far (all search entry points; for benchmarks). */
int64_t rv_index_kernel_launches(rv_index* idx);
/* Global row index of this shard's first row (rows are numbered base + local row in results). */
int rv_index_set_base(rv_index* idx, int64_t base);

/* SearchIndex::rank restricted to the best k: for each of nq queries (f32, [nq, dim], rounded
 * to bf16 like the stored rows) return its k best rows ordered by (score desc, row asc), scores
 * computed exactly (sequential f64 sum of exact bf16 products).  Rows scoring below threshold
 * are dropped: out_count[q] (optional) receives the number kept and the tail of out_idx is
 * filled with -1 / out_score with -inf.  out_idx [nq, k] int64, out_score [nq, k] f32; the f64
 * scores are also returned when out_score64 is non-null.  Host buffers. */
int rv_index_topk(rv_index* idx, const float* queries, int32_t nq, int32_t k, float threshold,
                  int64_t* out_idx, float* out_score, double* out_score64, int32_t* out_count);
/* Device-buffer variant of rv_index_topk (queries_dev f32 [nq, dim]; outputs on the device). */
int rv_index_topk_device(rv_index* idx, const float* queries_dev, int32_t nq, int32_t k,
                         float threshold, int64_t* out_idx_dev, float* out_score_dev,
                         double* out_score64_dev, void* stream);
/* SearchIndex::rank in full (crates/ripvec-core/src/index.rs:172-186): every row whose exact
 * score (as rv_index_topk) is >= threshold, ordered by (score desc, row asc); no cap on the
 * number of rows (MCP find_similar ranks at threshold 0.0 and pages through the whole result,
 * ripvec-mcp/src/tools.rs:563-570).  query: host f32 [dim].  The first min(count, capacity)
 * results go to out_idx / out_score (/ out_score64 when non-null), host buffers; *out_count
 * receives the total count, so a caller can size its buffers with capacity = 0 (or rv_index_size)
 * first.  threshold = -inf ranks every row. */
int rv_index_rank(rv_index* idx, const float* query, float threshold, int64_t capacity, int64_t* out_idx,
                  float* out_score, double* out_score64, int64_t* out_count);
/* Merges n_lists per-shard results [n_lists, nq, k] (device; idx int64, score f64, as returned
 * by rv_index_topk_device) into the global top k per query, ordered by (score desc, idx asc). */
int rv_topk_merge_device(int device, const int64_t* idx_in, const double* score_in,
                         int32_t n_lists, int32_t nq, int32_t k, float threshold,
                         int64_t* idx_out, float* score_out, double* score64_out, void* stream);

/* ---------------------------------------------------------------- row-sharded search over GPUs
 * A database too large for one GPU (or searched faster by several) is split into contiguous row
 * ranges, one rv_index per GPU with rv_index_set_base giving each its first global row.  The
 * ranks exchange their per-shard top-k lists over NCCL (one all-gather of [nq, k] rows and f64
 * scores; NVLink / NVSwitch between the GPUs of a node) and merge them on the device.  One
 * process or thread per GPU drives its rank.  NCCL is loaded at run time (libnccl.so.2); without
 * it these entry points return RV_E_COMM.  No counterpart in the reference, which ranks one
 * in-memory matrix (SearchIndex::rank, crates/ripvec-core/src/index.rs:172-186); the merged
 * result equals rv_index_topk over the whole database. */
typedef struct rv_comm rv_comm;
#define RV_COMM_ID_BYTES 128
/* Rank 0 creates the id and hands the same RV_COMM_ID_BYTES bytes to every rank (through the
 * caller's own channel: a store, a socket, a broadcast). */
int rv_comm_get_unique_id(uint8_t* id);
/* Joins the communicator of `world` ranks as `rank` on CUDA device `device`.  Every wait on the
 * communicator (this one included) gives up after timeout_ms, aborts the communicator and
 * returns RV_E_COMM, so a rank that never joins or stops answering ends the call with an error
 * rather than a hang. */
int rv_comm_create(int device, const uint8_t* id, int32_t rank, int32_t world, int32_t timeout_ms,
                   rv_comm** out);
void rv_comm_destroy(rv_comm* comm);
const char* rv_comm_last_error(const rv_comm* comm);
int rv_comm_rank(const rv_comm* comm);
int rv_comm_world(const rv_comm* comm);
/* The exact global top k of the queries over every rank's shard: this shard's best k
 * (rv_index_topk_device), the all-gather of every rank's lists, and the device merge by
 * (score desc, row asc).  Every rank passes the same queries (device f32 [nq, dim]) and receives
 * the same [nq, k] results (device buffers, as rv_index_topk_device); every rank must make the
 * same calls in the same order.  world * k <= 8192.  Returns when the results are written. */
int rv_index_topk_sharded(rv_index* idx, rv_comm* comm, const float* queries_dev, int32_t nq, int32_t k,
                          float threshold, int64_t* out_idx_dev, float* out_score_dev,
                          double* out_score64_dev, void* stream);

/* The same exact top-k as rv_index_topk_device for callers that cannot allocate device memory
 * (a host whose allocator or memory pool owns the whole device budget, or a serving thread that
 * must not let cudaMalloc / cudaFree synchronise the device).  No counterpart in the reference:
 * it exists only for such callers.  All scratch lives in one fixed device array inside the
 * library (about 5 MiB, held by every GPU that loads the library until exit); the call makes
 * no cudaMalloc / cudaFree.  Limits: nq <= 16 queries, k <= 64, rows of at most 4096
 * dimensions; larger requests return RV_E_INVALID.  Device buffers as in rv_index_topk_device;
 * runs on `stream` (0 = the index's stream) and returns when the results are written.  The first
 * call on a device looks up the array's device address; make it before any stream capture.
 * Calls share the array: calls that overlap on the GPU race and must be serialised by the
 * caller.  Near-tied scores that need a wider candidate list than the array holds return
 * RV_E_DEVICE (rv_index_topk_device handles them). */
int rv_index_topk_noalloc(rv_index* idx, const float* queries_dev, int32_t nq, int32_t k,
                          float threshold, int64_t* out_idx_dev, float* out_score_dev,
                          double* out_score64_dev, void* stream);

/* ---------------------------------------------------------------- PolarQuant ("TurboQuant") search
 * The approximate first phase of SearchIndex::rank_turboquant (crates/ripvec-core/src/
 * index.rs:196-234) over the 4-bit polar codes of turbo_quant.rs. */

/* PolarCodec::new + encode_batch (turbo_quant.rs:92-188), as SearchIndex::new builds it
 * (index.rs:136-158): encodes every stored row under `rotation` (host, [dim, dim] f32 row-major,
 * rotated_j = sum_d rotation[j][d] x_d; orthogonal in the reference, generate_rotation
 * turbo_quant.rs:335-343) with `bits` bits per angle (1..4; the reference uses 4).  Per pair of
 * rotated values: an f32 radius and an angle bin.  The rotation sums in order over d with
 * rounded products (no fused multiply-add) and the angle is the f64 atan2 rounded to f32, so
 * codes are reproducible bit for bit.  Rebuilding replaces the previous corpus.  The reference
 * builds it only for indexes of at least 4096 rows; that policy is the caller's. */
int rv_index_build_polar(rv_index* idx, const float* rotation, int32_t bits);
/* 1 when a PolarQuant corpus is present. */
int rv_index_has_polar(const rv_index* idx);
/* The corpus in the reference's SoA layout (CompressedCorpus, turbo_quant.rs:39-49): radii
 * [n, dim/2] f32 and angle bins [n, dim/2] u8, host buffers. */
int rv_index_polar_export(rv_index* idx, float* radii, uint8_t* bins);
/* PolarCodec::prepare_query + scan_corpus (turbo_quant.rs:212-289): approximate scores
 * [nq, n] f32 of the f32 queries [nq, dim] against every row, host buffers. */
int rv_index_polar_scores(rv_index* idx, const float* queries, int32_t nq, float* scores);
/* SearchIndex::rank_turboquant (index.rs:196-234) restricted to top_k results: approximate
 * scores of every row, the best min(10 * top_k, n) rows by (approximate score desc, row asc),
 * re-scored exactly (as rv_index_topk), rows below threshold dropped, the best top_k by
 * (score desc, row asc).  Without a corpus it equals rv_index_topk (the reference falls back to
 * rank, index.rs:202-204).  top_k in [1, 800].  Outputs as rv_index_topk; host buffers. */
int rv_index_rank_turboquant(rv_index* idx, const float* queries, int32_t nq, int32_t top_k, float threshold,
                             int64_t* out_idx, float* out_score, double* out_score64, int32_t* out_count);
/* Device-buffer variant of rv_index_rank_turboquant (outputs as rv_index_topk_device). */
int rv_index_rank_turboquant_device(rv_index* idx, const float* queries_dev, int32_t nq, int32_t top_k,
                                    float threshold, int64_t* out_idx_dev, float* out_score_dev,
                                    double* out_score64_dev, void* stream);

/* ---------------------------------------------------------------- MRL cascade search */
/* SearchIndex::new with cascade_dim (crates/ripvec-core/src/index.rs:99-132): builds the
 * truncated matrix of the stored rows: LayerNorm over the full row (mean, biased variance,
 * 1 / sqrt(var + 1e-5)), the first trunc_dim values, L2-normalised (norm floored at 1e-12); sums
 * in order over the dimensions in f32, stored in bf16.  trunc_dim is clamped to the row
 * dimension and must then be a multiple of 64.  Rebuilding replaces the previous matrix. */
int rv_index_build_cascade(rv_index* idx, int32_t trunc_dim);
/* The truncated dimension, or 0 without a truncated matrix (SearchIndex::truncated_dim). */
int rv_index_cascade_dim(const rv_index* idx);
/* The truncated matrix [n, trunc_dim] as f32 (the stored bf16 values), host buffer. */
int rv_index_cascade_rows(rv_index* idx, float* out);
/* SearchIndex::rank_cascade (index.rs:245-297): the query gets the same transform; the best
 * max(100, 3 top_k) rows of the truncated matrix (exact top-k there) are re-scored exactly
 * with the full rows (as rv_index_topk), rows below threshold dropped, the best top_k by
 * (score desc, row asc).  Without a truncated matrix it equals rv_index_topk (the reference
 * falls back to rank).  top_k in [1, 682].  Outputs as rv_index_topk; host buffers. */
int rv_index_rank_cascade(rv_index* idx, const float* queries, int32_t nq, int32_t top_k, float threshold,
                          int64_t* out_idx, float* out_score, double* out_score64, int32_t* out_count);

/* ---------------------------------------------------------------- embedding store */
/* The embeddings of one per-file cache object (crates/ripvec-core/src/cache/file_cache.rs:15-70,
 * read back by cache/reindex.rs:302, :411): a zstd frame around an rkyv 0.8 archive of
 * FileCache { chunks, embeddings: [n x hidden_dim] f32, hidden_dim }, or the bare archive.
 * Host-only (no device needed).  Rows: the chunks whose whole embedding slice is present,
 * min(chunks, len(embeddings) / hidden_dim) (cache/reindex.rs:578-587).  out_emb = NULL: only
 * *out_rows and *out_dim = hidden_dim are set; else rows * hidden_dim floats go to out_emb
 * (capacity_floats at least that).  Objects starting with "BC" (the portable bitcode form,
 * FileCache::to_portable_bytes) and malformed objects return RV_E_IO; the message is
 * rv_cache_last_error() (per thread).  zstd is the system's libzstd.so.1. */
int rv_cache_decode(const uint8_t* obj, uint64_t nbytes, float* out_emb, int64_t capacity_floats, int64_t* out_rows,
                    int32_t* out_dim);
const char* rv_cache_last_error(void);
/* Rows [row0, row0 + n) of an index, as stored (RV_DTYPE_BF16) or widened to f32 (exact), into a
 * host or device buffer: the export side of a device shard (rv_index_create reads it back). */
int rv_index_export(rv_index* idx, int64_t row0, int64_t n, int32_t dst_dtype, void* dst, int32_t dst_on_device);

/* ---------------------------------------------------------------- near-duplicate pairs */
/* SearchIndex::find_duplicates (crates/ripvec-core/src/index.rs:325-348): the pairs (a, b), a < b,
 * whose exact score (as rv_index_topk: sequential f64 sum of the bf16 products) is >= threshold,
 * ordered by (score desc, a asc, b asc), at most max_pairs of them.  Fewer than two rows give no
 * pairs.  Rows are numbered base + local row.  out_a / out_b [max_pairs] int64, out_score
 * [max_pairs] f32, out_score64 (optional) f64, *out_count = pairs written; host buffers.  One
 * pass keeps up to 8388608 candidate pairs (f32 score within the error bound, about
 * dim * 2^-22 for unit rows, of the cut).  When more reach the threshold's bound, the cut is
 * raised by bisection, one pass per step, until the candidates fit and at least max_pairs pairs
 * reach the cut; RV_E_DEVICE only when no cut does (more than 8388608 pairs within the bound
 * of the max_pairs-th best score, or of the threshold itself). */
int rv_index_find_duplicates(rv_index* idx, float threshold, int64_t max_pairs, int64_t* out_a, int64_t* out_b,
                             float* out_score, double* out_score64, int64_t* out_count);

/* ---------------------------------------------------------------- single-kernel entry points
 * Used by the parity tests to check one kernel against the CPU oracle.  Device pointers. */
/* C[M,N] (f32 or act) = A[M,K] B[N,K]^T with A, B of act dtype (RV_DTYPE_BF16/F16); bn = 128 or
 * 256 (one-CTA 128 x bn tiles) or 512 (two-CTA 256 x 256 tiles). */
int rv_op_gemm(int32_t act_dtype, const void* a, const void* b, void* c, int32_t c_dtype,
               int32_t M, int32_t N, int32_t K, int32_t bn, void* stream);
/* Attention over packed qkv [T, 3*heads*head_dim]; window_half < 0 = global.  head_dim 64 runs
 * the tcgen05 kernel (environment RV_ATTN_TC=0 selects the mma.sync kernel instead); head_dim
 * 32 always runs the mma.sync kernel.  A pipeline wait that expires returns RV_E_DEVICE. */
int rv_op_attention(int32_t act_dtype, const void* qkv, void* ctx_out, const int32_t* cu_seqlens_host,
                    int32_t n_seqs, int32_t num_heads, int32_t head_dim, int32_t window_half,
                    float scale, void* stream);
/* Test hook of the device-side error path (no counterpart in the reference; the reference's
 * contract is that errors propagate, backend/mod.rs:53-54).  While enabled, every tcgen05
 * attention launch (rv_op_attention and the attention of rv_embed_*) withholds the score signal
 * of each persistent CTA's first tile and bounds every pipeline wait by wait_limit_cycles SM
 * cycles: the softmax warps' wait expires, every role leaves through the kernel's bounded-wait
 * exit (copies and MMAs in flight are drained, TMEM is freed), and the call returns RV_E_DEVICE.
 * Nothing faults, traps or spins without bound.  enable = 0 restores normal launches.  Process
 * wide; for tests only. */
int rv_debug_stall_attention(int32_t enable, int64_t wait_limit_cycles);
/* Test hook (no counterpart in the reference): y[i] = 2^x[i] by the tcgen05 attention's
 * FMA-pipe exponential (range reduction by rint, degree-3 minimax polynomial, exponent add;
 * relative error below 7.6e-5 for x in [-125, 126], 0 below -125), which its
 * softmax computes for a quarter of the fully visible exponentials beside the MUFU ex2 when the
 * environment sets RV_ATTN_EXP2_POLY=1.  Device pointers; synchronous on stream. */
int rv_debug_exp2_poly(const float* x, float* y, int64_t n, void* stream);
/* out = LN(in) * gamma (+ beta); 16-bit rows. */
int rv_op_layernorm(int32_t act_dtype, const void* in, void* out, int32_t rows, int32_t hidden,
                    const float* gamma, const float* beta, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RIPVEC_B200_H */
