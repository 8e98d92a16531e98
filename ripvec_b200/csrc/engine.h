// Host-side engine shared by the C ABI translation units: the context object, weight storage,
// workspaces and small utilities.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <deque>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/ripvec_b200.h"
#include "kernels.h"

namespace rv {

// Rounds f32 to bf16 (round to nearest even), host side.
uint16_t f32_to_bf16_bits(float f);
uint16_t f32_to_f16_bits(float f);

// Converts host f32 to the device dtype and uploads.  Returns false on CUDA error.
bool upload_converted(const float* host, int64_t n, Act act, void** dev, std::string* why);
bool upload_f32(const float* host, int64_t n, float** dev, std::string* why);

struct DeviceMatrix {
  void* ptr = nullptr;   // [rows, cols] 16-bit, row-major
  int rows = 0, cols = 0;
  CUtensorMap tmap;      // B-operand map, box 64 x bn
  CUtensorMap tmap_half; // box 64 x 128: each CTA's half of a two-CTA 256-wide tile
  int bn = 256;
};

struct LayerWeights {
  DeviceMatrix wqkv, wo, wi, wo2;
  float* attn_norm = nullptr;  // ModernBERT (null for layer 0)
  float* mlp_norm = nullptr;
  float* csum_qkv = nullptr;   // column sums of the LayerNorm-folded Wqkv (layers > 0)
  float* csum_wi = nullptr;    // column sums of the LayerNorm-folded, interleaved Wi
  float* bqkv = nullptr;       // ClassicBert biases and post-LN parameters
  float* bo = nullptr;
  float* ln1_w = nullptr;
  float* ln1_b = nullptr;
  float* b1 = nullptr;
  float* b2 = nullptr;
  float* ln2_w = nullptr;
  float* ln2_b = nullptr;
  bool is_global = true;
};

}  // namespace rv

// Pinned host staging of one in-flight batch of the asynchronous path (rv_embed_submit).
struct AsyncSlot {
  int32_t* ids_h = nullptr;       // [t_max] token ids
  int* meta_h = nullptr;          // [2 (n_max + 1)] cu_seqlens and 64-query tile prefix
  int2* tiles_h = nullptr;        // [tiles_cap] 128-query attention tile records
  float* out_h = nullptr;         // [out_cap] embeddings of the batch
  size_t out_cap = 0;
  unsigned int* err_h = nullptr;  // the device error word after the batch
  cudaEvent_t done = nullptr;     // recorded after the batch's copies back
  bool busy = false;
};
// A batch queued by rv_embed_submit whose results still sit in its slot.
struct AsyncBatch {
  int slot;
  int64_t ticket;
  float* dst;  // caller's rows for this batch
  int nb;
};

struct rv_ctx {
  rv_model_desc d{};
  int device = 0;
  rv::Act adt = rv::Act::kBf16;  // device storage dtype
  bool ln_fused = true;          // ModernBERT LayerNorms folded into the GEMMs (RV_LN_FUSED=0 turns off)
  bool gemm_pair = true;         // two-CTA GEMM tiles for 256-wide projections (RV_GEMM_2SM=0 turns off)
  std::mutex mu;
  std::string err;
  cudaStream_t stream = nullptr;
  unsigned int* d_err = nullptr;
  int64_t launches = 0;
  bool finalized = false;
  std::map<std::string, std::vector<float>> host_w;  // staged until rv_finalize

  // device weights
  float* tok_emb = nullptr;     // [vocab, hidden] f32
  float* emb_norm_w = nullptr;
  float* emb_norm_b = nullptr;  // ClassicBert
  float* final_norm = nullptr;  // ModernBERT
  float* pos_emb = nullptr;     // ClassicBert [max_position, hidden]
  float* type_emb = nullptr;    // ClassicBert [type_vocab, hidden]
  float* rope_cos[2] = {nullptr, nullptr};  // [0] global theta, [1] local theta; [max_pos, 32]
  float* rope_sin[2] = {nullptr, nullptr};
  std::vector<rv::LayerWeights> layers;

  // workspaces
  int64_t t_max = 0;
  int n_max = 0;
  void* x = nullptr;    // residual stream [t_max, hidden]
  void* hn = nullptr;   // normalised input of the next projection
  void* qkv = nullptr;  // [t_max, 3*hidden]
  void* cbuf = nullptr; // attention context [t_max, hidden]
  void* act = nullptr;  // MLP activation [t_max, intermediate]
  void* stats_a = nullptr;  // float2 LayerNorm partials [t_max, 4] of x after the attention block
  void* stats_b = nullptr;  // ... and after the MLP block
  int* ids_d = nullptr;
  int* pos_d = nullptr;
  int* meta_d = nullptr;  // cu_seqlens (n_max+1) then 64-query tile starts (n_max+1)
  int2* tiles_d = nullptr; // 128-query tile records of the tcgen05 attention (tiles_cap)
  int2* tiles_h = nullptr; // pinned staging of tiles_d
  int64_t tiles_cap = 0;
  float* out_d = nullptr; // [n_max, hidden]
  int* meta_h = nullptr;  // pinned staging of meta_d
  cudaEvent_t meta_evt = nullptr;
  CUtensorMap map_x, map_hn, map_c, map_act;
  // TMA-staged epilogue outputs: 32-row boxes, one per epilogue warp (x_out is the residual
  // stream, read and written by the residual epilogues).
  CUtensorMap map_qkv_out, map_act_out, map_x_out;
  bool tma_epi = true;                   // TMA-staged GEMM epilogues (RV_TMA_EPI=0 turns off)
  bool attn_tc = true;                   // tcgen05 attention (RV_ATTN_TC=0 turns off)
  // Columns of each of Q, K, V in qkv and of the attention context cbuf: hidden, or heads x 64
  // when head_dim 32 (BERT-small) is zero-padded to 64 per head for the tcgen05 attention.
  int attn_width = 0;

  std::vector<void*> allocations;

  // asynchronous path (rv_embed_submit / rv_embed_wait): two slots of pinned staging, batches in
  // flight in submission order, and the status of tickets not yet waited on.
  static constexpr int kAsyncSlots = 2;
  AsyncSlot aslots[kAsyncSlots];
  bool aslots_ready = false;
  std::deque<AsyncBatch> inflight;
  int next_slot = 0;
  int64_t next_ticket = 1;
  std::map<int64_t, int> ticket_rc;  // tickets submitted and not yet waited on -> status

  // per-kernel profiling (rv_set_profiling)
  bool profiling = false;
  struct Mark {
    int kind;
    cudaEvent_t a, b;
    double flops;
  };
  std::vector<Mark> marks;            // recorded, not yet read
  std::vector<cudaEvent_t> ev_pool;   // free events
  double prof_ms[RV_KIND_COUNT] = {0};
  int64_t prof_n[RV_KIND_COUNT] = {0};
  double prof_flops[RV_KIND_COUNT] = {0};
};
