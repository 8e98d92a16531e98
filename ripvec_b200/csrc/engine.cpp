// C ABI of the embedding backend: context lifetime, weight upload, varlen token-budget packing
// and the encoder forward passes (ModernBERT and ClassicBert) as sequences of sm_100a kernels.
//
// Forward passes follow crates/ripvec-core/src/backend/arch/modern_bert.rs:888-1117 (FP32
// branch :1043-1069 is the numerical reference) and backend/cpu.rs:237-515, :722-748.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <new>
#include <thread>
#include <vector>

#include "engine.h"
#include "tmap.h"

using rv::Act;
using rv::GemmArgs;
using rv::GemmEpi;

namespace rv {

uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return static_cast<uint16_t>((u >> 16) | 0x40);
  const uint32_t rounding = 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>((u + rounding) >> 16);
}

uint16_t f32_to_f16_bits(float f) {
  __half h = __float2half_rn(f);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

bool upload_converted(const float* host, int64_t n, Act act, void** dev, std::string* why) {
  std::vector<uint16_t> tmp(static_cast<size_t>(n));
  if (act == Act::kBf16)
    for (int64_t i = 0; i < n; ++i) tmp[i] = f32_to_bf16_bits(host[i]);
  else
    for (int64_t i = 0; i < n; ++i) tmp[i] = f32_to_f16_bits(host[i]);
  cudaError_t e = cudaMalloc(dev, static_cast<size_t>(n) * 2);
  if (e != cudaSuccess) {
    *why = std::string("cudaMalloc: ") + cudaGetErrorString(e);
    return false;
  }
  e = cudaMemcpy(*dev, tmp.data(), static_cast<size_t>(n) * 2, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    *why = std::string("cudaMemcpy: ") + cudaGetErrorString(e);
    return false;
  }
  return true;
}

bool upload_f32(const float* host, int64_t n, float** dev, std::string* why) {
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(dev), static_cast<size_t>(n) * 4);
  if (e != cudaSuccess) {
    *why = std::string("cudaMalloc: ") + cudaGetErrorString(e);
    return false;
  }
  e = cudaMemcpy(*dev, host, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    *why = std::string("cudaMemcpy: ") + cudaGetErrorString(e);
    return false;
  }
  return true;
}

}  // namespace rv

namespace {

int fail(rv_ctx* c, int code, const std::string& msg) {
  if (c) c->err = msg;
  return code;
}

#define RV_CUDA_TRY(ctx, expr)                                                        \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    if (_e != cudaSuccess)                                                            \
      return fail(ctx, RV_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

cudaEvent_t take_event(rv_ctx* c) {
  if (!c->ev_pool.empty()) {
    cudaEvent_t e = c->ev_pool.back();
    c->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Reads the recorded event pairs (the stream must have been synchronised) into the totals.
void collect_marks(rv_ctx* c) {
  for (auto& m : c->marks) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, m.a, m.b) == cudaSuccess) {
      c->prof_ms[m.kind] += ms;
      c->prof_n[m.kind] += 1;
      c->prof_flops[m.kind] += m.flops;
    }
    c->ev_pool.push_back(m.a);
    c->ev_pool.push_back(m.b);
  }
  c->marks.clear();
}

// Launch wrapper: counts kernels, optionally brackets them with events, and turns launch errors
// into status codes.
#define RV_LAUNCH_K(ctx, kind, flops, expr)                                           \
  do {                                                                                \
    cudaEvent_t _a = nullptr, _b = nullptr;                                           \
    if ((ctx)->profiling) {                                                           \
      _a = take_event(ctx);                                                           \
      _b = take_event(ctx);                                                           \
      cudaEventRecord(_a, (ctx)->stream);                                             \
    }                                                                                 \
    cudaError_t _e = (expr);                                                          \
    (ctx)->launches++;                                                                \
    if ((ctx)->profiling) {                                                           \
      cudaEventRecord(_b, (ctx)->stream);                                             \
      (ctx)->marks.push_back({(kind), _a, _b, double(flops)});                        \
    }                                                                                 \
    if (_e != cudaSuccess)                                                            \
      return fail(ctx, RV_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)
#define RV_LAUNCH(ctx, expr) RV_LAUNCH_K(ctx, RV_KIND_EMBED, 0, expr)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

bool is_modern(const rv_ctx* c) { return c->d.arch == RV_ARCH_MODERNBERT; }

std::string strip_prefix(const std::string& name) {
  static const char* prefixes[] = {"model.", "bert."};
  for (const char* p : prefixes) {
    const size_t n = std::strlen(p);
    if (name.compare(0, n, p) == 0) return name.substr(n);
  }
  return name;
}

// Expected element count of a named weight, or -1 if the name is not part of the model.
int64_t expected_numel(const rv_ctx* c, const std::string& name) {
  const int64_t H = c->d.hidden, I = c->d.intermediate, V = c->d.vocab;
  if (is_modern(c)) {
    if (name == "embeddings.tok_embeddings.weight") return V * H;
    if (name == "embeddings.norm.weight" || name == "final_norm.weight") return H;
    int li = -1;
    char rest[128] = {0};
    if (std::sscanf(name.c_str(), "layers.%d.%127s", &li, rest) == 2 && li >= 0 &&
        li < c->d.num_layers) {
      const std::string r(rest);
      if (r == "attn.Wqkv.weight") return 3 * H * H;
      if (r == "attn.Wo.weight") return H * H;
      if (r == "attn_norm.weight") return li == 0 ? -1 : H;
      if (r == "mlp.Wi.weight") return 2 * I * H;
      if (r == "mlp.Wo.weight") return H * I;
      if (r == "mlp_norm.weight") return H;
    }
    return -1;
  }
  if (name == "embeddings.word_embeddings.weight") return V * H;
  if (name == "embeddings.position_embeddings.weight") return int64_t(c->d.max_position) * H;
  if (name == "embeddings.token_type_embeddings.weight") return int64_t(c->d.type_vocab) * H;
  if (name == "embeddings.LayerNorm.weight" || name == "embeddings.LayerNorm.bias") return H;
  int li = -1;
  char rest[160] = {0};
  if (std::sscanf(name.c_str(), "encoder.layer.%d.%159s", &li, rest) == 2 && li >= 0 &&
      li < c->d.num_layers) {
    const std::string r(rest);
    if (r == "attention.self.query.weight" || r == "attention.self.key.weight" ||
        r == "attention.self.value.weight" || r == "attention.output.dense.weight")
      return H * H;
    if (r == "attention.self.query.bias" || r == "attention.self.key.bias" ||
        r == "attention.self.value.bias" || r == "attention.output.dense.bias" ||
        r == "attention.output.LayerNorm.weight" || r == "attention.output.LayerNorm.bias" ||
        r == "output.dense.bias" || r == "output.LayerNorm.weight" || r == "output.LayerNorm.bias")
      return H;
    if (r == "intermediate.dense.weight") return I * H;
    if (r == "intermediate.dense.bias") return I;
    if (r == "output.dense.weight") return H * I;
  }
  return -1;
}

void* dalloc(rv_ctx* c, size_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
  c->allocations.push_back(p);
  return p;
}

const std::vector<float>* get_w(rv_ctx* c, const std::string& name) {
  auto it = c->host_w.find(name);
  return it == c->host_w.end() ? nullptr : &it->second;
}

int need(rv_ctx* c, const std::string& name, const std::vector<float>** out) {
  *out = get_w(c, name);
  if (!*out) return fail(c, RV_E_NOT_READY, "missing weight: " + name);
  return RV_OK;
}

int up_f32(rv_ctx* c, const std::vector<float>& v, float** dev) {
  std::string why;
  if (!rv::upload_f32(v.data(), static_cast<int64_t>(v.size()), dev, &why))
    return fail(c, RV_E_NOMEM, why);
  c->allocations.push_back(*dev);
  return RV_OK;
}

int up_matrix(rv_ctx* c, const std::vector<float>& v, int rows, int cols, int bn,
              rv::DeviceMatrix* m) {
  std::string why;
  if (!rv::upload_converted(v.data(), static_cast<int64_t>(v.size()), c->adt, &m->ptr, &why))
    return fail(c, RV_E_NOMEM, why);
  c->allocations.push_back(m->ptr);
  m->rows = rows;
  m->cols = cols;
  m->bn = bn;
  if (!rv::make_tmap_2d_16bit(&m->tmap, m->ptr, c->adt == Act::kBf16, cols, rows,
                              uint64_t(cols) * 2, 64, bn, &why) ||
      !rv::make_tmap_2d_16bit(&m->tmap_half, m->ptr, c->adt == Act::kBf16, cols, rows,
                              uint64_t(cols) * 2, 64, 128, &why))
    return fail(c, RV_E_CUDA, why);
  return RV_OK;
}

// RoPE tables exactly as the reference builds them on the host in f32
// (backend/driver/cpu.rs:670-688): freq = pos / theta^(2d/head_dim), cos/sin in f32.
void build_rope(int max_pos, int head_dim, float theta, std::vector<float>* cs,
                std::vector<float>* sn) {
  const int half = head_dim / 2;
  cs->resize(size_t(max_pos) * half);
  sn->resize(size_t(max_pos) * half);
  for (int p = 0; p < max_pos; ++p)
    for (int d = 0; d < half; ++d) {
      const float freq = static_cast<float>(p) /
                         powf(theta, 2.0f * static_cast<float>(d) / static_cast<float>(head_dim));
      (*cs)[size_t(p) * half + d] = cosf(freq);
      (*sn)[size_t(p) * half + d] = sinf(freq);
    }
}

// Folds a LayerNorm gain into the following projection: W'[n,k] = W[n,k] * gamma[k] (f32, then the
// upload rounds to the device dtype).  Returns c_n = sum_k W'[n,k] over the rounded values, the
// column sums the LayerNorm-folding epilogues subtract (mu * c_n).
std::vector<float> fold_gamma(std::vector<float>* w, int rows, int cols, const std::vector<float>& gamma,
                              Act adt) {
  std::vector<float> cs(rows);
  for (int r = 0; r < rows; ++r) {
    double sum = 0.0;
    float* row = w->data() + size_t(r) * cols;
    for (int k = 0; k < cols; ++k) {
      row[k] *= gamma[k];
      float q;
      if (adt == Act::kBf16) {
        const uint32_t b = uint32_t(rv::f32_to_bf16_bits(row[k])) << 16;
        std::memcpy(&q, &b, 4);
      } else {
        const uint16_t h = rv::f32_to_f16_bits(row[k]);
        __half hv;
        std::memcpy(&hv, &h, 2);
        q = __half2float(hv);
      }
      sum += q;
    }
    cs[r] = static_cast<float>(sum);
  }
  return cs;
}

int finalize_modern(rv_ctx* c) {
  const int H = c->d.hidden, I = c->d.intermediate, L = c->d.num_layers;
  const std::vector<float>* w;
  int rc;
  if ((rc = need(c, "embeddings.tok_embeddings.weight", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->tok_emb))) return rc;
  if ((rc = need(c, "embeddings.norm.weight", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->emb_norm_w))) return rc;
  if ((rc = need(c, "final_norm.weight", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->final_norm))) return rc;
  c->layers.assign(L, rv::LayerWeights{});
  for (int i = 0; i < L; ++i) {
    const std::string p = "layers." + std::to_string(i) + ".";
    rv::LayerWeights& lw = c->layers[i];
    lw.is_global = (i % c->d.global_every_n) == 0;
    const std::vector<float>* attn_g = nullptr;
    const std::vector<float>* mlp_g = nullptr;
    if (i > 0) {
      if ((rc = need(c, p + "attn_norm.weight", &attn_g))) return rc;
      if ((rc = up_f32(c, *attn_g, &lw.attn_norm))) return rc;
    }
    if ((rc = need(c, p + "mlp_norm.weight", &mlp_g))) return rc;
    if ((rc = up_f32(c, *mlp_g, &lw.mlp_norm))) return rc;

    if ((rc = need(c, p + "attn.Wqkv.weight", &w))) return rc;
    if (c->ln_fused && attn_g) {
      std::vector<float> wq(*w);
      std::vector<float> cs = fold_gamma(&wq, 3 * H, H, *attn_g, c->adt);
      if ((rc = up_matrix(c, wq, 3 * H, H, 256, &lw.wqkv))) return rc;
      if ((rc = up_f32(c, cs, &lw.csum_qkv))) return rc;
    } else if ((rc = up_matrix(c, *w, 3 * H, H, 256, &lw.wqkv))) {
      return rc;
    }
    if ((rc = need(c, p + "attn.Wo.weight", &w))) return rc;
    if ((rc = up_matrix(c, *w, H, H, 256, &lw.wo))) return rc;
    if ((rc = need(c, p + "mlp.Wi.weight", &w))) return rc;
    // Interleave value / gate rows in 32-row blocks so that every 64-column accumulator group of
    // the Wi GEMM holds 32 value columns followed by the 32 matching gate columns.
    std::vector<float> wi(w->size());
    for (int r = 0; r < 2 * I; ++r) {
      const int g = r / 64, within = r % 64;
      const int src = within < 32 ? g * 32 + within : I + g * 32 + (within - 32);
      std::memcpy(&wi[size_t(r) * H], &(*w)[size_t(src) * H], sizeof(float) * H);
    }
    if (c->ln_fused) {
      std::vector<float> cs = fold_gamma(&wi, 2 * I, H, *mlp_g, c->adt);
      if ((rc = up_f32(c, cs, &lw.csum_wi))) return rc;
    }
    if ((rc = up_matrix(c, wi, 2 * I, H, 256, &lw.wi))) return rc;
    if ((rc = need(c, p + "mlp.Wo.weight", &w))) return rc;
    if ((rc = up_matrix(c, *w, H, I, 256, &lw.wo2))) return rc;
  }
  const int hd = H / c->d.num_heads;
  for (int g = 0; g < 2; ++g) {
    std::vector<float> cs, sn;
    build_rope(c->d.max_position, hd, g == 0 ? c->d.global_rope_theta : c->d.local_rope_theta, &cs,
               &sn);
    if ((rc = up_f32(c, cs, &c->rope_cos[g]))) return rc;
    if ((rc = up_f32(c, sn, &c->rope_sin[g]))) return rc;
  }
  return RV_OK;
}

int finalize_classic(rv_ctx* c) {
  const int H = c->d.hidden, I = c->d.intermediate, L = c->d.num_layers;
  const std::vector<float>* w;
  int rc;
  if ((rc = need(c, "embeddings.word_embeddings.weight", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->tok_emb))) return rc;
  if ((rc = need(c, "embeddings.position_embeddings.weight", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->pos_emb))) return rc;
  if ((rc = need(c, "embeddings.token_type_embeddings.weight", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->type_emb))) return rc;
  if ((rc = need(c, "embeddings.LayerNorm.weight", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->emb_norm_w))) return rc;
  if ((rc = need(c, "embeddings.LayerNorm.bias", &w))) return rc;
  if ((rc = up_f32(c, *w, &c->emb_norm_b))) return rc;
  c->layers.assign(L, rv::LayerWeights{});
  auto opt_f32 = [&](const std::string& name, float** dev) -> int {
    const std::vector<float>* b = get_w(c, name);
    if (!b) {
      *dev = nullptr;
      return RV_OK;
    }
    return up_f32(c, *b, dev);
  };
  for (int i = 0; i < L; ++i) {
    const std::string p = "encoder.layer." + std::to_string(i) + ".";
    rv::LayerWeights& lw = c->layers[i];
    const std::vector<float>*q, *k, *v;
    if ((rc = need(c, p + "attention.self.query.weight", &q))) return rc;
    if ((rc = need(c, p + "attention.self.key.weight", &k))) return rc;
    if ((rc = need(c, p + "attention.self.value.weight", &v))) return rc;
    // Rows Q, K, V concatenated (backend/cpu.rs:526-533); with a padded attention width, head h's
    // hd rows of each go to rows h * 64 .. h * 64 + hd - 1 of its block and the rest are zero.
    const int W = c->attn_width, heads = c->d.num_heads, hd = H / heads, hs = W / heads;
    std::vector<float> qkv(size_t(3) * W * H, 0.0f);
    const std::vector<float>* parts[3] = {q, k, v};
    for (int m = 0; m < 3; ++m)
      for (int r = 0; r < H; ++r)
        std::copy(parts[m]->begin() + size_t(r) * H, parts[m]->begin() + size_t(r + 1) * H,
                  qkv.begin() + (size_t(m) * W + size_t(r / hd) * hs + r % hd) * H);
    if ((rc = up_matrix(c, qkv, 3 * W, H, 128, &lw.wqkv))) return rc;
    const std::vector<float>*qb = get_w(c, p + "attention.self.query.bias"),
                      *kb = get_w(c, p + "attention.self.key.bias"),
                      *vb = get_w(c, p + "attention.self.value.bias");
    if (qb && kb && vb) {
      std::vector<float> b(size_t(3) * W, 0.0f);
      const std::vector<float>* bs[3] = {qb, kb, vb};
      for (int m = 0; m < 3; ++m)
        for (int r = 0; r < H; ++r) b[size_t(m) * W + size_t(r / hd) * hs + r % hd] = (*bs[m])[r];
      if ((rc = up_f32(c, b, &lw.bqkv))) return rc;
    }
    if ((rc = need(c, p + "attention.output.dense.weight", &w))) return rc;
    if (W == H) {
      if ((rc = up_matrix(c, *w, H, H, 128, &lw.wo))) return rc;
    } else {  // context columns padded like Q, K, V: zero weights for the pad columns
      std::vector<float> wo(size_t(H) * W, 0.0f);
      for (int r = 0; r < H; ++r)
        for (int col = 0; col < H; ++col) wo[size_t(r) * W + size_t(col / hd) * hs + col % hd] = (*w)[size_t(r) * H + col];
      if ((rc = up_matrix(c, wo, H, W, 128, &lw.wo))) return rc;
    }
    if ((rc = opt_f32(p + "attention.output.dense.bias", &lw.bo))) return rc;
    if ((rc = need(c, p + "attention.output.LayerNorm.weight", &w))) return rc;
    if ((rc = up_f32(c, *w, &lw.ln1_w))) return rc;
    if ((rc = need(c, p + "attention.output.LayerNorm.bias", &w))) return rc;
    if ((rc = up_f32(c, *w, &lw.ln1_b))) return rc;
    if ((rc = need(c, p + "intermediate.dense.weight", &w))) return rc;
    if ((rc = up_matrix(c, *w, I, H, (I % 256 == 0) ? 256 : 128, &lw.wi))) return rc;
    if ((rc = opt_f32(p + "intermediate.dense.bias", &lw.b1))) return rc;
    if ((rc = need(c, p + "output.dense.weight", &w))) return rc;
    if ((rc = up_matrix(c, *w, H, I, 128, &lw.wo2))) return rc;
    if ((rc = opt_f32(p + "output.dense.bias", &lw.b2))) return rc;
    if ((rc = need(c, p + "output.LayerNorm.weight", &w))) return rc;
    if ((rc = up_f32(c, *w, &lw.ln2_w))) return rc;
    if ((rc = need(c, p + "output.LayerNorm.bias", &w))) return rc;
    if ((rc = up_f32(c, *w, &lw.ln2_b))) return rc;
  }
  return RV_OK;
}

int alloc_workspaces(rv_ctx* c) {
  const int64_t T = c->t_max;
  const int H = c->d.hidden, I = c->d.intermediate;
  const size_t es = 2;
  c->x = dalloc(c, size_t(T) * H * es);
  c->hn = dalloc(c, size_t(T) * H * es);
  const int W = c->attn_width;
  c->qkv = dalloc(c, size_t(T) * 3 * W * es);
  c->cbuf = dalloc(c, size_t(T) * W * es);
  c->act = dalloc(c, size_t(T) * I * es);
  if (is_modern(c) && c->ln_fused) {
    c->stats_a = dalloc(c, size_t(T) * 4 * sizeof(float2));
    c->stats_b = dalloc(c, size_t(T) * 4 * sizeof(float2));
    if (!c->stats_a || !c->stats_b) return fail(c, RV_E_NOMEM, "workspace allocation failed");
  }
  c->ids_d = static_cast<int*>(dalloc(c, size_t(T) * 4));
  c->pos_d = static_cast<int*>(dalloc(c, size_t(T) * 4));
  c->meta_d = static_cast<int*>(dalloc(c, size_t(2) * (c->n_max + 1) * 4));
  c->out_d = static_cast<float*>(dalloc(c, size_t(c->n_max) * H * 4));
  // A batch has at most t_max / 128 + n_max 128-query tiles.
  c->tiles_cap = c->t_max / 128 + c->n_max + 1;
  c->tiles_d = static_cast<int2*>(dalloc(c, size_t(c->tiles_cap) * sizeof(int2)));
  if (!c->x || !c->hn || !c->qkv || !c->cbuf || !c->act || !c->ids_d || !c->pos_d || !c->meta_d ||
      !c->out_d || !c->tiles_d)
    return fail(c, RV_E_NOMEM, "workspace allocation failed");
  if (cudaMallocHost(reinterpret_cast<void**>(&c->meta_h), size_t(2) * (c->n_max + 1) * 4) !=
          cudaSuccess ||
      cudaMallocHost(reinterpret_cast<void**>(&c->tiles_h), size_t(c->tiles_cap) * sizeof(int2)) !=
          cudaSuccess)
    return fail(c, RV_E_NOMEM, "pinned staging allocation failed");
  if (cudaEventCreateWithFlags(&c->meta_evt, cudaEventDisableTiming) != cudaSuccess)
    return fail(c, RV_E_CUDA, "event creation failed");
  std::string why;
  const bool bf = c->adt == Act::kBf16;
  if (!rv::make_tmap_2d_16bit(&c->map_x, c->x, bf, H, T, uint64_t(H) * 2, 64, 128, &why) ||
      !rv::make_tmap_2d_16bit(&c->map_hn, c->hn, bf, H, T, uint64_t(H) * 2, 64, 128, &why) ||
      !rv::make_tmap_2d_16bit(&c->map_c, c->cbuf, bf, c->attn_width, T, uint64_t(c->attn_width) * 2, 64, 128,
                              &why) ||
      !rv::make_tmap_2d_16bit(&c->map_act, c->act, bf, I, T, uint64_t(I) * 2, 64, 128, &why) ||
      !rv::make_tmap_2d_16bit(&c->map_qkv_out, c->qkv, bf, 3 * H, T, uint64_t(3 * H) * 2, 64, 32, &why) ||
      !rv::make_tmap_2d_16bit(&c->map_x_out, c->x, bf, H, T, uint64_t(H) * 2, 64, 32, &why) ||
      !rv::make_tmap_2d_16bit(&c->map_act_out, c->act, bf, I, T, uint64_t(I) * 2, 32, 32, &why, 64))
    return fail(c, RV_E_CUDA, why);
  return RV_OK;
}

int gemm(rv_ctx* c, const CUtensorMap& A, const rv::DeviceMatrix& B, int M, GemmEpi epi, void* out,
         int ldc, const float* bias = nullptr, int rope_cols = 0, const float* cs = nullptr,
         const float* sn = nullptr, void* stats = nullptr, const float* csum = nullptr) {
  GemmArgs a{};
  a.tmA = &A;
  a.pair = c->gemm_pair && B.bn == 256 && B.rows % 256 == 0;
  a.tmB = a.pair ? &B.tmap_half : &B.tmap;
  a.M = M;
  a.N = B.rows;
  a.K = B.cols;
  a.bn = B.bn;
  a.epi = epi;
  a.c = out;
  a.ldc = ldc;
  a.bias = bias;
  a.rope_cols = rope_cols;
  a.pos = c->pos_d;
  a.cos_t = cs;
  a.sin_t = sn;
  a.stats = stats;
  a.stats_ld = 4;
  a.stats_n = c->d.hidden / 256;
  a.csum = csum;
  a.eps = c->d.norm_eps;
  if (a.pair && c->tma_epi) {
    if (epi == GemmEpi::kQkvRope || epi == GemmEpi::kNormQkvRope) a.tmC = &c->map_qkv_out;
    else if (epi == GemmEpi::kResidualStats) a.tmC = &c->map_x_out;
    else if (epi == GemmEpi::kNormGeglu) a.tmC = &c->map_act_out;
  }
  RV_LAUNCH_K(c, RV_KIND_GEMM, 2.0 * double(M) * a.N * a.K, rv::gemm_tc(c->adt, a, c->d_err, c->stream));
  return RV_OK;
}

// One forward over a packed batch already on the device: ids (T tokens), meta_d holding
// cu_seqlens and q-tile starts for n sequences.  Writes f32 embeddings to out [n, hidden].
int forward(rv_ctx* c, const int* ids, int T, int n, int total_q_tiles, int total_q_tiles128,
            double pairs_global, double pairs_local, float* out) {
  const int H = c->d.hidden, heads = c->d.num_heads, hd = H / heads;
  const int* cu = c->meta_d;
  const int* qts = c->meta_d + (n + 1);
  cudaStream_t st = c->stream;
  RV_LAUNCH_K(c, RV_KIND_EMBED, 0, rv::build_positions(cu, n, T, c->pos_d, st));
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  auto attend = [&](int window_half) {
    return c->attn_tc && (hd == 64 || c->attn_width == 64 * heads)
               ? rv::attention_varlen_tc(c->adt, c->qkv, c->cbuf, T, c->tiles_d, total_q_tiles128, heads,
                                         window_half, scale, c->d_err, st)
               : rv::attention_varlen(c->adt, c->qkv, c->cbuf, cu, qts, n, total_q_tiles, heads, hd,
                                      window_half, scale, st);
  };
  if (is_modern(c)) {
    RV_LAUNCH_K(c, RV_KIND_EMBED, 0, rv::embed_ln(c->adt, ids, T, c->tok_emb, c->d.vocab, c->emb_norm_w, nullptr,
                              nullptr, nullptr, nullptr, H, c->d.norm_eps, c->x, c->d_err, st));
    for (int l = 0; l < c->d.num_layers; ++l) {
      const rv::LayerWeights& lw = c->layers[l];
      const int g = lw.is_global ? 0 : 1;
      const int wh = lw.is_global ? -1 : c->d.local_window / 2;
      int rc;
      if (c->ln_fused) {
        // LayerNorms folded into the projections: QKV / Wi read the raw residual rows and the
        // row statistics the previous residual epilogue wrote (stats_b after the MLP block,
        // stats_a after the attention block); layer 0 has no attention LayerNorm.
        if (l == 0) {
          if ((rc = gemm(c, c->map_x, lw.wqkv, T, GemmEpi::kQkvRope, c->qkv, 3 * H, nullptr, 2 * H,
                         c->rope_cos[g], c->rope_sin[g])))
            return rc;
        } else if ((rc = gemm(c, c->map_x, lw.wqkv, T, GemmEpi::kNormQkvRope, c->qkv, 3 * H, nullptr, 2 * H,
                              c->rope_cos[g], c->rope_sin[g], c->stats_b, lw.csum_qkv))) {
          return rc;
        }
        RV_LAUNCH_K(c, RV_KIND_ATTENTION, 4.0 * H * (lw.is_global ? pairs_global : pairs_local),
                    attend(wh));
        if ((rc = gemm(c, c->map_c, lw.wo, T, GemmEpi::kResidualStats, c->x, H, nullptr, 0, nullptr, nullptr,
                       c->stats_a)))
          return rc;
        if ((rc = gemm(c, c->map_x, lw.wi, T, GemmEpi::kNormGeglu, c->act, c->d.intermediate, nullptr, 0, nullptr,
                       nullptr, c->stats_a, lw.csum_wi)))
          return rc;
        if ((rc = gemm(c, c->map_act, lw.wo2, T, GemmEpi::kResidualStats, c->x, H, nullptr, 0, nullptr, nullptr,
                       c->stats_b)))
          return rc;
        continue;
      }
      if (l > 0)
        RV_LAUNCH_K(c, RV_KIND_NORM, 0, rv::layernorm(c->adt, c->x, c->hn, T, H, lw.attn_norm, nullptr,
                                                      c->d.norm_eps, st));
      if ((rc = gemm(c, l == 0 ? c->map_x : c->map_hn, lw.wqkv, T, GemmEpi::kQkvRope, c->qkv,
                     3 * H, nullptr, 2 * H, c->rope_cos[g], c->rope_sin[g])))
        return rc;
      RV_LAUNCH_K(c, RV_KIND_ATTENTION, 4.0 * H * (lw.is_global ? pairs_global : pairs_local),
                  attend(wh));
      if ((rc = gemm(c, c->map_c, lw.wo, T, GemmEpi::kResidual, c->x, H))) return rc;
      RV_LAUNCH_K(c, RV_KIND_NORM, 0, rv::layernorm(c->adt, c->x, c->hn, T, H, lw.mlp_norm, nullptr,
                                                    c->d.norm_eps, st));
      if ((rc = gemm(c, c->map_hn, lw.wi, T, GemmEpi::kGeglu, c->act, c->d.intermediate)))
        return rc;
      if ((rc = gemm(c, c->map_act, lw.wo2, T, GemmEpi::kResidual, c->x, H))) return rc;
    }
    RV_LAUNCH_K(c, RV_KIND_POOL, 0, rv::pool_l2(c->adt, c->x, cu, n, H, 0, c->final_norm, c->d.norm_eps, 0.0f, out,
                             st));
  } else {
    RV_LAUNCH_K(c, RV_KIND_EMBED, 0, rv::embed_ln(c->adt, ids, T, c->tok_emb, c->d.vocab, c->emb_norm_w,
                              c->emb_norm_b, c->pos_emb, c->pos_d, c->type_emb, H, c->d.norm_eps,
                              c->x, c->d_err, st));
    for (int l = 0; l < c->d.num_layers; ++l) {
      const rv::LayerWeights& lw = c->layers[l];
      int rc;
      if ((rc = gemm(c, c->map_x, lw.wqkv, T, GemmEpi::kBias, c->qkv, 3 * c->attn_width, lw.bqkv))) return rc;
      RV_LAUNCH_K(c, RV_KIND_ATTENTION, 4.0 * H * pairs_global,
                  attend(-1));
      if ((rc = gemm(c, c->map_c, lw.wo, T, GemmEpi::kResidual, c->x, H, lw.bo))) return rc;
      RV_LAUNCH_K(c, RV_KIND_NORM, 0, rv::layernorm(c->adt, c->x, c->x, T, H, lw.ln1_w, lw.ln1_b, c->d.norm_eps, st));
      if ((rc = gemm(c, c->map_x, lw.wi, T, GemmEpi::kBiasGelu, c->act, c->d.intermediate, lw.b1)))
        return rc;
      if ((rc = gemm(c, c->map_act, lw.wo2, T, GemmEpi::kResidual, c->x, H, lw.b2))) return rc;
      RV_LAUNCH_K(c, RV_KIND_NORM, 0, rv::layernorm(c->adt, c->x, c->x, T, H, lw.ln2_w, lw.ln2_b, c->d.norm_eps, st));
    }
    RV_LAUNCH_K(c, RV_KIND_POOL, 0, rv::pool_l2(c->adt, c->x, cu, n, H, c->d.pooling == RV_POOL_CLS ? 2 : 1, nullptr,
                             c->d.norm_eps, 1e-12f, out, st));
  }
  return RV_OK;
}

int check_device_error(rv_ctx* c) {
  unsigned int h = 0;
  RV_CUDA_TRY(c, cudaMemcpyAsync(&h, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream));
  RV_CUDA_TRY(c, cudaStreamSynchronize(c->stream));
  if (h) {
    cudaMemsetAsync(c->d_err, 0, 4, c->stream);
    cudaStreamSynchronize(c->stream);
    std::string m = "device error flags 0x" + [&] {
      char b[16];
      std::snprintf(b, sizeof b, "%x", h);
      return std::string(b);
    }();
    if (h & rv::kErrWaitTimeout) m += " (pipeline wait expired)";
    if (h & rv::kErrBadShape) m += " (token id out of range)";
    return fail(c, RV_E_DEVICE, m);
  }
  return RV_OK;
}

int validate_cu(rv_ctx* c, const int32_t* cu, int32_t n) {
  if (cu[0] != 0) return fail(c, RV_E_INVALID, "cu_seqlens[0] must be 0");
  for (int32_t b = 0; b < n; ++b) {
    const int64_t len = int64_t(cu[b + 1]) - cu[b];
    if (len < 0) return fail(c, RV_E_INVALID, "cu_seqlens must be non-decreasing");
    if (len > c->d.max_position)
      return fail(c, RV_E_INVALID,
                  "sequence " + std::to_string(b) + " has " + std::to_string(len) +
                      " tokens; the model supports at most " + std::to_string(c->d.max_position));
  }
  return RV_OK;
}

// Runs the packed batches covering sequences [0, n).  ids_src(b0, tokens) returns the device
// pointer of the ids of the batch starting at sequence b0 (copying them first when needed);
// out_dst(b0, nb, f32 src) moves the batch's embeddings to their destination.
//
// Batch rule (shared with the asynchronous path): consecutive sequences from b0 until the next
// one would pass t_max tokens or n_max sequences.
int32_t batch_end(const rv_ctx* c, const int32_t* cu, int32_t n, int32_t b0, int64_t* tokens) {
  int32_t b1 = b0;
  int64_t t = 0;
  while (b1 < n && (b1 - b0) < c->n_max) {
    const int64_t len = int64_t(cu[b1 + 1]) - cu[b1];
    if (t + len > c->t_max) break;
    t += len;
    ++b1;
  }
  *tokens = t;
  return b1;
}

// Fills the batch's metadata staging (cu_seqlens and the 64-query tile prefix into mh, the
// 128-query attention tile records into th) and counts its visible query-key pairs.
struct BatchMeta {
  int q = 0;            // 64-query tiles
  int n_tiles128 = 0;   // 128-query attention tiles (-1: a sequence too long for them)
  double pg = 0.0;      // visible query-key pairs, global layers
  double pl = 0.0;      // ... sliding-window layers
};
BatchMeta fill_batch_meta(const rv_ctx* c, const int32_t* cu, int32_t b0, int nb, int* mh, int2* th) {
  BatchMeta m;
  const int64_t w = c->d.local_window / 2;
  for (int i = 0; i <= nb; ++i) {
    mh[i] = cu[b0 + i] - cu[b0];
    mh[nb + 1 + i] = m.q;
    if (i < nb) {
      const int64_t len = cu[b0 + i + 1] - cu[b0 + i];
      m.q += static_cast<int>((len + 63) / 64);
      m.pg += double(len) * double(len);
      const int64_t k = std::min<int64_t>(w, len > 0 ? len - 1 : 0);
      m.pl += double(len) + 2.0 * (double(k) * len - double(k) * (k + 1) / 2.0);
    }
  }
  m.n_tiles128 = rv::fill_attention_tiles(mh, nb, th);
  return m;
}

// Enqueues the metadata copies of one batch from the given pinned staging.
int upload_meta(rv_ctx* c, const int* mh, const int2* th, int nb, const BatchMeta& m) {
  if (m.n_tiles128 < 0) return fail(c, RV_E_INVALID, "sequence too long for the attention tiles");
  RV_CUDA_TRY(c, cudaMemcpyAsync(c->meta_d, mh, sizeof(int) * 2 * (nb + 1), cudaMemcpyHostToDevice, c->stream));
  if (m.n_tiles128 > 0)
    RV_CUDA_TRY(c, cudaMemcpyAsync(c->tiles_d, th, sizeof(int2) * m.n_tiles128, cudaMemcpyHostToDevice,
                                   c->stream));
  return RV_OK;
}

template <class IdsFn, class OutFn>
int run_batches(rv_ctx* c, const int32_t* cu, int32_t n, IdsFn ids_src, OutFn out_dst) {
  int32_t b0 = 0;
  bool first = true;
  while (b0 < n) {
    int64_t tokens = 0;
    const int32_t b1 = batch_end(c, cu, n, b0, &tokens);
    const int nb = b1 - b0;
    // Staging buffer reuse: the previous batch's metadata copy must have executed.
    if (!first) RV_CUDA_TRY(c, cudaEventSynchronize(c->meta_evt));
    first = false;
    const BatchMeta m = fill_batch_meta(c, cu, b0, nb, c->meta_h, c->tiles_h);
    int rc = upload_meta(c, c->meta_h, c->tiles_h, nb, m);
    if (rc) return rc;
    RV_CUDA_TRY(c, cudaEventRecord(c->meta_evt, c->stream));
    const int* ids = ids_src(b0, static_cast<int>(tokens));
    if (!ids) return RV_E_CUDA;
    rc = forward(c, ids, static_cast<int>(tokens), nb, m.q, m.n_tiles128, m.pg, m.pl, c->out_d);
    if (rc) return rc;
    if ((rc = out_dst(b0, nb, c->out_d))) return rc;
    b0 = b1;
  }
  return RV_OK;
}

// ---------------------------------------------------------------- asynchronous path
int async_init(rv_ctx* c) {
  if (c->aslots_ready) return RV_OK;
  for (AsyncSlot& a : c->aslots) {
    if (cudaMallocHost(reinterpret_cast<void**>(&a.ids_h), size_t(c->t_max) * 4) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&a.meta_h), size_t(2) * (c->n_max + 1) * 4) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&a.tiles_h), size_t(c->tiles_cap) * sizeof(int2)) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void**>(&a.err_h), 4) != cudaSuccess ||
        cudaEventCreateWithFlags(&a.done, cudaEventDisableTiming) != cudaSuccess)
      return fail(c, RV_E_NOMEM, "pinned staging for the asynchronous path could not be allocated");
  }
  c->aslots_ready = true;
  return RV_OK;
}

void async_release(rv_ctx* c) {
  for (AsyncSlot& a : c->aslots) {
    if (a.ids_h) cudaFreeHost(a.ids_h);
    if (a.meta_h) cudaFreeHost(a.meta_h);
    if (a.tiles_h) cudaFreeHost(a.tiles_h);
    if (a.out_h) cudaFreeHost(a.out_h);
    if (a.err_h) cudaFreeHost(a.err_h);
    if (a.done) cudaEventDestroy(a.done);
    a = AsyncSlot{};
  }
  c->aslots_ready = false;
}

// Completes the oldest batch in flight: waits for its copies back, then moves its embeddings from
// the slot's pinned staging into the caller's rows (or records the device error of its ticket).
int async_finish_front(rv_ctx* c) {
  const AsyncBatch b = c->inflight.front();
  c->inflight.pop_front();
  AsyncSlot& a = c->aslots[b.slot];
  a.busy = false;
  int rc = RV_OK;
  const cudaError_t e = cudaEventSynchronize(a.done);
  if (e != cudaSuccess) {
    rc = fail(c, RV_E_CUDA, std::string("asynchronous batch: ") + cudaGetErrorString(e));
  } else if (*a.err_h) {
    std::string m = "device error flags " + std::to_string(*a.err_h);
    if (*a.err_h & rv::kErrWaitTimeout) m += " (pipeline wait expired)";
    if (*a.err_h & rv::kErrBadShape) m += " (token id out of range)";
    rc = fail(c, RV_E_DEVICE, m);
  } else {
    std::memcpy(b.dst, a.out_h, sizeof(float) * size_t(b.nb) * c->d.hidden);
  }
  auto it = c->ticket_rc.find(b.ticket);
  if (it != c->ticket_rc.end() && it->second == RV_OK) it->second = rc;
  return rc;
}

}  // namespace

extern "C" {

int rv_create(const rv_model_desc* desc, int device, rv_ctx** out) {
  if (!desc || !out) return RV_E_INVALID;
  *out = nullptr;
  const rv_model_desc& d = *desc;
  if (d.arch != RV_ARCH_MODERNBERT && d.arch != RV_ARCH_CLASSICBERT) return RV_E_INVALID;
  if (d.dtype != RV_DTYPE_BF16 && d.dtype != RV_DTYPE_F16) return RV_E_INVALID;
  if (d.hidden <= 0 || d.hidden > 768 || d.hidden % 64 != 0 || d.num_heads <= 0 ||
      d.hidden % d.num_heads != 0 || d.num_layers <= 0 || d.vocab <= 0 || d.max_position <= 0 ||
      d.intermediate <= 0 || d.intermediate % 64 != 0)
    return RV_E_INVALID;
  const int hd = d.hidden / d.num_heads;
  if (d.arch == RV_ARCH_MODERNBERT) {
    if (hd != 64 || d.global_every_n <= 0 || d.local_window < 0 || (3 * d.hidden) % 256 != 0 ||
        d.hidden % 256 != 0 || (2 * d.intermediate) % 256 != 0)
      return RV_E_INVALID;
  } else {
    if (hd != 32 && hd != 64) return RV_E_INVALID;
    if ((3 * d.hidden) % 128 != 0 || d.hidden % 128 != 0 || d.intermediate % 128 != 0 ||
        d.type_vocab <= 0)
      return RV_E_INVALID;
  }
  std::unique_ptr<rv_ctx> c(new (std::nothrow) rv_ctx());
  if (!c) return RV_E_NOMEM;
  c->d = d;
  c->device = device;
  c->adt = d.dtype == RV_DTYPE_BF16 ? Act::kBf16 : Act::kF16;
  if (const char* e = std::getenv("RV_GEMM_2SM")) c->gemm_pair = std::strcmp(e, "0") != 0;
  if (const char* e = std::getenv("RV_LN_FUSED")) c->ln_fused = std::strcmp(e, "0") != 0;
  if (const char* e = std::getenv("RV_TMA_EPI")) c->tma_epi = std::strcmp(e, "0") != 0;
  if (const char* e = std::getenv("RV_ATTN_TC")) c->attn_tc = std::strcmp(e, "0") != 0;
  c->t_max = d.max_batch_tokens > 0 ? d.max_batch_tokens : 262144;
  if (c->t_max < d.max_position) c->t_max = d.max_position;
  c->n_max = 65536;
  // The tcgen05 attention addresses the context with 32-bit element offsets.
  if (c->t_max * int64_t(d.hidden) > INT32_MAX) c->attn_tc = false;
  // head_dim 32: Q, K, V and the context are laid out with 64 columns per head (32 zeros), so the
  // tcgen05 head_dim-64 kernel computes the same scores and context.
  c->attn_width = d.hidden;
  if (c->attn_tc && d.num_heads > 0 && d.hidden == 32 * d.num_heads) {
    c->attn_width = 64 * d.num_heads;
    if (c->t_max * int64_t(c->attn_width) > INT32_MAX) {
      c->attn_tc = false;
      c->attn_width = d.hidden;
    }
  }
  if (cudaSetDevice(device) != cudaSuccess) return RV_E_CUDA;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) return RV_E_CUDA;
  c->d_err = static_cast<unsigned int*>(dalloc(c.get(), 4));
  if (!c->d_err || cudaMemset(c->d_err, 0, 4) != cudaSuccess) return RV_E_NOMEM;
  *out = c.release();
  return RV_OK;
}

void rv_destroy(rv_ctx* c) {
  if (!c) return;
  {
    DeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (void* p : c->allocations) cudaFree(p);
    if (c->meta_h) cudaFreeHost(c->meta_h);
    if (c->tiles_h) cudaFreeHost(c->tiles_h);
    if (c->meta_evt) cudaEventDestroy(c->meta_evt);
    async_release(c);
    for (auto& m : c->marks) {
      cudaEventDestroy(m.a);
      cudaEventDestroy(m.b);
    }
    for (cudaEvent_t e : c->ev_pool) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
  }
  delete c;
}

int rv_set_weight(rv_ctx* c, const char* name, const float* host, int64_t numel) {
  if (!c || !name || (!host && numel > 0)) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  if (c->finalized) return fail(c, RV_E_INVALID, "model already finalised");
  const std::string n = strip_prefix(name);
  const int64_t want = expected_numel(c, n);
  if (want < 0) return fail(c, RV_E_INVALID, "unknown weight name for this model: " + n);
  if (want != numel)
    return fail(c, RV_E_INVALID, "weight " + n + " has " + std::to_string(numel) +
                                     " elements, expected " + std::to_string(want));
  c->host_w[n].assign(host, host + numel);
  return RV_OK;
}

int rv_finalize(rv_ctx* c) {
  if (!c) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  if (c->finalized) return RV_OK;
  DeviceGuard g(c->device);
  int rc = is_modern(c) ? finalize_modern(c) : finalize_classic(c);
  if (rc) return rc;
  if ((rc = alloc_workspaces(c))) return rc;
  c->host_w.clear();
  c->finalized = true;
  return RV_OK;
}

int rv_embed_varlen(rv_ctx* c, const int32_t* ids, const int32_t* cu, int32_t n, float* out_host) {
  if (!c) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  if (n < 0 || (n > 0 && (!cu || !out_host))) return fail(c, RV_E_INVALID, "null argument");
  if (n == 0) return RV_OK;
  if (!c->finalized) return fail(c, RV_E_NOT_READY, "rv_finalize has not been called");
  int rc = validate_cu(c, cu, n);
  if (rc) return rc;
  const int64_t total = cu[n];
  if (total > 0 && !ids) return fail(c, RV_E_INVALID, "null ids");
  for (int64_t t = 0; t < total; ++t)
    if (ids[t] < 0 || ids[t] >= c->d.vocab)
      return fail(c, RV_E_INVALID, "token id " + std::to_string(ids[t]) + " at position " +
                                       std::to_string(t) + " is outside the vocabulary");
  DeviceGuard g(c->device);
  const int H = c->d.hidden;
  rc = run_batches(
      c, cu, n,
      [&](int32_t b0, int tokens) -> const int* {
        if (tokens > 0 &&
            cudaMemcpyAsync(c->ids_d, ids + cu[b0], sizeof(int) * size_t(tokens),
                            cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
          c->err = "ids upload failed";
          return nullptr;
        }
        return c->ids_d;
      },
      [&](int32_t b0, int nb, const float* src) -> int {
        RV_CUDA_TRY(c, cudaMemcpyAsync(out_host + size_t(b0) * H, src, sizeof(float) * size_t(nb) * H,
                                       cudaMemcpyDeviceToHost, c->stream));
        // The next batch overwrites out_d: wait for this copy (the device work of the next batch
        // is queued behind it anyway).
        RV_CUDA_TRY(c, cudaStreamSynchronize(c->stream));
        return RV_OK;
      });
  if (rc) return rc;
  rc = check_device_error(c);
  collect_marks(c);
  return rc;
}

int rv_embed_varlen_device(rv_ctx* c, const int32_t* ids_dev, const int32_t* cu, int32_t n,
                           void* out_dev, int32_t out_dtype, void* stream) {
  if (!c) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  if (n < 0 || (n > 0 && (!cu || !out_dev))) return fail(c, RV_E_INVALID, "null argument");
  if (out_dtype != RV_DTYPE_F32 && out_dtype != RV_DTYPE_BF16 && out_dtype != RV_DTYPE_F16)
    return fail(c, RV_E_INVALID, "unsupported output dtype");
  if (n == 0) return RV_OK;
  if (!c->finalized) return fail(c, RV_E_NOT_READY, "rv_finalize has not been called");
  int rc = validate_cu(c, cu, n);
  if (rc) return rc;
  DeviceGuard g(c->device);
  cudaStream_t user = static_cast<cudaStream_t>(stream);
  cudaEvent_t ev = nullptr;
  if (user) {  // order our stream after the caller's work on its stream
    RV_CUDA_TRY(c, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    RV_CUDA_TRY(c, cudaEventRecord(ev, user));
    RV_CUDA_TRY(c, cudaStreamWaitEvent(c->stream, ev, 0));
  }
  const int H = c->d.hidden;
  rc = run_batches(
      c, cu, n, [&](int32_t b0, int) -> const int* { return ids_dev + cu[b0]; },
      [&](int32_t b0, int nb, const float* src) -> int {
        if (out_dtype == RV_DTYPE_F32) {
          RV_CUDA_TRY(c, cudaMemcpyAsync(static_cast<float*>(out_dev) + size_t(b0) * H, src,
                                         sizeof(float) * size_t(nb) * H, cudaMemcpyDeviceToDevice,
                                         c->stream));
        } else {
          RV_LAUNCH(c, rv::convert_f32(out_dtype == RV_DTYPE_BF16 ? Act::kBf16 : Act::kF16, src,
                                       static_cast<uint16_t*>(out_dev) + size_t(b0) * H,
                                       int64_t(nb) * H, c->stream));
        }
        return RV_OK;
      });
  if (rc) {
    if (ev) cudaEventDestroy(ev);
    return rc;
  }
  if (user) {  // the caller's stream waits for the embeddings
    RV_CUDA_TRY(c, cudaEventRecord(ev, c->stream));
    RV_CUDA_TRY(c, cudaStreamWaitEvent(user, ev, 0));
    cudaEventDestroy(ev);
  }
  rc = check_device_error(c);
  collect_marks(c);
  return rc;
}

int rv_embed_submit(rv_ctx* c, const int32_t* ids, const int32_t* cu, int32_t n, float* out_host,
                    int64_t* ticket) {
  if (!c) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  if (!ticket || n < 0 || (n > 0 && (!cu || !out_host))) return fail(c, RV_E_INVALID, "null argument");
  *ticket = 0;
  if (!c->finalized) return fail(c, RV_E_NOT_READY, "rv_finalize has not been called");
  int rc = RV_OK;
  if (n > 0) {
    if ((rc = validate_cu(c, cu, n))) return rc;
    const int64_t total = cu[n];
    if (total > 0 && !ids) return fail(c, RV_E_INVALID, "null ids");
    for (int64_t t = 0; t < total; ++t)
      if (ids[t] < 0 || ids[t] >= c->d.vocab)
        return fail(c, RV_E_INVALID, "token id " + std::to_string(ids[t]) + " at position " + std::to_string(t) +
                                         " is outside the vocabulary");
  }
  DeviceGuard g(c->device);
  if ((rc = async_init(c))) return rc;
  const int64_t t = c->next_ticket++;
  c->ticket_rc[t] = RV_OK;
  const int H = c->d.hidden;
  int32_t b0 = 0;
  while (b0 < n && rc == RV_OK) {
    int64_t tokens = 0;
    const int32_t b1 = batch_end(c, cu, n, b0, &tokens);
    const int nb = b1 - b0;
    // A slot is reused once its previous batch has been moved to its caller (the bounded ring:
    // at most kAsyncSlots batches are in flight).
    const int si = c->next_slot;
    AsyncSlot& a = c->aslots[si];
    while (a.busy && !c->inflight.empty()) async_finish_front(c);
    const size_t need = size_t(nb) * H;
    if (a.out_cap < need) {
      if (a.out_h) cudaFreeHost(a.out_h);
      a.out_h = nullptr;
      a.out_cap = 0;
      if (cudaMallocHost(reinterpret_cast<void**>(&a.out_h), need * sizeof(float)) != cudaSuccess) {
        rc = fail(c, RV_E_NOMEM, "pinned output staging could not be allocated");
        break;
      }
      a.out_cap = need;
    }
    const BatchMeta m = fill_batch_meta(c, cu, b0, nb, a.meta_h, a.tiles_h);
    if ((rc = upload_meta(c, a.meta_h, a.tiles_h, nb, m))) break;
    if (tokens > 0) {
      std::memcpy(a.ids_h, ids + cu[b0], sizeof(int32_t) * size_t(tokens));
      if (cudaMemcpyAsync(c->ids_d, a.ids_h, sizeof(int32_t) * size_t(tokens), cudaMemcpyHostToDevice,
                          c->stream) != cudaSuccess) {
        rc = fail(c, RV_E_CUDA, "ids upload failed");
        break;
      }
    }
    if ((rc = forward(c, c->ids_d, static_cast<int>(tokens), nb, m.q, m.n_tiles128, m.pg, m.pl, c->out_d))) break;
    if (cudaMemcpyAsync(a.out_h, c->out_d, sizeof(float) * need, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(a.err_h, c->d_err, 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
        cudaMemsetAsync(c->d_err, 0, 4, c->stream) != cudaSuccess ||
        cudaEventRecord(a.done, c->stream) != cudaSuccess) {
      rc = fail(c, RV_E_CUDA, "asynchronous batch could not be queued");
      break;
    }
    a.busy = true;
    c->inflight.push_back(AsyncBatch{si, t, out_host + size_t(b0) * H, nb});
    c->next_slot = (si + 1) % rv_ctx::kAsyncSlots;
    b0 = b1;
  }
  if (rc != RV_OK) {
    // Nothing of a failed submission may write into the caller's buffer after this returns.
    const std::string msg = c->err;
    while (!c->inflight.empty()) async_finish_front(c);
    c->ticket_rc.erase(t);
    c->err = msg;
    return rc;
  }
  *ticket = t;
  return RV_OK;
}

int rv_embed_wait(rv_ctx* c, int64_t ticket) {
  if (!c) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  if (ticket <= 0 || ticket >= c->next_ticket) return fail(c, RV_E_INVALID, "unknown ticket");
  auto it = c->ticket_rc.find(ticket);
  if (it == c->ticket_rc.end()) return RV_OK;  // already waited on
  DeviceGuard g(c->device);
  std::string msg;
  while (!c->inflight.empty() && c->inflight.front().ticket <= ticket) {
    const int64_t bt = c->inflight.front().ticket;
    const int r = async_finish_front(c);
    if (r != RV_OK && bt == ticket) msg = c->err;
  }
  const int rc = c->ticket_rc[ticket];
  c->ticket_rc.erase(ticket);
  if (c->inflight.empty()) collect_marks(c);
  if (rc != RV_OK) c->err = msg.empty() ? c->err : msg;
  return rc;
}

int rv_embed_varlen_multi(rv_ctx* const* ctxs, int32_t n_ctx, const int32_t* ids, const int32_t* cu, int32_t n,
                          float* out_host) {
  if (!ctxs || n_ctx <= 0 || n < 0 || (n > 0 && (!cu || !out_host))) return RV_E_INVALID;
  for (int32_t i = 0; i < n_ctx; ++i)
    if (!ctxs[i] || ctxs[i]->d.hidden != ctxs[0]->d.hidden) return RV_E_INVALID;
  if (n == 0) return RV_OK;
  if (cu[0] != 0) return RV_E_INVALID;
  for (int32_t b = 0; b < n; ++b)
    if (cu[b + 1] < cu[b]) return RV_E_INVALID;
  if (cu[n] > 0 && !ids) return RV_E_INVALID;
  const int H = ctxs[0]->d.hidden;
  // Work is handed out in input order from one cursor: each worker takes the next run of
  // consecutive chunks that fills its context's token budget, embeds it with rv_embed_varlen
  // straight into its rows of out_host, and comes back for more, so a faster device takes more
  // runs.  The first failure stops the others from taking new runs.
  std::mutex mu;
  int32_t next = 0;
  int first_rc = RV_OK;
  int first_ctx = n_ctx;
  auto worker = [&](int32_t wi) {
    rv_ctx* c = ctxs[wi];
    const int64_t budget = std::max<int64_t>(1, c->t_max > 0 ? c->t_max : 262144);
    std::vector<int32_t> lcu;
    for (;;) {
      int32_t b0, b1;
      {
        std::lock_guard<std::mutex> lk(mu);
        if (first_rc != RV_OK || next >= n) return;
        b0 = next;
        b1 = b0 + 1;  // at least one chunk, even one longer than the budget (rv_embed_varlen checks it)
        while (b1 < n && int64_t(cu[b1 + 1]) - cu[b0] <= budget) ++b1;
        next = b1;
      }
      lcu.resize(size_t(b1 - b0) + 1);
      for (int32_t b = b0; b <= b1; ++b) lcu[b - b0] = cu[b] - cu[b0];
      const int rc = rv_embed_varlen(c, ids ? ids + cu[b0] : nullptr, lcu.data(), b1 - b0,
                                     out_host + size_t(b0) * H);
      if (rc != RV_OK) {
        std::lock_guard<std::mutex> lk(mu);
        if (first_rc == RV_OK || wi < first_ctx) {
          first_rc = rc;
          first_ctx = wi;
        }
        return;
      }
    }
  };
  if (n_ctx == 1) {
    worker(0);
  } else {
    std::vector<std::thread> ts;
    ts.reserve(size_t(n_ctx));
    for (int32_t i = 0; i < n_ctx; ++i) ts.emplace_back(worker, i);
    for (auto& t : ts) t.join();
  }
  return first_rc;
}

int rv_max_tokens(const rv_ctx* c) { return c ? c->d.max_position : 0; }
int rv_hidden_dim(const rv_ctx* c) { return c ? c->d.hidden : 0; }
const char* rv_name(const rv_ctx* c) {
  if (!c) return "";
  return c->d.arch == RV_ARCH_MODERNBERT ? "CUDA sm_100a (ModernBERT)" : "CUDA sm_100a (ClassicBert)";
}
int rv_is_gpu(const rv_ctx*) { return 1; }
const char* rv_last_error(const rv_ctx* c) { return c ? c->err.c_str() : "null context"; }
int64_t rv_kernel_launches(const rv_ctx* c) { return c ? c->launches : 0; }

int rv_set_profiling(rv_ctx* c, int enable) {
  if (!c) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  c->profiling = enable != 0;
  return RV_OK;
}

int rv_get_profile(rv_ctx* c, int kind, double* total_ms, int64_t* launches, double* flops) {
  if (!c || kind < 0 || kind >= RV_KIND_COUNT) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  if (total_ms) *total_ms = c->prof_ms[kind];
  if (launches) *launches = c->prof_n[kind];
  if (flops) *flops = c->prof_flops[kind];
  return RV_OK;
}

int rv_reset_profile(rv_ctx* c) {
  if (!c) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(c->mu);
  for (int k = 0; k < RV_KIND_COUNT; ++k) c->prof_ms[k] = c->prof_n[k] = c->prof_flops[k] = 0;
  return RV_OK;
}

}  // extern "C"
