// Embedding store import / export.
//
// rv_cache_decode reads the embeddings of one per-file cache object of the reference
// (crates/ripvec-core/src/cache/file_cache.rs:15-22, written by FileCache::to_bytes :43-49 and read
// back by cache/reindex.rs:302, :411): a zstd frame (magic 28 B5 2F FD, :27) around an rkyv 0.8
// archive of
//     FileCache { chunks: Vec<CodeChunk>, embeddings: Vec<f32>, hidden_dim: usize }
// or, for objects written before compression was added, the bare archive (:58-66).  rkyv 0.8's
// default format is little-endian with 32-bit relative pointers and lengths, and the root object
// sits at the end of the buffer.  The archived root is therefore 20 bytes,
//     chunks {i32 offset, u32 len}, embeddings {i32 offset, u32 len}, hidden_dim u32,
// and an offset is relative to the position of the pointer field itself.  Only the embeddings,
// the chunk count and hidden_dim are read; the chunks themselves (paths and source text) stay on
// the host side of the caller.  The portable form (magic "BC" + zstd of a bitcode encoding,
// :78-110) is bit-packed and is refused with RV_E_IO.
//
// zstd comes from the system's libzstd.so.1 through its public streaming API, loaded on first
// use; without it compressed objects are refused with RV_E_IO.
//
// rv_index_export copies rows of an index back out (bf16 as stored, or widened to f32), so a
// device shard can be written to the caller's store and recreated later with rv_index_create.
#include <dlfcn.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "index_impl.h"
#include "ripvec_b200.h"

namespace {

// The few declarations of zstd's stable public streaming API (zstd.h) this reader uses.
struct ZInBuffer {
  const void* src;
  size_t size;
  size_t pos;
};
struct ZOutBuffer {
  void* dst;
  size_t size;
  size_t pos;
};
struct ZstdApi {
  void* (*create_dctx)() = nullptr;
  size_t (*free_dctx)(void*) = nullptr;
  size_t (*decompress_stream)(void*, ZOutBuffer*, ZInBuffer*) = nullptr;
  unsigned (*is_error)(size_t) = nullptr;
  const char* (*error_name)(size_t) = nullptr;
  bool ok = false;
};

const ZstdApi& zstd() {
  static ZstdApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libzstd.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libzstd.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    api.create_dctx = reinterpret_cast<void* (*)()>(dlsym(h, "ZSTD_createDCtx"));
    api.free_dctx = reinterpret_cast<size_t (*)(void*)>(dlsym(h, "ZSTD_freeDCtx"));
    api.decompress_stream =
        reinterpret_cast<size_t (*)(void*, ZOutBuffer*, ZInBuffer*)>(dlsym(h, "ZSTD_decompressStream"));
    api.is_error = reinterpret_cast<unsigned (*)(size_t)>(dlsym(h, "ZSTD_isError"));
    api.error_name = reinterpret_cast<const char* (*)(size_t)>(dlsym(h, "ZSTD_getErrorName"));
    api.ok = api.create_dctx && api.free_dctx && api.decompress_stream && api.is_error && api.error_name;
  });
  return api;
}

thread_local std::string g_cache_error;

int cache_fail(int code, std::string msg) {
  g_cache_error = std::move(msg);
  return code;
}

constexpr uint8_t kZstdMagic[4] = {0x28, 0xB5, 0x2F, 0xFD};
constexpr uint64_t kMaxDecoded = uint64_t(1) << 34;  // 16 GiB: a guard against corrupt frames

// Decompresses every frame of [src, src + n) into out.  Returns an empty message on success.
std::string unzstd(const uint8_t* src, size_t n, std::vector<uint8_t>& out) {
  const ZstdApi& z = zstd();
  if (!z.ok) return "zstd-compressed object, but libzstd.so.1 could not be loaded";
  void* dctx = z.create_dctx();
  if (!dctx) return "ZSTD_createDCtx failed";
  ZInBuffer in{src, n, 0};
  out.clear();
  std::string err;
  size_t last = 1;
  while (in.pos < in.size || last != 0) {
    if (out.size() + (size_t(1) << 20) > kMaxDecoded) {
      err = "decompressed object larger than 16 GiB";
      break;
    }
    const size_t old = out.size();
    out.resize(old + (size_t(1) << 20));
    ZOutBuffer o{out.data() + old, size_t(1) << 20, 0};
    const size_t before_in = in.pos;
    last = z.decompress_stream(dctx, &o, &in);
    out.resize(old + o.pos);
    if (z.is_error(last)) {
      err = std::string("zstd: ") + z.error_name(last);
      break;
    }
    if (in.pos == in.size && last != 0 && o.pos == 0 && in.pos == before_in) {
      err = "zstd: truncated frame";
      break;
    }
  }
  z.free_dctx(dctx);
  return err;
}

int xfail(rv_index* x, int code, const std::string& m) {
  x->err = m;
  return code;
}

#define CX_TRY(x, expr)                                                              \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess)                                                           \
      return xfail(x, RV_E_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

// Makes `d` current for the scope and restores the caller's device.
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

uint32_t rd_u32(const uint8_t* p) {
  uint32_t v;
  std::memcpy(&v, p, 4);
  return v;  // little-endian host (x86-64, aarch64)
}

}  // namespace

extern "C" {

const char* rv_cache_last_error(void) { return g_cache_error.c_str(); }

int rv_cache_decode(const uint8_t* obj, uint64_t nbytes, float* out_emb, int64_t capacity_floats, int64_t* out_rows,
                    int32_t* out_dim) {
  if (!out_rows || !out_dim || (nbytes > 0 && !obj) || capacity_floats < 0)
    return cache_fail(RV_E_INVALID, "null argument or negative capacity");
  *out_rows = 0;
  *out_dim = 0;
  std::vector<uint8_t> raw;
  const uint8_t* a = obj;
  size_t n = size_t(nbytes);
  // The portable form is recognised by its two magic bytes alone, as load_file_cache does
  // (cache/reindex.rs:524-530).
  if (n >= 2 && obj[0] == 'B' && obj[1] == 'C')
    return cache_fail(RV_E_IO, "portable (bitcode) cache objects are not supported; read the rkyv form");
  if (n >= 4 && std::memcmp(obj, kZstdMagic, 4) == 0) {
    const std::string err = unzstd(obj, n, raw);
    if (!err.empty()) return cache_fail(RV_E_IO, err);
    a = raw.data();
    n = raw.size();
  }
  // Archived root: the last 20 bytes, 4-byte aligned.
  constexpr size_t kRoot = 20;
  if (n < kRoot || n % 4 != 0) return cache_fail(RV_E_IO, "not an rkyv FileCache archive (size)");
  const size_t root = n - kRoot;
  const uint32_t n_chunks = rd_u32(a + root + 4);
  int32_t rel;
  std::memcpy(&rel, a + root + 8, 4);
  const uint32_t n_floats = rd_u32(a + root + 12);
  const uint32_t dim = rd_u32(a + root + 16);
  if (dim == 0 || dim > (1u << 20)) return cache_fail(RV_E_IO, "not an rkyv FileCache archive (hidden_dim)");
  const int64_t data = int64_t(root) + 8 + rel;  // relative to the pointer field
  if (n_floats > 0 && (data < 0 || data % 4 != 0 || uint64_t(data) + uint64_t(n_floats) * 4 > root))
    return cache_fail(RV_E_IO, "embeddings pointer outside the archive");
  // Chunk i keeps its embedding only when the whole slice [i * dim, (i + 1) * dim) exists
  // (cache/reindex.rs:578-587).
  const int64_t rows = std::min<int64_t>(n_chunks, n_floats / dim);
  *out_rows = rows;
  *out_dim = int32_t(dim);
  if (!out_emb) return RV_OK;  // size query
  if (capacity_floats < rows * int64_t(dim))
    return cache_fail(RV_E_INVALID, "output holds " + std::to_string(capacity_floats) + " floats, need " +
                                        std::to_string(rows * int64_t(dim)));
  if (rows > 0) std::memcpy(out_emb, a + data, size_t(rows) * dim * 4);
  return RV_OK;
}

int rv_index_export(rv_index* x, int64_t row0, int64_t n, int32_t dst_dtype, void* dst, int32_t dst_on_device) {
  if (!x) return RV_E_INVALID;
  std::lock_guard<std::mutex> lk(x->mu);
  if (row0 < 0 || n < 0 || row0 + n > x->n || (n > 0 && !dst) ||
      (dst_dtype != RV_DTYPE_BF16 && dst_dtype != RV_DTYPE_F32))
    return xfail(x, RV_E_INVALID, "row range outside the index, null output or unsupported dtype");
  if (n == 0) return RV_OK;
  DeviceScope g(x->device);
  const size_t elems = size_t(n) * x->dim;
  const __nv_bfloat16* src = x->db + size_t(row0) * x->dim;
  if (dst_dtype == RV_DTYPE_BF16) {
    CX_TRY(x, cudaMemcpyAsync(dst, src, elems * 2, dst_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                              x->stream));
    CX_TRY(x, cudaStreamSynchronize(x->stream));
    return RV_OK;
  }
  // f32: widen on the host, in slices (bf16 -> f32 is exact).
  const size_t slice = size_t(1) << 22;
  std::vector<uint16_t> tmp;
  std::vector<float> wide;
  for (size_t s = 0; s < elems; s += slice) {
    const size_t e = std::min(elems, s + slice);
    tmp.resize(e - s);
    CX_TRY(x, cudaMemcpyAsync(tmp.data(), src + s, (e - s) * 2, cudaMemcpyDeviceToHost, x->stream));
    CX_TRY(x, cudaStreamSynchronize(x->stream));
    float* out = static_cast<float*>(dst) + s;
    if (dst_on_device) {
      wide.resize(e - s);
      out = wide.data();
    }
    for (size_t i = 0; i < e - s; ++i) {
      const uint32_t bits = uint32_t(tmp[i]) << 16;
      std::memcpy(out + i, &bits, 4);
    }
    if (dst_on_device) {
      CX_TRY(x, cudaMemcpyAsync(static_cast<float*>(dst) + s, wide.data(), (e - s) * 4, cudaMemcpyHostToDevice,
                                x->stream));
      CX_TRY(x, cudaStreamSynchronize(x->stream));
    }
  }
  return RV_OK;
}

}  // extern "C"
