// Persistent tcgen05 GEMM for sm_100a: C[M,N] = A[M,K] * B[N,K]^T with fused epilogues.
//
// A (activations, row-major [M,K]) and B (weights, row-major [N,K]) are both K-major; TMA moves
// 128x64 / BNx64 tiles into 128-byte-swizzled shared memory, one thread issues
// tcgen05.mma (M=128, N=BN, K=16 per instruction) into a double-buffered TMEM accumulator, and
// four epilogue warps drain TMEM with tcgen05.ld while the next tile accumulates.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lane quadrant w % 4).
//
// This replaces the reference's cublasGemmEx calls for the QKV / attention-output / MLP
// projections (crates/ripvec-core/src/backend/driver/cuda.rs:3263-3357, called from
// backend/arch/modern_bert.rs:483-492, :718-747, :791-799, :830-838) and their follow-on
// elementwise kernels (RoPE driver/cuda.rs:1126, GeGLU :1188, residual add :1206, bias/GELU
// :519-543), which become epilogues of the one kernel.
#pragma once

#include <type_traits>
#include <utility>

#include "common.cuh"
#include "tmap.h"

namespace rv {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (BN >= 256) ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr uint32_t kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;
  static constexpr int kEpiSmemBytes = 10240;  // staged epilogue vectors (<= 2560 floats)
};

// ---------------------------------------------------------------- epilogues
// An epilogue handles one output row and one group of 64 consecutive accumulator columns
// [col, col+64): v0 holds columns col..col+31 and v1 holds col+32..col+63, in f32.  Global
// inputs an epilogue needs (residual, rotary tables) are fetched by load() into a Pre object one
// group ahead of apply(), and for the first group before the accumulator is ready, so their
// memory latency overlaps the tensor-core work instead of serialising the epilogue.

struct NoPre {};
struct NoTile {};

// Optional epilogue hook `finish(int t)`, called once by each of the 128 epilogue threads (index
// t) after the CTA's last tile, behind a barrier of those threads.
template <class E, class = void>
struct HasFinish : std::false_type {};
template <class E>
struct HasFinish<E, std::void_t<decltype(std::declval<const E&>().finish(0))>> : std::true_type {};

// Optional epilogue constant `kColumnMajorTiles = true`: persistent CTAs walk the tiles column
// block by column block (all row blocks of one B tile, then the next) instead of row block by row
// block.  For a GEMM whose B operand is larger than L2 and whose A operand fits in it, each B
// tile is then read from HBM once instead of once per row block.
template <class E, class = void>
struct ColumnMajorTiles : std::false_type {};
template <class E>
struct ColumnMajorTiles<E, std::void_t<decltype(E::kColumnMajorTiles)>>
    : std::integral_constant<bool, E::kColumnMajorTiles> {};

template <class Epi>
__device__ __forceinline__ void tile_origin(int t, int num_m, int num_n, int bn, int& m0, int& n0) {
  if constexpr (ColumnMajorTiles<Epi>::value) {
    m0 = (t % num_m) * kGemmBM;
    n0 = (t / num_m) * bn;
  } else {
    m0 = (t / num_n) * kGemmBM;
    n0 = (t % num_n) * bn;
  }
}

template <typename T>
struct EpiStore {
  T* c;
  int ldc;
  using Pre = NoPre;
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    uint4* dst = reinterpret_cast<uint4*>(c + static_cast<size_t>(row) * ldc + col);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = pack8<T>(&v0[8 * i]);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[4 + i] = pack8<T>(&v1[8 * i]);
  }
};

struct EpiStoreF32 {
  float* c;
  int ldc;
  using Pre = NoPre;
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    float4* dst = reinterpret_cast<float4*>(c + static_cast<size_t>(row) * ldc + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(v0[4 * i], v0[4 * i + 1], v0[4 * i + 2], v0[4 * i + 3]);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[8 + i] = make_float4(v1[4 * i], v1[4 * i + 1], v1[4 * i + 2], v1[4 * i + 3]);
  }
};

// c <- c + acc (+ bias): the residual add after the attention-output and MLP-output projections
// (reference residual_add, driver/cpu.rs:1319-1331; fused_bias_residual :1292-1305).
template <typename T>
struct EpiResidual {
  T* c;              // read (residual) and written (sum), same element
  int ldc;
  const float* bias; // optional [N]
  struct Pre {
    uint4 r[8];
  };
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre& p, int row, int col) const {
    const uint4* src = reinterpret_cast<const uint4*>(c + static_cast<size_t>(row) * ldc + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) p.r[i] = src[i];
  }
  __device__ __forceinline__ void apply(const Pre& p, Tile&, int row, int col,
                                        const float (&v0)[32], const float (&v1)[32]) const {
    uint4* dst = reinterpret_cast<uint4*>(c + static_cast<size_t>(row) * ldc + col);
    float r[8], o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      unpack8<T>(p.r[i], r);
      const float* v = (i < 4) ? &v0[8 * i] : &v1[8 * (i - 4)];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[j] + (bias ? bias[col + 8 * i + j] : 0.0f) + r[j];
      dst[i] = pack8<T>(o);
    }
  }
};

// GeGLU on an interleaved Wi: in each 64-column group the first 32 accumulator columns are the
// value half and the next 32 the matching gate half; out[row, col/2 + i] = gelu(v0[i]) * v1[i]
// (reference split + geglu, driver/cpu.rs:1188-1207, :1233-1246).
template <typename T>
struct EpiGeglu {
  T* out;
  int ldo;
  using Pre = NoPre;
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * ldo + (col >> 1));
    float o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = gelu_tanh(v0[8 * i + j]) * v1[8 * i + j];
      dst[i] = pack8<T>(o);
    }
  }
};

// Optional bias then tanh-GELU (ClassicBert FFN input projection; reference cpu.rs:426-462).
template <typename T>
struct EpiBiasGelu {
  T* c;
  int ldc;
  const float* bias;
  using Pre = NoPre;
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    uint4* dst = reinterpret_cast<uint4*>(c + static_cast<size_t>(row) * ldc + col);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float* v = (i < 4) ? &v0[8 * i] : &v1[8 * (i - 4)];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = gelu_tanh(v[j] + (bias ? bias[col + 8 * i + j] : 0.0f));
      dst[i] = pack8<T>(o);
    }
  }
};

// Plain store with optional bias (ClassicBert QKV projection with bias).
template <typename T>
struct EpiBias {
  T* c;
  int ldc;
  const float* bias;
  using Pre = NoPre;
  using Tile = NoTile;
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile&, int, int) const {}
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre&, Tile&, int row, int col, const float (&v0)[32],
                                        const float (&v1)[32]) const {
    uint4* dst = reinterpret_cast<uint4*>(c + static_cast<size_t>(row) * ldc + col);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float* v = (i < 4) ? &v0[8 * i] : &v1[8 * (i - 4)];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[j] + (bias ? bias[col + 8 * i + j] : 0.0f);
      dst[i] = pack8<T>(o);
    }
  }
};

// QKV projection with rotary position embedding applied to the Q and K heads (columns
// < rope_cols) in f32 before rounding; head_dim is 64, so one 64-column group is one head and
// the rotate-half pairs are (v0[d], v1[d]).  pos[row] is the token's position inside its
// sequence; cos/sin tables are [max_pos, 32] f32 built on the host like the reference
// (driver/cpu.rs:670-688 table, :1155-1186 rotation).  Every head of a row uses the same
// position, so the row's 32 cos and 32 sin values are fetched once per tile, before the
// accumulator is ready.
template <typename T>
struct EpiQkvRope {
  T* c;
  int ldc;
  int rope_cols;
  const int* pos;
  const float* cos_t;
  const float* sin_t;
  using Pre = NoPre;
  struct Tile {
    float4 cv[8], sv[8];
  };
  __device__ __forceinline__ void stage(float*, int, int) const {}
  __device__ __forceinline__ void tile_load(Tile& t, int row, int n0) const {
    if (n0 >= rope_cols) return;
    const int p = pos[row];
    const float4* cs = reinterpret_cast<const float4*>(cos_t + static_cast<size_t>(p) * 32);
    const float4* sn = reinterpret_cast<const float4*>(sin_t + static_cast<size_t>(p) * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      t.cv[i] = cs[i];
      t.sv[i] = sn[i];
    }
  }
  __device__ __forceinline__ void load(Pre&, int, int) const {}
  __device__ __forceinline__ void apply(const Pre&, Tile& t, int row, int col,
                                        const float (&v0)[32], const float (&v1)[32]) const {
    uint4* dst = reinterpret_cast<uint4*>(c + static_cast<size_t>(row) * ldc + col);
    if (col < rope_cols) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float cc[8] = {t.cv[2 * i].x, t.cv[2 * i].y, t.cv[2 * i].z, t.cv[2 * i].w,
                             t.cv[2 * i + 1].x, t.cv[2 * i + 1].y, t.cv[2 * i + 1].z, t.cv[2 * i + 1].w};
        const float ss[8] = {t.sv[2 * i].x, t.sv[2 * i].y, t.sv[2 * i].z, t.sv[2 * i].w,
                             t.sv[2 * i + 1].x, t.sv[2 * i + 1].y, t.sv[2 * i + 1].z, t.sv[2 * i + 1].w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float f = v0[8 * i + j], s = v1[8 * i + j];
          a[j] = f * cc[j] - s * ss[j];
          b[j] = f * ss[j] + s * cc[j];
        }
        dst[i] = pack8<T>(a);
        dst[4 + i] = pack8<T>(b);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = pack8<T>(&v0[8 * i]);
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[4 + i] = pack8<T>(&v1[8 * i]);
    }
  }
};

// ---------------------------------------------------------------- kernel
template <typename T, int BN, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   int M, int N, int K, int b_row_offset, Epi epi, unsigned int* err) {
  using Cfg = GemmCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  constexpr uint32_t kIdesc = idesc_f16(kGemmBM, BN, Elem<T>::kBf16);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * Cfg::kBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + kGemmBM - 1) / kGemmBM;
  const int num_n = N / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = K / kGemmBK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int m0, n0;
        tile_origin<Epi>(t, num_m, num_n, BN, m0, n0);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(sA + stage * Cfg::kABytes, &tmA, &full[stage], kb * kGemmBK, m0);
          tma_load_2d(sB + stage * Cfg::kBBytes, &tmB, &full[stage], kb * kGemmBK, n0 + b_row_offset);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, kErrWaitTimeout);
        // Let the copies already issued land before the CTA exits.
        for (int s = 0; s < kStages; ++s)
          if (issued & (1u << s)) {
            volatile int no_abort = 0;
            mbar_wait(&full[s], (issued_parity >> s) & 1u, &no_abort);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            tc_mma_f16(d_tmem, smem_desc_sw128(a_addr + 32 * k), smem_desc_sw128(b_addr + 32 * k),
                       kIdesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) tc_commit(&tfull[acc]);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, kErrWaitTimeout);
      }
      // Drain: wait until every MMA this thread issued has completed before TMEM is freed.
      tc_commit(drain);
      volatile int no_abort = 0;
      if (!mbar_wait(drain, 0, &no_abort)) atomicOr(err, kErrWaitTimeout);
    }
  } else {
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    // Epilogue-constant vectors (column sums of folded weights) go to shared memory once.
    float* epi_smem = reinterpret_cast<float*>(smem + kStages * Cfg::kStageBytes + 256);
    epi.stage(epi_smem, threadIdx.x - 64, 128);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      int m0, n0;
      tile_origin<Epi>(t, num_m, num_n, BN, m0, n0);
      const int row = m0 + quad * 32 + lane;
      const bool live = row < M;
      typename Epi::Pre pre[2];
      typename Epi::Tile tile;
      if (live) {  // before the accumulator is ready
        epi.tile_load(tile, row, n0);
        epi.load(pre[0], row, n0);
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) { ok = false; break; }
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll
      for (int g = 0; g < BN / 64; ++g) {
        if (g + 1 < BN / 64 && live) epi.load(pre[(g + 1) & 1], row, n0 + (g + 1) * 64);
        float v0[32], v1[32];
        tmem_ld32(tbase + g * 64, v0);
        tmem_ld32(tbase + g * 64 + 32, v1);
        tc_wait_ld();
        if (live) epi.apply(pre[g & 1], tile, row, n0 + g * 64, v0, v1);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(err, kErrWaitTimeout);
    }
    if constexpr (HasFinish<Epi>::value) {
      // Every epilogue warp reaches this point exactly once (finished or aborted), so the
      // barrier of the 128 epilogue threads always completes.
      asm volatile("bar.sync 1, 128;" ::: "memory");
      epi.finish(threadIdx.x - 64);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// Host-side launch.  grid = min(tiles, sms) persistent CTAs.  Returns the launch status.
template <typename T, int BN, class Epi>
cudaError_t launch_gemm_tc(const CUtensorMap& tmA, const CUtensorMap& tmB, int M, int N, int K,
                           int b_row_offset, const Epi& epi, unsigned int* err, int num_sms,
                           cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  static PerDeviceOnce attr_set;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr_set.run([&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<T, BN, Epi>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Cfg::kSmemBytes + Cfg::kEpiSmemBytes);
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  if (M <= 0) return cudaSuccess;
  const int tiles = ((M + kGemmBM - 1) / kGemmBM) * (N / BN);
  const int grid = tiles < num_sms ? tiles : num_sms;
  gemm_tc_kernel<T, BN, Epi><<<grid, kGemmThreads, Cfg::kSmemBytes + Cfg::kEpiSmemBytes, stream>>>(
      tmA, tmB, M, N, K, b_row_offset, epi, err);
  return cudaGetLastError();
}

}  // namespace rv
