// Two-CTA tcgen05 GEMM with a TMA-staged epilogue (the encoder's projection GEMMs).
//
// Mainloop as gemm_tc2_kernel (cta_group::2, 256 x 256 pair tiles, 4 stages of 32 KB per CTA)
// into two TMEM accumulators.  Epilogue: two warpgroups of 128 threads, warpgroup e draining
// accumulator e (every other tile), so two tiles' epilogues run at once.  Each processes its
// 128 x 256 block in four 64-column groups through its own ring of two 16 KB shared-memory
// tiles, and within it each warp handles its own 32 rows: when the epilogue reads the output as
// well (residual add), the warp's lane 0 TMA-loads the warp's 32 x 64 block of C into its part of
// the ring one group ahead; every thread then combines its row with its accumulator columns and
// writes the result into the same place (128-byte swizzled, bank-conflict free), and lane 0
// TMA-stores the warp's 32 rows (the output tensor maps have 32-row boxes).  No barrier couples
// the warps; epilogue threads never wait on global memory; the accumulator is released as soon as
// the last TMEM load of a tile is done.
#pragma once

#include "gemm_epi_tma.cuh"
#include "gemm_tc2.cuh"

namespace rv {

struct Gemm2TmaCfg {
  static constexpr int kBN = 256;
  static constexpr int kHalfN = 128;
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = kHalfN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;  // 32 KB
  static constexpr int kStages = 4;
  static constexpr int kEpiGroups = 2;                    // epilogue warpgroups (one per accumulator)
  static constexpr int kEpiWarps = 4 * kEpiGroups;
  static constexpr int kRing = 2;                         // staging tiles per epilogue warpgroup
  static constexpr int kRingBytes = 16384;                // 128 rows x 128 B
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kEpiSmemBytes = 10240;
  static constexpr int kThreads = 64 + 128 * kEpiGroups;  // producer, MMA issuer, 8 epilogue warps
  static constexpr int kSmemBytes =
      1024 + kStages * kStageBytes + kEpiGroups * kRing * kRingBytes + 256 + kEpiSmemBytes;
};

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Byte offset of 16-byte chunk j of row r in a tile written by TMA with 128-byte (rows of 128 B)
// or 64-byte (rows of 64 B) swizzling; the tile base is 1024-byte aligned.
template <int kRowBytes>
__device__ __forceinline__ uint32_t swz(int r, int j) {
  if (kRowBytes == 128) return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
  return static_cast<uint32_t>(r * 64 + ((j ^ ((r >> 1) & 3)) << 4));
}

template <typename T, class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Gemm2TmaCfg::kThreads, 1)
    gemm_tc2_tma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, int M, int N, int K, Epi epi,
                        unsigned int* err) {
  using Cfg = Gemm2TmaCfg;
  constexpr int kStages = Cfg::kStages;
  constexpr int kBN = Cfg::kBN;
  constexpr int kOutCols = Epi::kOutCols;           // 64 (128-B rows) or 32 (64-B rows)
  constexpr int kRowBytes = kOutCols * 2;
  constexpr uint32_t kIdesc = idesc_f16(2 * kGemmBM, kBN, Elem<T>::kBf16);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kABytes;
  uint8_t* ring = smem + kStages * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + Cfg::kEpiGroups * Cfg::kRing * Cfg::kRingBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* rfull = drain + 1;  // [epilogue warp][kRing]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rfull + Cfg::kEpiWarps * Cfg::kRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* epi_smem = reinterpret_cast<float*>(ring + Cfg::kEpiGroups * Cfg::kRing * Cfg::kRingBytes + 256);
  static_assert((2 * kStages + 2 + 2 + 1 + Cfg::kEpiWarps * Cfg::kRing) * 8 + 8 <= 256, "barrier area");

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    mbar_init(drain, 1);
    for (int b = 0; b < Cfg::kEpiWarps * Cfg::kRing; ++b) mbar_init(&rfull[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + 2 * kGemmBM - 1) / (2 * kGemmBM);
  const int num_n = N / kBN;
  const int num_tiles = num_m * num_n;
  const int num_kb = K / kGemmBK;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters) {
        const int m0 = (t / num_n) * (2 * kGemmBM) + static_cast<int>(rank) * kGemmBM;
        const int nb = (t % num_n) * kBN + static_cast<int>(rank) * Cfg::kHalfN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          const uint32_t fb = full0 + static_cast<uint32_t>(stage) * 8u;
          tma_load_2d_pair(sA + stage * Cfg::kABytes, &tmA, fb, kb * kGemmBK, m0);
          tma_load_2d_pair(sB + stage * Cfg::kBBytes, &tmB, fb, kb * kGemmBK, nb);
          issued = true;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, kErrWaitTimeout);
        if (issued) settle_inflight_copies();
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int t = cluster_id; t < num_tiles && ok; t += num_clusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cluster(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k)
            tc_mma_f16_pair(d_tmem, smem_desc_sw128(a_addr + 32 * k), smem_desc_sw128(b_addr + 32 * k), kIdesc,
                            (kb | k) != 0 ? 1u : 0u);
          tc_commit_pair(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) tc_commit_pair(&tfull[acc]);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, kErrWaitTimeout);
      }
      tc_commit_pair_mask(drain, 0x1);
      volatile int no_abort = 0;
      if (!mbar_wait_cluster(drain, 0, &no_abort)) atomicOr(err, kErrWaitTimeout);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (2 x 128 threads)
    // Epilogue warpgroup ewg drains accumulator ewg, i.e. every other tile of the CTA; the two
    // warpgroups work on consecutive tiles at the same time.  Each warp owns its 32 rows (its
    // TMEM lane quadrant) of every 64-column group: its lane 0 TMA-loads the warp's rows of C one
    // group ahead (when the epilogue reads the output) into the warp's 32-row part of the
    // warpgroup's staging tile and TMA-stores the warp's results from there, so the four warps of
    // a warpgroup never wait for one another.
    const int ewg = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int rl = quad * 32 + lane;             // row inside this CTA's 128-row block = TMEM lane
    constexpr uint32_t kSubBytes = 32 * kRowBytes;  // this warp's 32 rows of a staging tile
    uint8_t* ring_w = ring + ewg * Cfg::kRing * Cfg::kRingBytes + quad * kSubBytes;
    uint64_t* rfull_w = rfull + (warp - 2) * Cfg::kRing;
    const uint32_t tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    epi.stage(epi_smem, threadIdx.x - 64, 128 * Cfg::kEpiGroups);
    asm volatile("bar.sync 3, %0;" ::"n"(128 * Cfg::kEpiGroups) : "memory");
    constexpr int kGroups = kBN / 64;
    const int my_tiles = cluster_id < num_tiles ? (num_tiles - 1 - cluster_id) / num_clusters + 1 : 0;
    const int ew_tiles = my_tiles > ewg ? (my_tiles - 1 - ewg) / Cfg::kEpiGroups + 1 : 0;
    const int total_groups = ew_tiles * kGroups;
    // Group q of this warpgroup: its (q / kGroups)-th tile, i.e. CTA tile it = 2 (q / kGroups) + ewg.
    auto group_tile = [&](int q) { return cluster_id + (Cfg::kEpiGroups * (q / kGroups) + ewg) * num_clusters; };
    // First output row of this warp in tile t.
    auto warp_row0 = [&](int t) { return (t / num_n) * (2 * kGemmBM) + static_cast<int>(rank) * kGemmBM + quad * 32; };
    if (Epi::kReadsC && lane == 0 && total_groups > 0) {
      const int t = group_tile(0);
      mbar_arrive_expect_tx(&rfull_w[0], kSubBytes);
      tma_load_2d(ring_w, &tmC, &rfull_w[0], (t % num_n) * kBN, warp_row0(t));
    }
    bool ok = true;
    int last_load = Epi::kReadsC && total_groups > 0 ? 0 : -1;  // newest group whose C load is in flight (lane 0)
    typename Epi::Tile tile;
    for (int q = 0; q < total_groups; ++q) {
      const int g = q % kGroups;
      const int j = q / kGroups;
      const int t = group_tile(q);
      const int acc = ewg;
      const uint32_t acc_phase = j & 1;  // accumulator ewg's j-th use
      const int m0 = (t / num_n) * (2 * kGemmBM) + static_cast<int>(rank) * kGemmBM;
      const int n0 = (t % num_n) * kBN;
      const int row = m0 + rl;
      const bool live = row < M;
      const int b = q % Cfg::kRing;
      uint8_t* buf = ring_w + b * Cfg::kRingBytes;
      if (lane == 0 && Epi::kReadsC && q + 1 < total_groups) {
        // C of group q + 1 goes into slot (q + 1) % 2, which this warp's store of group q - 1 reads.
        bulk_wait_read<0>();
        const int qn = q + 1, tn = group_tile(qn), bn = qn % Cfg::kRing;
        fence_proxy_async();
        mbar_arrive_expect_tx(&rfull_w[bn], kSubBytes);
        tma_load_2d(ring_w + bn * Cfg::kRingBytes, &tmC, &rfull_w[bn], (tn % num_n) * kBN + (qn % kGroups) * 64,
                    warp_row0(tn));
        last_load = qn;
      }
      bool fail = false;
      if (g == 0) {
        if (live) epi.tile_load(tile, row, n0);
        const bool w = mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag);
        fail = !__all_sync(0xffffffffu, w);
        tc_fence_after();
      }
      float v0[32], v1[32];
      if (!fail) {
        const uint32_t tbase =
            tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * kBN);
        tmem_ld32(tbase + g * 64, v0);
        tmem_ld32(tbase + g * 64 + 32, v1);
        tc_wait_ld();
        if (g == kGroups - 1) {  // the accumulator can be reused as soon as it has been read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty0 + static_cast<uint32_t>(acc) * 8u);
        }
      }
      float r[64];
      if (Epi::kReadsC && !fail) {
        const bool w = mbar_wait(&rfull_w[b], (q / Cfg::kRing) & 1, abort_flag);
        fail = !__all_sync(0xffffffffu, w);
        if (!fail) {
#pragma unroll
          for (int jj = 0; jj < 8; ++jj)
            unpack8<T>(*reinterpret_cast<const uint4*>(buf + swz<128>(lane, jj)), &r[8 * jj]);
        }
      }
      if (!fail) {
        epi.compute(tile, row, n0 + g * 64, r, v0, v1, live);
#pragma unroll
        for (int jj = 0; jj < kOutCols / 8; ++jj) {
          const float* v = (jj < 4) ? &v0[8 * jj] : &v1[8 * (jj - 4)];
          *reinterpret_cast<uint4*>(buf + swz<kRowBytes>(lane, jj)) = pack8<T>(v);
        }
      }
      fence_proxy_async();
      if (__any_sync(0xffffffffu, fail || *abort_flag != 0)) {  // a warp-uniform exit decision
        ok = false;
        break;
      }
      __syncwarp();  // the warp's rows are in the staging tile before lane 0 stores them
      if (lane == 0) {
        const int out_col = (kOutCols == 64) ? n0 + g * 64 : (n0 + g * 64) / 2;
        tma_store_2d(&tmC, buf, out_col, m0 + quad * 32);
        bulk_commit();
        // Group q + 1 overwrites slot (q + 1) % 2 = (q - 1) % 2: this warp's store of group q - 1
        // has read it once at most the newest store (group q) is outstanding.
        bulk_wait_read<1>();
      }
      __syncwarp();
    }
    if (!ok && lane == 0 && last_load >= 0) {  // let the C load still in flight land (bounded)
      volatile int no_abort = 0;
      mbar_wait(&rfull_w[last_load % Cfg::kRing], (last_load / Cfg::kRing) & 1, &no_abort);
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(err, kErrWaitTimeout);
    }
    if (lane == 0) bulk_wait_all();  // every store of this warp has landed before the kernel ends
  }

  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

template <typename T, class Epi>
cudaError_t launch_gemm_tc2_tma(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmC, int M,
                                int N, int K, const Epi& epi, unsigned int* err, int num_sms, cudaStream_t stream) {
  using Cfg = Gemm2TmaCfg;
  static PerDeviceOnce attr_set;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr_set.run([&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(gemm_tc2_tma_kernel<T, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Cfg::kSmemBytes);
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  if (M <= 0) return cudaSuccess;
  if (N % Cfg::kBN != 0 || K % kGemmBK != 0) return cudaErrorInvalidValue;
  const int tiles = ((M + 2 * kGemmBM - 1) / (2 * kGemmBM)) * (N / Cfg::kBN);
  const int clusters = tiles < num_sms / 2 ? tiles : num_sms / 2;
  gemm_tc2_tma_kernel<T, Epi><<<2 * clusters, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(tmA, tmB, tmC, M, N, K,
                                                                                        epi, err);
  return cudaGetLastError();
}

}  // namespace rv
