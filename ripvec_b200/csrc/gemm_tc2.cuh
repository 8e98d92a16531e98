// Two-SM variant of the persistent tcgen05 GEMM: a cluster of two CTAs computes one 256 x 256
// output tile with tcgen05.mma.cta_group::2 (M = 256 split 128 / 128 across the pair, N = 256).
// Each CTA loads only its own 128 rows of A and its own 128 rows of B per k-block (32 KB per
// stage instead of 48 KB for a 128 x 256 tile), so shared-memory fill traffic from L2 per FLOP
// drops by a third and six pipeline stages fit.  No load is multicast: every CTA issues its own
// TMA copies into its own shared memory; only barrier signals cross the pair.
//
// Protocol (rank 0 = leader):
//   full[s]   leader-owned; leader producer arrives with expect_tx(both CTAs' bytes); both
//             producers' TMA loads complete_tx on it (cta_group::2 loads name the leader's barrier).
//   empty[s]  one per CTA; the leader's MMA thread commits with multicast to both.
//   tfull[a]  one per CTA; leader commits with multicast when accumulator a is complete.
//   tempty[a] leader-owned, 8 arrivals (4 epilogue warps x 2 CTAs, peers arrive remotely).
// Every wait is bounded (mbar_wait); both CTAs always reach the closing cluster barrier.
#pragma once

#include "gemm_tc.cuh"

namespace rv {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (for barriers that receive arrivals from the peer).
__device__ __forceinline__ bool mbar_try_wait_cluster_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (mbar_try_wait_cluster_sleep(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitLimitCycles) return false;
  }
}
// 2-D tiled load into this CTA's shared memory that completes on a barrier given by its
// shared::cluster address (the leader's), no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on the barrier at the same offset in both CTAs of the pair once every MMA issued so far
// by this thread has completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

struct Gemm2Cfg {
  static constexpr int kBN = 256;                            // pair tile N
  static constexpr int kHalfN = 128;                         // B rows loaded per CTA
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;      // 16 KB
  static constexpr int kBBytes = kHalfN * kGemmBK * 2;       // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;      // 32 KB per CTA
  static constexpr int kStages = 6;
  static constexpr uint32_t kTmemCols = 512;                 // 2 accumulators x 256 columns
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;
  static constexpr int kEpiSmemBytes = 10240;  // staged epilogue vectors (<= 2560 floats)
};

__device__ __forceinline__ void tc_commit_pair_mask(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// Lets copies already issued by this CTA land before it leaves (abort path only): their
// completion is counted on the leader's barrier, which this CTA cannot observe, so it waits a
// bounded time that is far longer than any copy takes.
__device__ __forceinline__ void settle_inflight_copies() {
  const long long t0 = clock64();
  while (clock64() - t0 < 4000000LL) {
  }
}

template <typename T, class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    int M, int N, int K, Epi epi, unsigned int* err) {
  using Cfg = Gemm2Cfg;
  constexpr int kStages = Cfg::kStages;
  constexpr int kBN = Cfg::kBN;
  constexpr uint32_t kIdesc = idesc_f16(2 * kGemmBM, kBN, Elem<T>::kBf16);

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
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before any signal crosses the pair
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
      const uint32_t full0 = mapa_shared(smem_u32(&full[0]), 0);  // the leader's full[0]
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
      // Drain: every MMA issued has completed before TMEM is freed.
      tc_commit_pair_mask(drain, 0x1);
      volatile int no_abort = 0;
      if (!mbar_wait_cluster(drain, 0, &no_abort)) atomicOr(err, kErrWaitTimeout);
    }
  } else {
    const int quad = warp & 3;
    const uint32_t tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);  // the leader's tempty[0]
    float* epi_smem = reinterpret_cast<float*>(smem + kStages * Cfg::kStageBytes + 256);
    epi.stage(epi_smem, threadIdx.x - 64, 128);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    int it = 0;
    bool ok = true;
    for (int t = cluster_id; t < num_tiles; t += num_clusters, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int m0 = (t / num_n) * (2 * kGemmBM) + static_cast<int>(rank) * kGemmBM;
      const int n0 = (t % num_n) * kBN;
      const int row = m0 + quad * 32 + lane;
      const bool live = row < M;
      typename Epi::Pre pre[2];
      typename Epi::Tile tile;
      if (live) {
        epi.tile_load(tile, row, n0);
        epi.load(pre[0], row, n0);
      }
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(&tfull[acc], acc_phase, abort_flag))) { ok = false; break; }
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * kBN);
#pragma unroll
      for (int g = 0; g < kBN / 64; ++g) {
        if (g + 1 < kBN / 64 && live) epi.load(pre[(g + 1) & 1], row, n0 + (g + 1) * 64);
        float v0[32], v1[32];
        tmem_ld32(tbase + g * 64, v0);
        tmem_ld32(tbase + g * 64 + 32, v1);
        tc_wait_ld();
        if (live) epi.apply(pre[g & 1], tile, row, n0 + g * 64, v0, v1);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + static_cast<uint32_t>(acc) * 8u);
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicOr(err, kErrWaitTimeout);
    }
  }

  __syncthreads();
  cluster_sync_all();  // both CTAs are done with TMEM before the pair frees it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

template <typename T, class Epi>
cudaError_t launch_gemm_tc2(const CUtensorMap& tmA, const CUtensorMap& tmB, int M, int N, int K,
                            const Epi& epi, unsigned int* err, int num_sms, cudaStream_t stream) {
  using Cfg = Gemm2Cfg;
  static PerDeviceOnce attr_set;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr_set.run([&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(gemm_tc2_kernel<T, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Cfg::kSmemBytes + Cfg::kEpiSmemBytes);
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  if (M <= 0) return cudaSuccess;
  if (N % Cfg::kBN != 0 || K % kGemmBK != 0) return cudaErrorInvalidValue;
  const int tiles = ((M + 2 * kGemmBM - 1) / (2 * kGemmBM)) * (N / Cfg::kBN);
  const int clusters = tiles < num_sms / 2 ? tiles : num_sms / 2;
  gemm_tc2_kernel<T, Epi><<<2 * clusters, kGemmThreads, Cfg::kSmemBytes + Cfg::kEpiSmemBytes, stream>>>(tmA, tmB, M, N, K, epi, err);
  return cudaGetLastError();
}

}  // namespace rv
