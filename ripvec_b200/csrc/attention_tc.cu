// Varlen attention on the 5th-generation tensor cores (head_dim 64, bf16 or f16).
//
// Work item = (128-query tile of one sequence, head); the host lists the tiles as
// {sequence start, length | first query << 16} records, longest sequences first.  The kernel is
// persistent: two CTAs per SM each walk the items blockIdx.x, blockIdx.x + gridDim.x, ...
// (head-major, so the items in flight share their sequences' K/V in L2), and every ring below
// runs across item boundaries, so the next item's Q and K/V load while the current one finishes.
// Warp roles (192 threads):
//   warp 0      TMA producers: lane 0 loads Q per item (2 buffers) and K tiles, lane 1 loads V
//               tiles, 64 keys per tile; both rings are as deep as the score ring, so slot
//               g % 3 of K is free once S of tile g completed (s_full) and slot g % 3 of V once
//               P V of tile g completed (p_empty): the MMA thread commits once per MMA group,
//   warp 1      TMEM owner and single-thread tcgen05.mma issuer,
//   warps 2..5  softmax: warp w owns TMEM lane quadrant w % 4 (32 query rows, one per thread)
//               and all 64 keys of every tile.
// Per key tile g (counted across items):
//   S[g%3] = Q K^T      tcgen05.mma M=128 N=64 K=64 into TMEM, issued three tiles ahead, so the
//                       softmax warps find the next tile's scores ready when they finish one and
//                       the MMA round trip stays off their critical path,
//   softmax             each thread reads its row's 64 scores with tcgen05.ld, masks keys past
//                       the sequence end and, on sliding-window layers, keys with |i - j| > w/2
//                       (32-key halves that no row of the warp can see skip the exponentials);
//                       P = exp2(s - m) (MUFU ex2; with RV_ATTN_EXP2_POLY=1 one pair in
//                       four on the FMA pipe by exp2_poly) is
//                       written as packed 16-bit pairs over S[g%3] in TMEM (tcgen05.st),
//   O += P V            tcgen05.mma M=128 N=64 K=64 with P (A) read from TMEM and V as an
//                       MN-major shared-memory operand, into the TMEM accumulator O; the
//                       reference max m moves only when a row's max grows by more than 2^8
//                       (then the row's O is rescaled in TMEM), and the item's context rows are
//                       read out of O after the next item's first P is written, before that
//                       item's first P V overwrites O.
// Reference semantics: backend/arch/modern_bert.rs:250-322 and driver/cpu.rs:1016-1074 (scores *
// 1/sqrt(d), additive -1e9 masks for padding and |i-j| > window/2, max-subtracted softmax, P V);
// masked keys get weight 0 exactly, as exp(-1e9 - max) does in f32.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "tmap.h"

namespace rv {

namespace {

constexpr int kBQ = 128;       // queries per item
constexpr int kBKV = 64;       // keys per tile
constexpr int kD = 64;         // head dim
// Score buffers in TMEM: S of tile g + 3 is issued once P V of tile g (which reads P out of the
// same columns) has been issued.  K is on the critical path (S needs it kSBufs tiles ahead of
// the softmax) and is loaded kKStages tiles ahead; V is needed only when P V is issued.
constexpr int kSBufs = 3;
constexpr int kKStages = 3;  // == kSBufs: slot g % 3 of K is free when S of tile g completes
constexpr int kVStages = 3;  // == kSBufs: slot g % 3 of V is free when P V of tile g completes
constexpr int kQBytes = kBQ * kD * 2;    // 16 KB
constexpr int kKVBytes = kBKV * kD * 2;  // 8 KB
constexpr int kOCol = kSBufs * kBKV;     // O after the score buffers
constexpr int kTmemCols = 256;           // S[3] at columns 0, 64, 128; O at 192
static_assert(kOCol + kD <= kTmemCols, "TMEM layout");
constexpr int kThreads = 192;  // producer, MMA issuer, 4 softmax warps
constexpr int kSoftmaxWarps = 4;
// 90 KB: two CTAs fit an SM; TMEM (256 columns per CTA) keeps it at two.
constexpr int kSmem = 1024 + 2 * kQBytes + (kKStages + kVStages) * kKVBytes + 512;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA and integer pipes instead of the MUFU unit, so that part of the softmax
// exponentials can run beside the hardware ex2.  Method: Cody-Waite style range reduction
// x = n + f with n = rint(x), taken from the round-to-nearest sum x + 1.5 * 2^23 (whose low
// mantissa bits hold n), f = x - n exact in [-1/2, 1/2]; 2^f by a degree-3 polynomial whose
// coefficients are this project's own Remez (minimax relative error) fit on [-1/2, 1/2]; 2^n by
// adding n to the exponent field.  Relative error below 7.6e-5 for x in [-125, 126] (the
// polynomial's minimax error; the reduction and the scaling are exact), against 2^-9 and 2^-12
// for the bf16 and f16 rounding of P.  Below -125 the result is 0, so a masked score (-inf)
// gets weight 0 exactly, as with ex2.approx.ftz, which also flushes results below 2^-126.
constexpr float kExpShift = 12582912.0f;  // 1.5 * 2^23
constexpr float kExpC0 = 0.99992806f, kExpC1 = 0.69326097f, kExpC2 = 0.24261113f, kExpC3 = 0.055171669f;
__device__ __forceinline__ float exp2_poly(float x) {
  // Scalar arithmetic, so that the constants come from the constant bank rather than registers.
  const float xc = fmaxf(x, -125.f);
  const float t = __fadd_rn(xc, kExpShift);  // 1.5 * 2^23 + rint(x)
  const float n = __fsub_rn(t, kExpShift);   // rint(x), exact
  const float f = __fsub_rn(xc, n);          // x - rint(x), exact
  float p = fmaf(kExpC3, f, kExpC2);
  p = fmaf(p, f, kExpC1);
  p = fmaf(p, f, kExpC0);
  // t's bits are those of 1.5 * 2^23 plus n; shifted left by 23 only n << 23 remains (mod 2^32).
  const float r = __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
  return x < -125.f ? 0.f : r;
}

// Shared-memory descriptor of an MN-major operand tile written by TMA with 128-byte swizzling:
// rows of 64 16-bit elements along N (128 B), 8-row swizzle atoms of 1024 B stacked along K.
// The stride between 8-row K groups is 1024 B; the tile is a single 64-wide N block, so the
// N-block stride is never used and is given the same value (every address the descriptor can
// form stays inside the 8 KB tile).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1024u >> 4) << 16;   // leading byte offset
  d |= static_cast<uint64_t>(1024u >> 4) << 32;   // stride byte offset (8-row K groups)
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Completion wait that ignores the abort flag (bounded by time only): used on error paths to let
// copies and MMAs already in flight finish before the CTA releases its memory.
__device__ __forceinline__ bool wait_done(uint64_t* bar, uint32_t parity) {
  volatile int no_abort = 0;
  return mbar_wait(bar, parity, &no_abort);
}

__host__ __device__ constexpr uint32_t idesc_f16_bmn(int M, int N, bool is_bf16) {
  return idesc_f16(M, N, is_bf16) | (1u << 16);  // B operand MN-major
}

// Class of 32 keys [kb, kb + 31] for the 32 queries [qa, qb] of one warp: 0 = visible to none of
// them, 2 = every key visible to every query, 1 = mask per element.
__device__ __forceinline__ int half_class(int kb, int L, int qa, int qb, int wh) {
  const int ke = kb + 31;
  if (kb >= L) return 0;
  if (wh < 0) return ke < L ? 2 : 1;
  if (ke < qa - wh || kb > qb + wh) return 0;
  return (ke < L && kb >= qb - wh && ke <= qa + wh) ? 2 : 1;
}

// Masks (class 1) the 32 scores of keys kb..kb+31 for query qi to -inf and returns their max.
// The visible keys of a row form one interval [max(0, qi - wh), min(L - 1, qi + wh)] (wh < 0:
// [0, L - 1]); its intersection with the half is turned into a 32-bit mask with a few integer
// operations, then each score costs one bit test and one select.
__device__ __forceinline__ float masked_max(float (&s)[32], int cls, int kb, int L, int qi, int wh) {
  if (cls == 1) {
    const int lo = max(wh < 0 ? 0 : qi - wh, 0) - kb;           // first visible offset
    const int hi = min(wh < 0 ? L - 1 : qi + wh, L - 1) - kb;   // last visible offset
    const int a = max(lo, 0), b = min(hi, 31);
    // bits a..b set (none when a > b)
    const uint32_t vis = a > b ? 0u : ((0xffffffffu >> (31 - b)) & (0xffffffffu << a));
#pragma unroll
    for (int c = 0; c < 32; ++c)
      if (!((vis >> c) & 1u)) s[c] = -INFINITY;
  }
  float mx[4] = {fmax3(s[0], s[1], s[2]), fmax3(s[3], s[4], s[5]), fmax3(s[6], s[7], s[8]),
                 fmax3(s[9], s[10], s[11])};
#pragma unroll
  for (int c = 12; c < 32; c += 2) mx[(c >> 1) & 3] = fmax3(mx[(c >> 1) & 3], s[c], s[c + 1]);
  return fmax3(mx[0], mx[1], fmaxf(mx[2], mx[3]));
}

// P = exp2(s * scale_log2 - m) of 32 keys as 16 packed 16-bit pairs (zeros when the half is
// not visible); adds the f32 values to the two packed partial sums ps.  sl2 = {scale_log2,
// scale_log2}, nm2 = {-m, -m}.  With kPoly, one pair in four is computed with exp2_poly on the
// FMA pipe and the rest with the MUFU ex2, so the two units share the exponentials.
template <typename T, bool kPoly>
__device__ __forceinline__ void make_p(bool live, const float (&s)[32], uint64_t sl2, uint64_t nm2,
                                       uint64_t (&ps)[2], uint32_t (&w)[16]) {
  // One branch for the whole half (not one per pair), so the 32 exponentials form a single
  // basic block that the compiler can interleave.
  if (!live) {
#pragma unroll
    for (int e = 0; e < 16; ++e) w[e] = 0u;
    return;
  }
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    // Masked scores are -inf: exp2(-inf) = 0 exactly (ex2 and exp2_poly alike).
    float x0, x1;
    f2_unpack(f2_fma(f2_pack(s[2 * e], s[2 * e + 1]), sl2, nm2), x0, x1);
    const bool fma_pipe = kPoly && (e & 3) == 3;
    const float p0 = fma_pipe ? exp2_poly(x0) : ex2(x0);
    const float p1 = fma_pipe ? exp2_poly(x1) : ex2(x1);
    ps[e & 1] = f2_add(ps[e & 1], f2_pack(p0, p1));
    auto v = Elem<T>::pack(p0, p1);
    w[e] = *reinterpret_cast<uint32_t*>(&v);
  }
}

// Evaluates exp2_poly on n floats (device pointers): the test hook that bounds its error.
__global__ void exp2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    y[i] = exp2_poly(x[i]);
}

// The (item, key tile) sequence one CTA processes: items w = blockIdx.x + k * gridDim.x; item w
// is query tile w % n_tiles of head w / n_tiles.  The launch constants (tiles, n_tiles, n_items,
// window) stay in the parameter bank; the next item's record is loaded one item ahead so its
// latency overlaps the current item.
struct Walk {
  int w;  // current item (done when >= n_items)
  int i;  // ordinal of the item within this CTA
  int j;  // key tile within the item
  int s0, L, q0, t_lo, n_kv;
  int2 nxt;

  __device__ __forceinline__ static int2 load(const int2* tiles, int n_tiles, int item) {
    return __ldg(&tiles[item - (item / n_tiles) * n_tiles]);
  }
  __device__ __forceinline__ int head(int n_tiles) const { return w / n_tiles; }
  __device__ __forceinline__ void set(int2 rec, int wh) {
    s0 = rec.x;
    L = rec.y & 0xFFFF;
    q0 = rec.y >> 16;
    int kv_lo = 0, kv_hi = L;
    if (wh >= 0) {
      kv_lo = max(0, q0 - wh);
      kv_hi = min(L, q0 + kBQ + wh);
    }
    t_lo = kv_lo / kBKV;
    n_kv = (kv_hi + kBKV - 1) / kBKV - t_lo;  // >= 1 because q0 < L
  }
  __device__ __forceinline__ void init(const int2* tiles, int n_tiles, int n_items, int wh) {
    w = blockIdx.x;
    i = 0;
    j = 0;
    if (w < n_items) {
      set(load(tiles, n_tiles, w), wh);
      if (w + static_cast<int>(gridDim.x) < n_items) nxt = load(tiles, n_tiles, w + gridDim.x);
    }
  }
  __device__ __forceinline__ bool valid(int n_items) const { return w < n_items; }
  __device__ __forceinline__ bool last_tile() const { return j == n_kv - 1; }
  __device__ __forceinline__ void next(const int2* tiles, int n_tiles, int n_items, int wh) {
    if (++j < n_kv) return;
    j = 0;
    ++i;
    w += gridDim.x;
    if (w < n_items) {
      set(nxt, wh);
      if (w + static_cast<int>(gridDim.x) < n_items) nxt = load(tiles, n_tiles, w + gridDim.x);
    }
  }
};

template <typename T, bool kPoly>
__global__ void __launch_bounds__(kThreads, 2) attn_tc_kernel(const __grid_constant__ CUtensorMap tmQKV,
                                                              T* __restrict__ ctx,
                                                              const int2* __restrict__ tiles,
                                                              int n_tiles, int n_items, int H,
                                                              int window_half, float scale_log2,
                                                              unsigned int* err, long long wait_limit,
                                                              int stall) {
  constexpr bool kBf = Elem<T>::kBf16;
  constexpr uint32_t kIdS = idesc_f16(kBQ, kBKV, kBf);
  constexpr uint32_t kIdO = idesc_f16_bmn(kBQ, kD, kBf);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                        // [2] x 16 KB
  uint8_t* sK = sQ + 2 * kQBytes;            // [kKStages] x 8 KB
  uint8_t* sV = sK + kKStages * kKVBytes;    // [kVStages] x 8 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(sV + kVStages * kKVBytes);
  uint64_t* q_full = bar;          // [2] Q landed
  uint64_t* q_empty = bar + 2;     // [2] last S MMA of the item that read Q completed
  uint64_t* k_full = bar + 4;                 // [kKStages]
  uint64_t* v_full = k_full + kKStages;       // [kVStages]
  uint64_t* s_full = v_full + kVStages;       // [kSBufs] scores in TMEM (K slot free again)
  uint64_t* p_full = s_full + kSBufs;         // [kSBufs] P written over S in TMEM by the 8 softmax warps
  uint64_t* p_empty = p_full + kSBufs;        // [kSBufs] P V MMA of the tile completed (O updated, V slot free)
  uint64_t* o_empty = p_empty + kSBufs;       // [1] the previous item's O read out by the 8 softmax warps
  uint64_t* drain = o_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
    }
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], kSoftmaxWarps);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(o_empty, kSoftmaxWarps);
    for (int b = 0; b < kKStages; ++b) mbar_init(&k_full[b], 1);
    for (int b = 0; b < kVStages; ++b) mbar_init(&v_full[b], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQKV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  static_assert((4 + 3 * kSBufs + 1 + kKStages + kVStages + 1) * 8 + 8 <= 512, "barrier area");
  static_assert(kKStages == kSBufs && kVStages == kSBufs, "K / V slots are released by s_full / p_empty");

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producers
    // Lane 0 loads Q and K, lane 1 loads V; each walks the same tile sequence with its own ring,
    // so a V slot that is still being read never holds back the next K load.
    if (lane < 2) {
      const bool kq = lane == 0;
      Walk wk;
      wk.init(tiles, n_tiles, n_items, window_half);
      bool ok = true;
      // Per-slot record of issued loads (bit = slot issued, parity of its last phase), so that an
      // aborting CTA can let them land before it exits.
      uint32_t q_iss = 0, q_par = 0, iss = 0, par = 0;
      const int stages = kq ? kKStages : kVStages;
      uint64_t* full = kq ? k_full : v_full;
      uint64_t* empty = kq ? s_full : p_empty;
      uint8_t* ring = kq ? sK : sV;
      const int col0 = (kq ? H : 2 * H);
      int rs = 0;
      uint32_t rph = 0;
      while (wk.valid(n_items)) {
        if (kq && wk.j == 0) {
          const int qs = wk.i & 1;
          const uint32_t qph = (wk.i >> 1) & 1;
          if (!mbar_wait(&q_empty[qs], qph ^ 1u, abort_flag, wait_limit)) { ok = false; break; }
          mbar_arrive_expect_tx(&q_full[qs], kQBytes);
          tma_load_2d(sQ + qs * kQBytes, &tmQKV, &q_full[qs], wk.head(n_tiles) * kD, wk.s0 + wk.q0);
          tma_load_2d(sQ + qs * kQBytes + kQBytes / 2, &tmQKV, &q_full[qs], wk.head(n_tiles) * kD,
                      wk.s0 + wk.q0 + kBQ / 2);
          q_iss |= 1u << qs;
          q_par = (q_par & ~(1u << qs)) | (qph << qs);
        }
        const int row = wk.s0 + (wk.t_lo + wk.j) * kBKV;
        if (!mbar_wait(&empty[rs], rph ^ 1u, abort_flag, wait_limit)) { ok = false; break; }
        mbar_arrive_expect_tx(&full[rs], kKVBytes);
        tma_load_2d(ring + rs * kKVBytes, &tmQKV, &full[rs], col0 + wk.head(n_tiles) * kD, row);
        iss |= 1u << rs;
        par = (par & ~(1u << rs)) | (rph << rs);
        if (++rs == stages) { rs = 0; rph ^= 1u; }
        wk.next(tiles, n_tiles, n_items, window_half);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, kErrWaitTimeout);
      }
      // Every issued copy has landed before the CTA can exit, also when another role aborted
      // before consuming it (on the normal path these waits pass at once).
      for (int b = 0; b < 2; ++b)
        if (q_iss & (1u << b)) wait_done(&q_full[b], (q_par >> b) & 1u);
      for (int b = 0; b < stages; ++b)
        if (iss & (1u << b)) wait_done(&full[b], (par >> b) & 1u);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      Walk ws, wp;  // S runs kSBufs tiles ahead of P V
      ws.init(tiles, n_tiles, n_items, window_half);
      wp.init(tiles, n_tiles, n_items, window_half);
      int ks = 0, vs = 0, sb = 0, pb = 0;  // ring slots and score buffers of the next S / P V
      uint32_t kph = 0, vph = 0, pph = 0;
      // Shared-memory descriptors of the ring bases, built once.  Advancing 16 keys (K-major,
      // 32 bytes), 16 rows (MN-major V, 2048 bytes) or one ring slot adds to the 16-byte address
      // field.
      const uint64_t dq0 = smem_desc_sw128(smem_u32(sQ)), dq1 = dq0 + (kQBytes >> 4);
      const uint64_t dk0 = smem_desc_sw128(smem_u32(sK));
      const uint64_t dv0 = smem_desc_sw128_mn(smem_u32(sV));
      // S[sb] = Q K^T over the 64-wide head dim (4 MMAs of K = 16).  S[sb] is free: P V of the
      // tile that last used it was issued before this MMA, in this thread's order.
      auto issue_s = [&]() -> bool {
        const int qs = ws.i & 1;
        if (ws.j == 0 && !mbar_wait(&q_full[qs], (ws.i >> 1) & 1, abort_flag, wait_limit)) return false;
        if (!mbar_wait(&k_full[ks], kph, abort_flag, wait_limit)) return false;
        tc_fence_after();
        const uint64_t aq = qs ? dq1 : dq0;
        const uint64_t bk = dk0 + static_cast<uint64_t>(ks * (kKVBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          tc_mma_f16(tmem_base + sb * kBKV, aq + 2 * kk, bk + 2 * kk, kIdS, kk > 0 ? 1u : 0u);
        // Test hook (rv_debug_stall_attention): the first tile's scores are never signalled, so
        // the softmax warps' bounded wait expires and the launch ends with kErrWaitTimeout.
        if (!(stall && ws.w == static_cast<int>(blockIdx.x) && ws.j == 0)) tc_commit(&s_full[sb]);
        if (ws.last_tile()) tc_commit(&q_empty[qs]);
        if (++ks == kKStages) { ks = 0; kph ^= 1u; }
        if (++sb == kSBufs) sb = 0;
        ws.next(tiles, n_tiles, n_items, window_half);
        return true;
      };
      bool ok = true;
      for (int f = 0; f < kSBufs && ok && ws.valid(n_items); ++f) ok = issue_s();
      while (ok && wp.valid(n_items)) {
        // O (+)= P V: P (16-bit, written over S[pb] in TMEM: 128 lanes x 32 columns) is the A
        // operand, V is MN-major in shared memory (keys x head dim).  An item's first tile
        // overwrites O once the previous item has been read out of it (o_empty; a fresh
        // barrier passes the first item).  S of tile gp + kSBufs reuses S[pb] only after this
        // MMA, in this thread's issue order.
        if ((wp.j == 0 && !mbar_wait(o_empty, (wp.i & 1) ^ 1u, abort_flag, wait_limit)) ||
            !mbar_wait_spin(&p_full[pb], pph, abort_flag, wait_limit) || !mbar_wait(&v_full[vs], vph, abort_flag, wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t bv = dv0 + static_cast<uint64_t>(vs * (kKVBytes >> 4));
#pragma unroll
        for (int kk = 0; kk < kBKV / 16; ++kk)
          tc_mma_f16_ts(tmem_base + kOCol, tmem_base + pb * kBKV + 8 * kk, bv + 128 * kk, kIdO,
                        (wp.j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&p_empty[pb]);
        if (++vs == kVStages) { vs = 0; vph ^= 1u; }
        if (++pb == kSBufs) { pb = 0; pph ^= 1u; }
        wp.next(tiles, n_tiles, n_items, window_half);
        if (ws.valid(n_items)) ok = issue_s();
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(err, kErrWaitTimeout);
      }
      // Every MMA this thread issued completes before TMEM is released.
      tc_commit(drain);
      if (!wait_done(drain, 0)) atomicOr(err, kErrWaitTimeout);
    }
  } else {
    // ---------------------------------------------------------------- softmax
    // Warp w (2..5) owns the 32 query rows of TMEM lane quadrant w % 4 and all 64 keys of each
    // tile: one row per thread, so the row max, the sum and the rescaling stay in the thread.
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row of the item (= TMEM lane)
    const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    Walk wk;
    wk.init(tiles, n_tiles, n_items, window_half);
    // Reference max m (log2 units, kNone until a key is visible) and sum l of the row for the
    // current item.  P = exp2(s - m) accumulates into O in TMEM; m only moves when a tile's max
    // exceeds it by more than kRescale (then O and l are rescaled), so P stays <= 2^kRescale.
    constexpr float kRescale = 8.f;
    constexpr float kNone = -1e30f;
    float m = kNone, l = 0.f;
    // The finished item whose context row is written after the next item's first P, so its last
    // P V MMA completes behind that tile's softmax.
    bool fin = false, fin_live = false;
    int fin_b = 0;
    float fin_l = 0.f;
    uint32_t fin_ph = 0, fin_off = 0;  // fin_off: element offset (T * H < 2^31, host-checked)
    // Score buffer and barrier parity of tile g.
    int b = 0;
    uint32_t ph = 0;
    bool fail = false;  // a wait of this thread expired or another role aborted
    const uint64_t sl2 = f2_pack(scale_log2, scale_log2);

    for (;;) {
      const bool have = wk.valid(n_items);
      const int qi = wk.q0 + r;
      if (have) {
        if (wk.j == 0) {
          m = kNone;
          l = 0.f;
        }
        const int qa = wk.q0 + quad * 32;
        const int kb = (wk.t_lo + wk.j) * kBKV;
        const int cls0 = half_class(kb, wk.L, qa, qa + 31, window_half);
        const int cls1 = half_class(kb + 32, wk.L, qa, qa + 31, window_half);
        // S of tile g is committed after the MMA thread issued P V of tile g - kSBufs, and
        // tcgen05.commit tracks every earlier MMA of that thread: this wait also means that P V
        // of g - kSBufs (and every earlier tile) has updated O, so the rescale and read-out
        // waits on p_empty below (tiles g - 1 and later) target the barrier's current phase.
        fail = fail || !__all_sync(0xffffffffu, mbar_wait(&s_full[b], ph, abort_flag, wait_limit));
        if (fail) break;
        float s0[32], s1[32];
        tc_fence_after();
        tmem_ld32(trow + b * kBKV, s0);
        tmem_ld32(trow + b * kBKV + 32, s1);
        tc_wait_ld();
        float mt = -INFINITY;
        if (cls0) mt = masked_max(s0, cls0, kb, wk.L, qi, window_half);
        if (cls1) mt = fmaxf(mt, masked_max(s1, cls1, kb + 32, wk.L, qi, window_half));
        mt *= scale_log2;
        // A row that has seen no key yet (its O row is 0) adopts the tile's max; a row whose max
        // grew by more than kRescale rescales its O and l (rare: the warp waits for the previous
        // P V into O, then reads, scales and rewrites its 32 lanes x 64 columns).
        const bool need = m != kNone && mt > m + kRescale;
        if (m == kNone) m = fmaxf(m, mt);
        if (__any_sync(0xffffffffu, need)) {
          // P V of tile g - 1: the buffer before b, one phase back when b wrapped around.
          const int pb = b == 0 ? kSBufs - 1 : b - 1;
          const uint32_t pph = b == 0 ? ph ^ 1u : ph;
          fail = !__all_sync(0xffffffffu, mbar_wait(&p_empty[pb], pph, abort_flag, wait_limit));
          if (fail) break;
          tc_fence_after();
          const float alpha = need ? ex2(m - mt) : 1.f;
          float t[32];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            tmem_ld32(trow + kOCol + 32 * h, t);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] *= alpha;
            tmem_st32(trow + kOCol + 32 * h, t);
          }
          tc_wait_st();
          if (need) {
            l *= alpha;
            m = mt;
          }
        }
        // P of the 64 keys as 32 packed 16-bit pairs over the first 32 columns of S[b] (the
        // scores were all read above).
        const uint64_t nm2 = f2_pack(-m, -m);
        uint64_t ps[2] = {0ull, 0ull};  // two packed partial sums (f32 zero bits)
        uint32_t w[16];
        make_p<T, kPoly>(cls0 != 0, s0, sl2, nm2, ps, w);
        tmem_st16(trow + b * kBKV, w);
        make_p<T, kPoly>(cls1 != 0, s1, sl2, nm2, ps, w);
        tmem_st16(trow + b * kBKV + 16, w);
        float p0, p1, p2, p3;
        f2_unpack(ps[0], p0, p1);
        f2_unpack(ps[1], p2, p3);
        l += (p0 + p1) + (p2 + p3);
        tc_wait_st();  // P is in TMEM before the MMA thread may read it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
      }
      if (fin) {
        // Context row = O / l, read from TMEM once the item's last P V completed (p_empty of its
        // score buffer); then O is released for the next item's first P V (o_empty).
        fail = !__all_sync(0xffffffffu, mbar_wait(&p_empty[fin_b], fin_ph, abort_flag, wait_limit));
        if (fail) break;
        const float inv = fin_l > 0.f ? 1.0f / fin_l : 0.f;
        tc_fence_after();
        float t[32];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tmem_ld32(trow + kOCol + 32 * h, t);
          tc_wait_ld();
          if (fin_live) {
            uint4* dst = reinterpret_cast<uint4*>(ctx + fin_off + 32 * h);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = t[8 * c + e] * inv;
              dst[c] = pack8<T>(f);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_empty);
        fin = false;
      }
      if (!have) break;
      if (wk.last_tile()) {
        fin = true;
        fin_live = qi < wk.L;
        fin_b = b;
        fin_ph = ph;
        fin_l = l;
        fin_off = static_cast<uint32_t>((wk.s0 + qi) * H + wk.head(n_tiles) * kD);
      }
      if (++b == kSBufs) {
        b = 0;
        ph ^= 1u;
      }
      wk.next(tiles, n_tiles, n_items, window_half);
    }
    if (fail && lane == 0) {
      *abort_flag = 1;
      atomicOr(err, kErrWaitTimeout);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Test hook state (attention_set_stall): withhold the first score signal of every CTA and use a
// short wait limit, so that a launch ends through the bounded-wait error path.
std::atomic<int> g_stall{0};
std::atomic<long long> g_stall_limit{kWaitLimitCycles};

template <typename T, bool kPoly>
cudaError_t launch_attn_tc(const CUtensorMap& tm, void* ctx, const int2* tiles, int n_tiles,
                           int num_heads, int window_half, float scale, unsigned int* err,
                           cudaStream_t st) {
  static PerDeviceOnce attr_set;  // per-device attribute, set once under a lock
  {
    const cudaError_t e_once = attr_set.run([&]() -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<T, kPoly>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
      if (e != cudaSuccess) return e;
      return cudaSuccess;
    });
    if (e_once != cudaSuccess) return e_once;
  }
  const int n_items = n_tiles * num_heads;
  const int slots = 2 * device_sm_count();
  const int grid = n_items < slots ? n_items : slots;
  const float scale_log2 = scale * 1.4426950408889634f;
  const int stall = g_stall.load(std::memory_order_relaxed);
  const long long limit = stall ? g_stall_limit.load(std::memory_order_relaxed) : kWaitLimitCycles;
  attn_tc_kernel<T, kPoly><<<grid, kThreads, kSmem, st>>>(tm, static_cast<T*>(ctx), tiles, n_tiles, n_items,
                                                          num_heads * kD, window_half, scale_log2, err, limit,
                                                          stall);
  return cudaGetLastError();
}

// Whether the softmax shares its exponentials between the MUFU ex2 and exp2_poly (environment
// RV_ATTN_EXP2_POLY=1), read at every launch.
bool use_exp2_poly() {
  const char* e = std::getenv("RV_ATTN_EXP2_POLY");
  return e && std::strcmp(e, "1") == 0;
}

}  // namespace

cudaError_t attention_varlen_tc(Act act, const void* qkv, void* ctx, int total_tokens,
                                const int2* tiles, int n_tiles, int num_heads, int window_half,
                                float scale, unsigned int* err, cudaStream_t st) {
  if (n_tiles <= 0 || total_tokens <= 0) return cudaSuccess;
  if (int64_t(n_tiles) * num_heads > INT32_MAX ||
      int64_t(total_tokens) * num_heads * kD > INT32_MAX)
    return cudaErrorInvalidValue;
  const int H = num_heads * kD;
  // Rows past the batch read as zeros (TMA out-of-bounds fill), so the last sequence's ragged
  // key tile never sees stale workspace contents.
  CUtensorMap tm;
  if (!make_tmap_2d_16bit(&tm, qkv, act == Act::kBf16, uint64_t(3) * H, uint64_t(total_tokens),
                          uint64_t(3) * H * 2, 64, 64, nullptr))
    return cudaErrorInvalidValue;
  const bool poly = use_exp2_poly();
  if (act == Act::kBf16)
    return poly ? launch_attn_tc<__nv_bfloat16, true>(tm, ctx, tiles, n_tiles, num_heads, window_half, scale, err, st)
                : launch_attn_tc<__nv_bfloat16, false>(tm, ctx, tiles, n_tiles, num_heads, window_half, scale, err, st);
  return poly ? launch_attn_tc<__half, true>(tm, ctx, tiles, n_tiles, num_heads, window_half, scale, err, st)
              : launch_attn_tc<__half, false>(tm, ctx, tiles, n_tiles, num_heads, window_half, scale, err, st);
}

cudaError_t exp2_poly_eval(const float* x, float* y, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 4096);
  exp2_poly_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(x, y, n);
  return cudaGetLastError();
}

void attention_set_stall(int enable, long long wait_limit_cycles) {
  g_stall_limit.store(wait_limit_cycles > 0 ? wait_limit_cycles : kWaitLimitCycles, std::memory_order_relaxed);
  g_stall.store(enable ? 1 : 0, std::memory_order_relaxed);
}

int fill_attention_tiles(const int* cu_seqlens, int n_seqs, int2* out) {
  // Longest sequences first: the persistent CTAs take items in this order (per head), so the
  // items with the most key tiles start first and the short ones fill the end of each wave.
  std::vector<int> order;
  order.reserve(size_t(n_seqs > 0 ? n_seqs : 0));
  for (int b = 0; b < n_seqs; ++b) {
    const int L = cu_seqlens[b + 1] - cu_seqlens[b];
    if (L < 0 || L > kMaxAttnSeq) return -1;
    if (L > 0) order.push_back(b);
  }
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    return cu_seqlens[a + 1] - cu_seqlens[a] > cu_seqlens[b + 1] - cu_seqlens[b];
  });
  int t = 0;
  for (int b : order) {
    const int s0 = cu_seqlens[b], L = cu_seqlens[b + 1] - s0;
    for (int q0 = 0; q0 < L; q0 += kBQ) out[t++] = make_int2(s0, L | (q0 << 16));
  }
  return t;
}

}  // namespace rv
