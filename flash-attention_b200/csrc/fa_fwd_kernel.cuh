// Warp-specialised FlashAttention-2 forward for sm_100a (B200).
//
// Replaces the reference's live kernel flash_attention_forward_v6_mma
// (src/forward/forward_v6_mma.cuh:325-412), which computes one 64-row query tile
// per CTA with sm_80 mma.sync.  Same mathematics (softmax(scale*Q K^T [+causal]) V
// with the online softmax of src/softmax/online_softmax.cuh:13-252), new machine:
//
//  * one persistent CTA (512 threads) per SM; a CTA work unit ("tile") is a pair
//    of 128-row query tiles Q0, Q1 of one (batch, head) slice, handed out by an
//    atomic counter in a global workspace (heaviest causal tiles first, grouped by
//    slice so the K/V of the slices in flight stay in L2);
//  * warp 12 : TMA producer - Q0/Q1 once per tile, then K/V tiles through a
//              ring of STAGES shared-memory slots used two at a time: slot pair
//              {V_j, K_j+1} behind one full and one empty mbarrier, so the MMA
//              thread acquires and releases once per key block.  A tile's last V
//              shares its pair with the next tile's K_0 (K_0 alone only for a
//              CTA's first tile);
//  * warp 13 : MMA issuer   - tcgen05.mma S_i = Q_i K_j^T (smem x smem -> TMEM)
//              and O_i += P_i V_j (P from TMEM, V from smem, O in TMEM); the
//              warp runs converged and elect.sync picks the issuing lane.  It
//              issues the next tile's S_i(0) inside the current tile's last key
//              block, so the stream PV0, S0, PV1, S1 runs on across tiles;
//  * warps 0-3 / 4-7 : softmax warpgroup i for query tile i, one thread per row
//              (= TMEM lane): tcgen05.ld of the S row, mask, row max, exp2 with
//              the scale folded in (part of them on the FMA pipe, see exp2_fma),
//              row sum, P rounded to the input type and written back over the S
//              columns with tcgen05.st; lazy O rescale (only when the running max
//              grows by more than 2^8);
//  * warps 8-11 : epilogue warpgroup - O_i from TMEM, 1/l normalise, O store and
//              logsumexp, so the softmax warps go straight on to the next tile;
//  * warps 14-15 idle.  setmaxnreg gives softmax 176 registers per thread, the
//    epilogue 80 and the producer / MMA warpgroup 80 (2*128*176 + 128*80 +
//    128*80 = 64K, the whole register file; every warp of a warpgroup must
//    request the same count).
//
// TMEM (512 columns x 128 lanes of 32 bit): S0 [0,128) S1 [128,256)
// O0 [256,256+D) O1 [256+D,256+2D); P_i aliases the first 64 columns of S_i.
//
// Every mbarrier wait is bounded in time: on expiry the CTA records a status
// code, raises a shared abort flag that ends every other role's waits, drains its
// own copies and MMAs in flight, frees TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "ptx.cuh"
#include "schedule.h"
#include "umma_layout.h"

#ifndef FA_EXP2_FMA_PAIRS
// Of every 8 column pairs of an unmasked S row, how many take exp2 on the FMA
// pipe instead of the MUFU unit (0..8).
#define FA_EXP2_FMA_PAIRS 2
#endif

namespace fa {

struct KernelParams {
  void* O;
  float* LSE;
  int64_t o_stride_b, o_stride_h, o_stride_s;  // elements
  int batch, heads, seq_len;
  float scale_log2;  // softmax_scale * log2(e)
  int n_pairs;       // ceil(N / 256): query-tile pairs per slice
  int n_kv;          // ceil(N / 128): key/value blocks per slice
  int num_tiles;     // batch * heads * n_pairs
  int group_bh;      // slices per scheduling group
  int* tile_counter; // workspace words: [0] unit counter, [1] finished CTAs; both zero at
                    // launch, and the last CTA to finish sets both back to zero
  int* status;       // optional device status word (may be null)
  unsigned long long timeout_ns;
};

// Status codes written to KernelParams::status: 0x100 | where.
enum : int {
  kWaitSched = 1, kWaitQEmpty, kWaitKvEmpty, kWaitQFull, kWaitKvFull, kWaitPFull, kWaitOEmpty,
  kWaitSFull, kWaitOFull, kWaitStatsFull, kWaitStatsEmpty,
};

constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kNumThreads = 512;
constexpr int kEpilogueWarp0 = 8;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only if the max grew by > 2^8

template <int D>
struct Cfg {
  static constexpr uint32_t SW = swizzle_bytes(D);
  static constexpr int CHUNKS = D * 2 / SW;
  static constexpr uint32_t TILE_BYTES = kBlockM * D * 2;  // Q, K and V tiles are all 128 x D
  static constexpr int STAGES = D == 128 ? 4 : (D == 64 ? 6 : 8);  // K/V tile slots
  static constexpr int NPAIRS = STAGES / 2;                           // slot pairs
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t KV_OFF = 2 * TILE_BYTES;
  static constexpr uint32_t STATS_OFF = KV_OFF + STAGES * TILE_BYTES;  // float2 [wg][slot][row]
  static constexpr uint32_t BAR_OFF = STATS_OFF + 2 * 2 * 128 * 8;
  // barrier index layout, see fa_fwd_sm100_kernel
  static constexpr int NBARS = 25 + 2 * NPAIRS;
  static constexpr uint32_t MISC_OFF = BAR_OFF + NBARS * 8;  // tmem slot, sched slots, abort flag
  static constexpr uint32_t SMEM_BYTES = MISC_OFF + 64 + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = 512;
  // TMEM columns of S_i (P_i aliases its first 64 columns) and of O_i.
  __host__ __device__ static constexpr uint32_t s_col(int i) { return 128u * i; }
  __host__ __device__ static constexpr uint32_t o_col(int i) { return 256u + D * i; }
};

__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                             const KernelParams& p, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 31u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > p.timeout_ns) {
        *abort_flag = 1;
        if (p.status) atomicCAS(p.status, 0, 0x100 | where);
        return false;
      }
    }
  }
}

// Bounded wait for roles off the critical path (TMA producer, epilogue): the
// hardware may suspend the waiting thread (up to 20 us per try, it resumes when
// the phase completes), so it does not take issue slots from the softmax warps
// on its SM sub-partition.
__device__ __forceinline__ bool sleepy_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                            const KernelParams& p, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > p.timeout_ns) {
      *abort_flag = 1;
      if (p.status) atomicCAS(p.status, 0, 0x100 | where);
      return false;
    }
  }
}

// Wait of the softmax warps for their next S tile.  It polls once; then the
// hardware may suspend the warp for up to kSoftmaxSleepNs per try, so that a
// waiting softmax warp does not take issue slots from the other warpgroup's
// softmax warp on the same SM sub-partition.  The bound keeps the wake-up late
// by at most that much.
constexpr uint32_t kSoftmaxSleepNs = 200;
__device__ __forceinline__ bool short_sleep_warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                      const KernelParams& p, int where) {
  bool ok = mbar_try_wait(bar, parity);
  if (!ok) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
      if (mbar_try_wait_sleep(bar, parity, kSoftmaxSleepNs)) {
        ok = true;
        break;
      }
      if (*abort_flag) break;
      if (globaltimer_ns() - t0 > p.timeout_ns) {
        *abort_flag = 1;
        if (p.status) atomicCAS(p.status, 0, 0x100 | where);
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ bool sleepy_warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                 const KernelParams& p, int where) {
  const bool ok = sleepy_wait(bar, parity, abort_flag, p, where);
  return __all_sync(0xffffffffu, ok);
}

// Warp-uniform bounded wait: every lane polls, the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          const KernelParams& p, int where) {
  const bool ok = bounded_wait(bar, parity, abort_flag, p, where);
  return __all_sync(0xffffffffu, ok);
}

// Wait that ignores the abort flag; used only to drain work already in flight.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return;
  }
}

template <bool CAUSAL>
__device__ __forceinline__ TileInfo decode_tile(int tile, const KernelParams& p) {
  return decode_unit(tile, p.batch, p.heads, p.seq_len, p.n_pairs, p.n_kv, p.group_bh, kBlockN, CAUSAL);
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// 2^x for two lanes on the FMA pipe (no MUFU).  Cody-Waite style split
// x = n + f with n = round-to-nearest(x) (obtained by adding 1.5*2^23, which
// leaves n in the low mantissa bits), f in [-0.5, 0.5]; 2^f from the polynomial
// 1 + f (c1 + f (c2 + f (c3 + f c4))), fitted for this kernel as the minimax
// relative-error approximation on [-0.5, 0.5] under the constraint p(0) = 1
// (linear programming on a dense grid; max relative error 2.9e-6 evaluated in
// fp32); 2^n applied by adding n to the exponent field.  x is clamped to
// >= -127: a masked score (x = -inf) becomes x = -127, f = 0, p(0) = 1.0, and
// adding n = -127 to the exponent field of 1.0 gives the bit pattern 0, so P is
// exactly +0 there, as on the MUFU path (ex2.approx.ftz of -inf).  The same
// p(0) = 1 makes the row-max element's P exactly 1.  Callers pass x <= 2^8.
constexpr float kExp2C1 = 0.693124235f;
constexpr float kExp2C2 = 0.240240902f;
constexpr float kExp2C3 = 0.0559063852f;
constexpr float kExp2C4 = 0.00958323106f;
__device__ __forceinline__ float2 exp2_fma(float2 x) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -127.0f);
  x.y = fmaxf(x.y, -127.0f);
  const float2 t = add2(x, make_float2(kShift, kShift));
  const float2 n = add2(t, make_float2(-kShift, -kShift));
  const float2 f = fma2(n, make_float2(-1.0f, -1.0f), x);
  float2 q = fma2(make_float2(kExp2C4, kExp2C4), f, make_float2(kExp2C3, kExp2C3));
  q = fma2(q, f, make_float2(kExp2C2, kExp2C2));
  q = fma2(q, f, make_float2(kExp2C1, kExp2C1));
  q = fma2(q, f, make_float2(1.0f, 1.0f));
  float2 r;
  r.x = __uint_as_float(__float_as_uint(t.x) * 8388608u + __float_as_uint(q.x));
  r.y = __uint_as_float(__float_as_uint(t.y) * 8388608u + __float_as_uint(q.y));
  return r;
}

// S_i = Q_i K^T: D/16 MMAs of K = 16 in one asm block with one elect.sync, so
// the issuing warp takes few issue slots from the softmax warps on its SM
// sub-partition.  Step kk adds ((kk*32)/SW)*(128*SW/16) + ((kk*32)%SW)/16 to the
// low word of both descriptors (16-byte units; no carry, shared memory offsets
// stay below 2^18 bytes).
#define FA_SS2(off, pred)                                                   \
  "add.u32 al, %1, " #off ";\n\tadd.u32 bl, %2, " #off ";\n\t"              \
  "mov.b64 ra, {al, %3};\n\tmov.b64 rb, {bl, %3};\n\t"                     \
  "@e tcgen05.mma.cta_group::1.kind::f16 [%0], ra, rb, %4, " #pred ";\n\t"
#define FA_SS2_HEAD                                                         \
  "{\n\t.reg .b32 al, bl;\n\t.reg .b64 ra, rb;\n\t.reg .pred e, pf, pt;\n\t" \
  "setp.ne.b32 pf, %4, %4;\n\tsetp.eq.b32 pt, %4, %4;\n\t"                 \
  "elect.sync _|e, 0xffffffff;\n\t"
template <int D>
__device__ __forceinline__ void mma_chain_s(uint32_t d, uint32_t a_lo, uint32_t b_lo, uint32_t hi, uint32_t idesc) {
  if constexpr (D == 128) {
    static_assert(Cfg<D>::SW == 128, "layout");
    asm volatile(FA_SS2_HEAD FA_SS2(0, pf) FA_SS2(2, pt) FA_SS2(4, pt) FA_SS2(6, pt) FA_SS2(1024, pt)
                     FA_SS2(1026, pt) FA_SS2(1028, pt) FA_SS2(1030, pt) "}" ::"r"(d),
                 "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc)
                 : "memory");
  } else if constexpr (D == 64) {
    static_assert(Cfg<D>::SW == 128, "layout");
    asm volatile(FA_SS2_HEAD FA_SS2(0, pf) FA_SS2(2, pt) FA_SS2(4, pt) FA_SS2(6, pt) "}" ::"r"(d), "r"(a_lo),
                 "r"(b_lo), "r"(hi), "r"(idesc)
                 : "memory");
  } else {
    static_assert(Cfg<D>::SW == 64, "layout");
    asm volatile(FA_SS2_HEAD FA_SS2(0, pf) FA_SS2(2, pt) "}" ::"r"(d), "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc)
                 : "memory");
  }
}
#undef FA_SS2_HEAD
#undef FA_SS2

// O_i += P_i V: 8 MMAs of K = 16 rows of V in one asm block; P step kk is TMEM
// columns [8kk, 8kk+8) of the S_i region, V step kk starts SW 16-byte units on.
#define FA_TS2(acol, boff, pred)                                            \
  "add.u32 ra, %1, " #acol ";\n\tadd.u32 bl, %2, " #boff ";\n\t"            \
  "mov.b64 rb, {bl, %3};\n\t"                                              \
  "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [ra], rb, %4, " #pred ";\n\t"
#define FA_TS2_HEAD                                                         \
  "{\n\t.reg .b32 ra, bl;\n\t.reg .b64 rb;\n\t.reg .pred e, pa, pt;\n\t"    \
  "setp.ne.b32 pa, %5, 0;\n\tsetp.eq.b32 pt, %4, %4;\n\t"                  \
  "elect.sync _|e, 0xffffffff;\n\t"
template <int D>
__device__ __forceinline__ void mma_chain_pv(uint32_t d, uint32_t a, uint32_t b_lo, uint32_t hi, uint32_t idesc,
                                             uint32_t acc) {
  static_assert(kBlockN == 128, "8 steps of 16 keys");
  if constexpr (Cfg<D>::SW == 128) {
    asm volatile(FA_TS2_HEAD FA_TS2(0, 0, pa) FA_TS2(8, 128, pt) FA_TS2(16, 256, pt) FA_TS2(24, 384, pt)
                     FA_TS2(32, 512, pt) FA_TS2(40, 640, pt) FA_TS2(48, 768, pt) FA_TS2(56, 896, pt) "}" ::"r"(d),
                 "r"(a), "r"(b_lo), "r"(hi), "r"(idesc), "r"(acc)
                 : "memory");
  } else {
    static_assert(Cfg<D>::SW == 64, "layout");
    asm volatile(FA_TS2_HEAD FA_TS2(0, 0, pa) FA_TS2(8, 64, pt) FA_TS2(16, 128, pt) FA_TS2(24, 192, pt)
                     FA_TS2(32, 256, pt) FA_TS2(40, 320, pt) FA_TS2(48, 384, pt) FA_TS2(56, 448, pt) "}" ::"r"(d),
                 "r"(a), "r"(b_lo), "r"(hi), "r"(idesc), "r"(acc)
                 : "memory");
  }
}
#undef FA_TS2_HEAD
#undef FA_TS2

template <int D, bool BF16, bool CAUSAL>
__global__ void __launch_bounds__(kNumThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const KernelParams p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::BAR_OFF;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * i; };
  // barrier indices ([2] = per query tile / ring slot)
  constexpr int SCHED_FULL = 0, SCHED_EMPTY = 2, Q_FULL = 4, Q_EMPTY = 6, S_FULL = 8, P_FULL = 10,
                O_FULL = 12, O_EMPTY = 14, DRAIN = 16, STATS_FULL = 17 /* [wg][slot] */,
                STATS_EMPTY = 21 /* [wg][slot] */, KV_FULL = 25 /* [pair] */, KV_EMPTY = 25 + C::NPAIRS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
  volatile int* sched_tile = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 32);
  float2* stats = reinterpret_cast<float2*>(smem + C::STATS_OFF);  // (m*scale*log2e, l)

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(SCHED_FULL + i), 1);
      mbar_init(bar(SCHED_EMPTY + i), 1 + 256 + 128);  // MMA thread + softmax + epilogue
      mbar_init(bar(Q_FULL + i), 1);
      mbar_init(bar(Q_EMPTY + i), 1);
      mbar_init(bar(S_FULL + i), 1);
      mbar_init(bar(P_FULL + i), 128);
      mbar_init(bar(O_FULL + i), 1);
      mbar_init(bar(O_EMPTY + i), 128);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(bar(STATS_FULL + i), 128);
      mbar_init(bar(STATS_EMPTY + i), 128);
    }
    mbar_init(bar(DRAIN), 1);
    for (int s = 0; s < C::NPAIRS; ++s) {
      mbar_init(bar(KV_FULL + s), 1);
      mbar_init(bar(KV_EMPTY + s), 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // Everything above touches only this CTA's shared memory and TMEM; with a
  // programmatic launch the previous kernel on the stream may still be running
  // (and writing Q, K, V, O, LSE or the workspace) until this returns.
  grid_dependency_wait();

  if (warp >= kProducerWarp) {
    setmaxnreg_dec<80>();
    if (warp == kProducerWarp && lane == 0) {
      // ---------------------------------------------------------- TMA producer
      const uint64_t pol_kv = l2_policy_evict_last();
      const uint64_t pol_q = l2_policy_evict_first();
      int tile = blockIdx.x;
      uint32_t sched_cnt = 0, kv_cnt = 0, q_cnt[2] = {0, 0};
      // parity of the last arming of each full barrier, for the abort drain
      uint32_t kv_armed = 0, q_armed = 0, kv_par = 0, q_par = 0;
      bool ok = true;
      auto load_q = [&](int i, const TileInfo& t) -> bool {
        if (!sleepy_wait(bar(Q_EMPTY + i), (q_cnt[i] & 1) ^ 1, abort_flag, p, kWaitQEmpty)) return false;
        const uint32_t fb = bar(Q_FULL + i);
        mbar_arrive_expect_tx(fb, C::TILE_BYTES);
        q_armed |= 1u << i;
        q_par = (q_par & ~(1u << i)) | ((q_cnt[i] & 1) << i);
        const uint32_t dst = sbase + C::Q_OFF + i * C::TILE_BYTES;
#pragma unroll
        for (int c = 0; c < C::CHUNKS; ++c)
          tma_load_4d(dst + c * kBlockM * C::SW, &tmQ, fb, c * int(C::SW / 2), t.pair * 256 + i * 128, t.h, t.b,
                      pol_q);
        ++q_cnt[i];
        return true;
      };
      // Loads V rows [128 v, 128 v + 128) of unit tv into the pair's first slot and
      // K rows [128 k, 128 k + 128) of unit tk into its second (v or k < 0: that
      // slot stays unused).  A unit's last V shares its pair with the next unit's
      // first K, so the MMA warp can start the next unit inside the last step.
      auto load_pair = [&](int v, const TileInfo& tv, int k, const TileInfo& tk) -> bool {
        const uint32_t pr = kv_cnt % C::NPAIRS;
        const uint32_t ph = (kv_cnt / C::NPAIRS) & 1;
        if (!sleepy_wait(bar(KV_EMPTY + pr), ph ^ 1, abort_flag, p, kWaitKvEmpty)) return false;
        const uint32_t fb = bar(KV_FULL + pr);
        mbar_arrive_expect_tx(fb, (v >= 0 ? C::TILE_BYTES : 0u) + (k >= 0 ? C::TILE_BYTES : 0u));
        kv_armed |= 1u << pr;
        kv_par = (kv_par & ~(1u << pr)) | (ph << pr);
        const uint32_t dst = sbase + C::KV_OFF + 2 * pr * C::TILE_BYTES;
        if (v >= 0) {
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_4d(dst + c * kBlockN * C::SW, &tmV, fb, c * int(C::SW / 2), v * kBlockN, tv.h, tv.b, pol_kv);
        }
        if (k >= 0) {
#pragma unroll
          for (int c = 0; c < C::CHUNKS; ++c)
            tma_load_4d(dst + C::TILE_BYTES + c * kBlockN * C::SW, &tmK, fb, c * int(C::SW / 2), k * kBlockN, tk.h,
                        tk.b, pol_kv);
        }
        ++kv_cnt;
        return true;
      };
      // Hands a unit index (or an end marker >= num_tiles) to the other roles.
      auto publish = [&](int unit) -> bool {
        const uint32_t slot = sched_cnt & 1;
        if (!sleepy_wait(bar(SCHED_EMPTY + slot), ((sched_cnt >> 1) & 1) ^ 1, abort_flag, p, kWaitSched)) return false;
        sched_tile[slot] = unit;
        mbar_arrive(bar(SCHED_FULL + slot));
        ++sched_cnt;
        return true;
      };
      ok = publish(tile);
      if (ok && tile < p.num_tiles) {
        TileInfo t = decode_tile<CAUSAL>(tile, p);
        ok = load_q(0, t) && load_pair(-1, t, 0, t);
        if (ok && t.n1 > 0) ok = load_q(1, t);
        while (ok) {
          const int nmax = max(t.n0, t.n1);
          for (int j = 0; ok && j + 1 < nmax; ++j) ok = load_pair(j, t, j + 1, t);
          if (!ok) break;
          // Claim the next unit only now, when its first K tile is due (the ring
          // keeps this thread at most NPAIRS key blocks ahead of the MMAs), so
          // units are handed out in the order CTAs run out of work.
          const int next = atomicAdd(p.tile_counter, 1) + static_cast<int>(gridDim.x);
          const bool has_next = next < p.num_tiles;
          TileInfo tn = t;
          if (has_next) tn = decode_tile<CAUSAL>(next, p);
          ok = publish(next);
          if (!ok) break;
          if (!has_next) {
            // No more units for this CTA: a dependent launch may take the SM as
            // soon as it exits.
            grid_launch_dependents();
            ok = load_pair(nmax - 1, t, -1, t);
            break;
          }
          ok = load_pair(nmax - 1, t, 0, tn) && load_q(0, tn);
          if (ok && tn.n1 > 0) ok = load_q(1, tn);
          t = tn;
        }
      }
      if (*abort_flag) {
        // Let every copy this thread started land before the CTA exits.
        for (int s = 0; s < C::NPAIRS; ++s)
          if (kv_armed & (1u << s)) drain_wait(bar(KV_FULL + s), (kv_par >> s) & 1, 200000000ull);
        for (int i = 0; i < 2; ++i)
          if (q_armed & (1u << i)) drain_wait(bar(Q_FULL + i), (q_par >> i) & 1, 200000000ull);
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------- MMA issuer
      // All 32 lanes run this loop (elect.sync in the MMA chains and commits).  A
      // wait's try_wait is one instruction for the whole warp, so every lane sees
      // the same outcome and the loop stays converged; single arrivals come from
      // lane 0.
      constexpr uint32_t idesc_qk = make_idesc_f16(BF16, kBlockM, kBlockN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(BF16, kBlockM, D, false, true);
      uint32_t sched_cnt = 0, kv_cnt = 0, qf_cnt[2] = {0, 0}, pf_cnt[2] = {0, 0}, oe_cnt[2] = {0, 0};
      bool ok = true;
      // Slot pair pr holds V in slot 2 pr and K in slot 2 pr + 1.
      auto acquire = [&](uint32_t& pr) -> bool {
        pr = kv_cnt % C::NPAIRS;
        const uint32_t ph = (kv_cnt / C::NPAIRS) & 1;
        ++kv_cnt;
        return bounded_wait(bar(KV_FULL + pr), ph, abort_flag, p, kWaitKvFull);
      };
      // Descriptor words: the high word (stride offset, version, swizzle) is the
      // same for every tile of this kernel; low words step by whole tiles.
      constexpr uint64_t kdesc0 = kmajor_desc(0, kBlockM, C::SW, 0);
      constexpr uint64_t vdesc0 = mnmajor_desc(0, kBlockN, C::SW, 0);
      constexpr uint32_t k_hi = static_cast<uint32_t>(kdesc0 >> 32);
      constexpr uint32_t v_hi = static_cast<uint32_t>(vdesc0 >> 32);
      const uint32_t q_lo0 = static_cast<uint32_t>(kdesc0) + ((sbase + C::Q_OFF) >> 4);
      const uint32_t k_lo0 = static_cast<uint32_t>(kdesc0) + ((sbase + C::KV_OFF) >> 4);
      const uint32_t v_lo0 = static_cast<uint32_t>(vdesc0) + ((sbase + C::KV_OFF) >> 4);
      constexpr uint32_t kTileUnits = C::TILE_BYTES >> 4;
      auto issue_s = [&](int i, uint32_t stage) {
        mma_chain_s<D>(tmem_base + C::s_col(i), q_lo0 + i * kTileUnits, k_lo0 + stage * kTileUnits, k_hi,
                       idesc_qk);
      };
      auto issue_pv = [&](int i, uint32_t stage, bool accumulate) {
        mma_chain_pv<D>(tmem_base + C::o_col(i), tmem_base + C::s_col(i), v_lo0 + stage * kTileUnits, v_hi, idesc_pv,
                        accumulate ? 1u : 0u);
      };
      auto wait_p = [&](int i, int j) -> bool {
        if (!bounded_wait(bar(P_FULL + i), pf_cnt[i] & 1, abort_flag, p, kWaitPFull)) return false;
        ++pf_cnt[i];
        if (j == 0) {
          if (!bounded_wait(bar(O_EMPTY + i), (oe_cnt[i] & 1) ^ 1, abort_flag, p, kWaitOEmpty)) return false;
          ++oe_cnt[i];
        }
        tc_fence_after();
        return true;
      };
      // Reads the next unit index from the scheduler ring (-1: the wait failed).
      auto read_unit = [&]() -> int {
        const uint32_t slot = sched_cnt & 1;
        if (!bounded_wait(bar(SCHED_FULL + slot), (sched_cnt >> 1) & 1, abort_flag, p, kWaitSched)) return -1;
        const int unit = sched_tile[slot];
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(SCHED_EMPTY + slot));
        ++sched_cnt;
        return unit;
      };
      // S_i(0) of a unit with n_i key blocks for tile i, from the K tile in slot
      // kslot (Q_i must land first).  I is a compile-time tile index.
      auto issue_first_s = [&](auto I, int n_i, uint32_t kslot) -> bool {
        constexpr int i = decltype(I)::value;
        if (!bounded_wait(bar(Q_FULL + i), qf_cnt[i] & 1, abort_flag, p, kWaitQFull)) return false;
        ++qf_cnt[i];
        tc_fence_after();
        issue_s(i, kslot);
        umma_commit(bar(S_FULL + i));
        if (n_i == 1) umma_commit(bar(Q_EMPTY + i));
        return true;
      };
      int tile = read_unit();
      ok = tile >= 0;
      bool started = false;  // S_i(0) of this unit already issued in the previous unit's last step
      while (ok && tile < p.num_tiles) {
        const TileInfo t = decode_tile<CAUSAL>(tile, p);
        const int n0 = t.n0, n1 = t.n1, nmax = max(n0, n1);
        if (!started) {
          uint32_t pk;
          ok = acquire(pk) && issue_first_s(std::integral_constant<int, 0>{}, n0, 2 * pk + 1) &&
               (n1 == 0 || issue_first_s(std::integral_constant<int, 1>{}, n1, 2 * pk + 1));
          if (!ok) break;
          umma_commit(bar(KV_EMPTY + pk));
        }
        int next = p.num_tiles, next_n0 = 0, next_n1 = 0;
        bool chain = false;
        for (int j = 0; j < nmax; ++j) {
          uint32_t pj;
          if (!acquire(pj)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sv = 2 * pj, skn = 2 * pj + 1;
          const bool last = j == nmax - 1;
          if (last) {
            // The producer publishes the next unit before loading this pair, whose
            // K slot holds that unit's first K tile.
            next = read_unit();
            if (next < 0) { ok = false; break; }
            chain = next < p.num_tiles;
            if (chain) {
              const TileInfo tn = decode_tile<CAUSAL>(next, p);
              next_n0 = tn.n0;
              next_n1 = tn.n1;
            }
          }
          if (j < n0) {
            if (!wait_p(0, j)) { ok = false; break; }
            issue_pv(0, sv, j > 0);
            if (j == n0 - 1) umma_commit(bar(O_FULL + 0));
          }
          if (j + 1 < n0) {
            issue_s(0, skn);
            umma_commit(bar(S_FULL + 0));
            if (j + 2 == n0) umma_commit(bar(Q_EMPTY + 0));
          } else if (last && chain) {
            if (!issue_first_s(std::integral_constant<int, 0>{}, next_n0, skn)) { ok = false; break; }
          }
          if (j < n1) {
            if (!wait_p(1, j)) { ok = false; break; }
            issue_pv(1, sv, j > 0);
            if (j == n1 - 1) umma_commit(bar(O_FULL + 1));
          }
          if (j + 1 < n1) {
            issue_s(1, skn);
            umma_commit(bar(S_FULL + 1));
            if (j + 2 == n1) umma_commit(bar(Q_EMPTY + 1));
          } else if (last && chain && next_n1 > 0) {
            if (!issue_first_s(std::integral_constant<int, 1>{}, next_n1, skn)) { ok = false; break; }
          }
          umma_commit(bar(KV_EMPTY + pj));
        }
        if (!ok) break;
        tile = next;
        started = true;
      }
      // Every MMA issued by this thread completes before TMEM and smem go away.
      umma_commit(bar(DRAIN));
      drain_wait(bar(DRAIN), 0, 200000000ull);
    }
  } else if (warp >= kEpilogueWarp0) {
    setmaxnreg_dec<80>();
    // ------------------------------------------------------------ epilogue warpgroup
    const int row_in_tile = threadIdx.x % 128;
    const uint32_t lane_addr = static_cast<uint32_t>((warp % 4) * 32) << 16;
    uint32_t sched_cnt = 0, o_cnt[2] = {0, 0}, st_cnt[2] = {0, 0};
    while (true) {
      const uint32_t slot = sched_cnt & 1;
      if (!sleepy_warp_wait(bar(SCHED_FULL + slot), (sched_cnt >> 1) & 1, abort_flag, p, kWaitSched)) break;
      const int tile = sched_tile[slot];
      mbar_arrive(bar(SCHED_EMPTY + slot));
      ++sched_cnt;
      if (tile >= p.num_tiles) break;
      const TileInfo t = decode_tile<CAUSAL>(tile, p);
      bool failed = false;
      for (int i = 0; i < 2 && !failed; ++i) {
        if ((i == 0 ? t.n0 : t.n1) == 0) continue;
        const uint32_t ss = st_cnt[i] & 1;
        if (!sleepy_warp_wait(bar(STATS_FULL + 2 * i + ss), (st_cnt[i] >> 1) & 1, abort_flag, p, kWaitStatsFull) ||
            !sleepy_warp_wait(bar(O_FULL + i), o_cnt[i] & 1, abort_flag, p, kWaitOFull)) {
          failed = true;
          break;
        }
        ++o_cnt[i];
        ++st_cnt[i];
        tc_fence_after();
        const float2 ml = stats[(i * 2 + ss) * 128 + row_in_tile];
        mbar_arrive(bar(STATS_EMPTY + 2 * i + ss));
        const float inv_l = 1.f / ml.y;
        const int row = t.pair * 256 + i * 128 + row_in_tile;
        const bool row_ok = row < p.seq_len;
        uint8_t* orow = reinterpret_cast<uint8_t*>(p.O) +
                        2 * (t.b * p.o_stride_b + t.h * p.o_stride_h + static_cast<int64_t>(row) * p.o_stride_s);
        const uint32_t o_addr = tmem_base + lane_addr + C::o_col(i);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          __syncwarp();
          uint32_t r[32];
          tmem_ld32(o_addr + c * 32, r);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = pack2<BF16>(__uint_as_float(r[2 * e]) * inv_l, __uint_as_float(r[2 * e + 1]) * inv_l);
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 4; ++v)
              st_global_v4(orow + c * 64 + v * 16, pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(bar(O_EMPTY + i));
        if (row_ok && p.LSE != nullptr)
          p.LSE[(static_cast<int64_t>(t.b) * p.heads + t.h) * p.seq_len + row] =
              (ml.x + log2f(ml.y)) * 0.69314718055994531f;
      }
      if (failed) break;
    }
    tc_fence_before();
  } else {
    setmaxnreg_inc<176>();
    // ------------------------------------------------------------ softmax warpgroups
    const int wg = warp / 4;                    // query tile 0 or 1
    const int row_in_tile = threadIdx.x % 128;  // = TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>((warp % 4) * 32) << 16;
    const uint32_t s_addr = tmem_base + lane_addr + C::s_col(wg);
    const uint32_t o_addr = tmem_base + lane_addr + C::o_col(wg);
    uint32_t sched_cnt = 0, s_cnt = 0, st_cnt = 0;
    const float sl2 = p.scale_log2;
    while (true) {
      const uint32_t slot = sched_cnt & 1;
      if (!warp_wait(bar(SCHED_FULL + slot), (sched_cnt >> 1) & 1, abort_flag, p, kWaitSched)) break;
      const int tile = sched_tile[slot];
      mbar_arrive(bar(SCHED_EMPTY + slot));
      ++sched_cnt;
      if (tile >= p.num_tiles) break;
      const TileInfo t = decode_tile<CAUSAL>(tile, p);
      const int n = wg == 0 ? t.n0 : t.n1;
      if (n == 0) continue;
      const int row = t.pair * 256 + wg * 128 + row_in_tile;
      float m_ref = -INFINITY, l = 0.f;
      bool failed = false;
      for (int j = 0; j < n; ++j) {
        if (!short_sleep_warp_wait(bar(S_FULL + wg), s_cnt & 1, abort_flag, p, kWaitSFull)) { failed = true; break; }
        ++s_cnt;
        tc_fence_after();
        float s[kBlockN];
#pragma unroll
        for (int c = 0; c < kBlockN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(s_addr + c * 32, r);
#pragma unroll
          for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(r[e]);
        }
        tmem_wait_ld();
        const bool masked = j == n - 1 && (CAUSAL || (p.seq_len % kBlockN) != 0);
        if (masked) {
          const int k0 = j * kBlockN;
          int lim = p.seq_len - 1 - k0;
          if (CAUSAL) lim = min(lim, row - k0);
#pragma unroll
          for (int c = 0; c < kBlockN; ++c) s[c] = c > lim ? -INFINITY : s[c];
        }
        // row max as a breadth-first tree of 3-input maxima (42 independent
        // triples, then 14, 5 and 2), so the scheduler always has independent work
        float m1[43];
#pragma unroll
        for (int k = 0; k < 42; ++k) m1[k] = fmax3(s[3 * k], s[3 * k + 1], s[3 * k + 2]);
        m1[42] = fmaxf(s[126], s[127]);
        float m2[15];
#pragma unroll
        for (int k = 0; k < 14; ++k) m2[k] = fmax3(m1[3 * k], m1[3 * k + 1], m1[3 * k + 2]);
        m2[14] = m1[42];
        float m3[5];
#pragma unroll
        for (int k = 0; k < 5; ++k) m3[k] = fmax3(m2[3 * k], m2[3 * k + 1], m2[3 * k + 2]);
        const float mt = fmax3(fmax3(m3[0], m3[1], m3[2]), m3[3], m3[4]);
        const float m_new = fmaxf(m_ref, mt);
        // Lazy rescale: keep the old reference max unless the row max grew by
        // more than 2^8 (then O and l are scaled by alpha, after P is written).
        float alpha = 1.f;
        bool rescale_warp = false;
        if (j == 0) {
          m_ref = m_new;
        } else {
          const bool need = (m_new - m_ref) * sl2 > kRescaleThreshold;
          rescale_warp = __any_sync(0xffffffffu, need);
          if (need) {
            alpha = ex2_approx((m_ref - m_new) * sl2);
            l *= alpha;
            m_ref = m_new;
          }
        }
        const float mc = m_ref == -INFINITY ? 0.f : m_ref * sl2;
        const float2 scale2 = make_float2(sl2, sl2);
        const float2 neg_mc = make_float2(-mc, -mc);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        // One loop for every block (one copy of this code in the instruction
        // cache).  A masked score (-inf) gives x = -inf, and P = 0 exactly on
        // both exp2 paths (ex2.approx of -inf, and the FMA-pipe exp2's factor 0).
#pragma unroll
        for (int c = 0; c < kBlockN / 64; ++c) {
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float2 x = fma2(make_float2(s[c * 64 + 2 * e], s[c * 64 + 2 * e + 1]), scale2, neg_mc);
            float2 pp;
            if ((e & 7) < FA_EXP2_FMA_PAIRS) {
              pp = exp2_fma(x);
            } else {
              pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
            }
            acc[e & 3] = add2(acc[e & 3], pp);
            pk[e] = pack2<BF16>(pp.x, pp.y);
          }
          tmem_st32(s_addr + c * 32, pk);
        }
        const float2 a = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
        l += a.x + a.y;
        if (rescale_warp) {
          // O_i(j-1) is complete: the commit that signalled S_i(j) covers PV_i(j-1).
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(o_addr + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st32(o_addr + c * 32, r);
          }
        }
        if (j == n - 1) {
          // Hand (m, l) of this row to the epilogue warpgroup.
          const uint32_t ss = st_cnt & 1;
          if (!warp_wait(bar(STATS_EMPTY + 2 * wg + ss), ((st_cnt >> 1) & 1) ^ 1, abort_flag, p, kWaitStatsEmpty)) {
            failed = true;
            break;
          }
          stats[(wg * 2 + ss) * 128 + row_in_tile] = make_float2(mc, l);
          mbar_arrive(bar(STATS_FULL + 2 * wg + ss));
          ++st_cnt;
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar(P_FULL + wg));
      }
      if (failed) break;
    }
    // An abort can leave this warp's last tcgen05.st of P (or of a rescaled O)
    // in flight; it completes before TMEM is freed after the final barrier.
    tmem_wait_st();
    tc_fence_before();
  }

  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    // Every unit claim of this CTA (its producer's atomics, whose results it
    // used) is complete; the CTA that finishes last knows all CTAs' claims are,
    // and leaves the workspace zeroed for the next launch on the stream.
    __threadfence();
    unsigned* done = reinterpret_cast<unsigned*>(p.tile_counter + 1);
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      __threadfence();
      atomicExch(p.tile_counter, 0);
      atomicExch(reinterpret_cast<int*>(done), 0);
    }
  }
}

}  // namespace fa
