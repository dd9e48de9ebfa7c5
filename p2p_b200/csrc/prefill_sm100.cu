// prefill_sm100.cu -- flash attention forward on the 5th-generation tensor cores (sm_100a).
//
// Replaces ATTN for M > 1 (causal GQA prefill over the KV cache,
// src/scripts/lfm-engine/kernels.js:268-319) and VISION_ATTN (bidirectional MHA,
// src/scripts/lfm-engine/vision-kernels.js:176-258).  Same math as the shaders -- scores
// q.k * scale, online softmax (running max / sum), P.V accumulated in f32, out = acc / sum in
// f16 -- reorganised into 128 x 128 tiles on tcgen05 / TMEM / TMA:
//
//   CTA = one (image, q head, 128-row q tile) with 8 warps, two CTAs per SM (NT = 1, the
//   default), or one (image, q head, pair of q tiles) with 12 warps, one CTA per SM (NT = 2);
//   the two independent pipelines of NT = 1 overlap each other better than the two softmax
//   warpgroups of one NT = 2 CTA.  The producer warpgroup (warps 4NT .. 4NT+3) hands registers
//   to the softmax warpgroup(s) with setmaxnreg so the 128-score rows and their 64 packed P
//   pairs stay in registers.
//   warp 4NT    TMA producer: the Q tile(s) once, then K/V tiles of 128 keys (SWIZZLE_128B)
//               into a 3-stage (NT = 1) or 5-stage (NT = 2) ring; mbarrier complete_tx.
//   warp 4NT+1  allocates 256 / 512 TMEM columns and issues tcgen05.mma (cta_group::1, f16)
//               from the converged warp, one elected lane per MMA group:
//                 S_w(j)  = Q_w K_j^T -> TMEM S_w   (M128 N128 K64)
//                 O_w    += P_w(j) V_j -> TMEM O_w  (M128 N64 K128, A = P from TMEM, V an
//                                                  MN-major shared-memory operand)
//               S_w(j+1) is issued as soon as softmax warpgroup w has read S_w(j), so the
//               tensor core computes it while the softmax of tile j runs.
//   warps 0-3   softmax warpgroup 0 (q tile 0; NT = 2: warps 4-7 warpgroup 1, q tile 1): one
//               thread per q row (= TMEM lane).  tcgen05.ld of the S row; mask only on tiles that
//               cross the causal diagonal / the key end; row max with 3-input max; exp2 with
//               the scale folded into one packed FFMA2 and evaluated two at a time, mostly by
//               MUFU.EX2 on f16x2 and for 5 of every 16 pairs by a cubic on the FMA pipe (the
//               result is already the f16 P pair; the row sum adds the same rounded values);
//               all of P(j) is computed before waiting for P(j-1).V to free the P buffer; P
//               is stored into TMEM (tcgen05.st) and the P.V MMA takes its A operand from
//               there, so P never touches shared memory.  O stays in TMEM; it is rescaled (tcgen05.ld/st) only when a
//               row's max grows by more than 2^8 (lazy rescale: the final O / l is exact for
//               any reference max), so most tiles skip it.
//
// Every mbarrier wait is bounded (about one second); a wait that gives up sets the device
// error word, tells the other roles to stop, and the CTA still frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace p2p {
namespace {

using namespace sm100;

constexpr int BM = 128;  // q rows per tile
constexpr int BN = 128;  // keys per tile
constexpr int D = kHeadDim;
// Two layouts, NT = q tiles per CTA:
//  NT = 2: 12 warps (three warpgroups): 0-7 softmax (two warpgroups), 8 TMA, 9 MMA, 10-11
//    idle; 5-stage K/V ring; 512 TMEM columns; one CTA per SM.  The block launches with 168
//    registers per thread (the cap for 384 threads); the producer warpgroup then gives
//    registers back (104 each) and the softmax warpgroups take 192 each:
//    8 * 32 * 192 + 4 * 32 * 104 = 62464 <= 384 * 168 = 64512, so the increase never waits.
//  NT = 1: 8 warps: 0-3 softmax, 4 TMA, 5 MMA, 6-7 idle; 3-stage ring; 256 TMEM columns; two
//    CTAs per SM (112 KB of shared memory each), each with its own pipeline.  Launched with
//    128 registers per thread: 4 * 32 * 192 + 4 * 32 * 64 = 32768 = 256 * 128.
template <int NT>
struct Cfg;
template <>
struct Cfg<2> {
  static constexpr int kStages = 5;  // TMA latency (~2 us under load) spans >1 tile
  static constexpr int kThreads = 384, kMinBlocks = 1, kLaunchRegs = 168;
  static constexpr int kSoftmaxRegs = 192, kProducerRegs = 104;
  static constexpr uint32_t kTmemCols = 512;
};
template <>
struct Cfg<1> {
  static constexpr int kStages = 3;
  static constexpr int kThreads = 256, kMinBlocks = 2, kLaunchRegs = 128;
  static constexpr int kSoftmaxRegs = 192, kProducerRegs = 64;
  static constexpr uint32_t kTmemCols = 256;
};
template <int NT>
constexpr bool split_fits() {
  return NT * 4 * 32 * Cfg<NT>::kSoftmaxRegs + 4 * 32 * Cfg<NT>::kProducerRegs <=
         Cfg<NT>::kThreads * Cfg<NT>::kLaunchRegs;
}
static_assert(split_fits<1>() && split_fits<2>(), "register split");
constexpr uint32_t kTileBytes = BM * D * 2;  // one Q, K or V tile: 16 KB
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr float kRescaleLog2 = 8.0f;  // lazy rescale threshold (factor 256)
#ifndef P2P_POLY_PAIRS
#define P2P_POLY_PAIRS 5
#endif
constexpr int kPolyPairs = P2P_POLY_PAIRS;  // of every 16 exp pairs, these use the cubic

// TMEM columns of q tile w: S at 256w (128 f32 columns), P at 256w + 128 (128 keys as 64
// packed f16x2 columns), O at 256w + 192 (64 f32 columns).
__device__ __forceinline__ uint32_t col_s(int w) { return uint32_t(w) * 256u; }
__device__ __forceinline__ uint32_t col_p(int w) { return uint32_t(w) * 256u + 128u; }
__device__ __forceinline__ uint32_t col_o(int w) { return uint32_t(w) * 256u + 192u; }

// The tiles start on a 1024-byte boundary (128-byte swizzle); every tile is 16 KB.
template <int NT, int ST>
struct __align__(128) SmemT {
  __half q[NT][BM * D];
  __half k[ST][BN * D];
  __half v[ST][BN * D];
  uint64_t bar_q;
  uint64_t k_full[ST], v_full[ST], kv_empty[ST];
  uint64_t s_full[NT], s_free[NT], p_full[NT], pv_done[NT];
  uint32_t tmem_base;
  volatile int abort_flag;
};

struct FlashParams {
  __half* out[kMaxFlashOuts];  // [0] this GPU's output; the others are peers' (NVLink stores)
  int32_t n_out;
  int32_t out_head0;           // head h is written at column (out_head0 + h) * 64
  __half* mc_out;              // non-null: multicast address; one store reaches every GPU
  int64_t ld_o;
  int64_t bs_q, bs_kv;  // rows between images
  int64_t kv_rows_total;
  const uint32_t* meta;
  int32_t* err;
  int32_t pos0_host;
  int32_t s_q, s_kv;
  int32_t hq, hkv;
  int32_t causal;
  int32_t n_qpairs;  // work items along the q rows (pairs of q tiles for NT = 2, tiles for 1)
  float scale_log2;
  int32_t wait_deficit;  // test hook (0 normally): the Q-tile wait then runs out
  // Non-causal 1-D grid (lin != 0): CTA i < n_pair covers item i (a pair of q tiles); CTA
  // n_pair + t covers one 128-row q tile (t & 1) of item n_pair + t / 2.  Items are numbered
  // head-fastest, then q pair, then image.
  int32_t lin, n_pair;
};

// Bounded wait on an mbarrier phase; false when the limit passed or another role gave up.
template <class Smem>
__device__ __forceinline__ bool wait_bar(Smem& s, uint64_t* bar, uint32_t parity,
                                         int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (s.abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      s.abort_flag = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int NT>
__global__ void __launch_bounds__(Cfg<NT>::kThreads, Cfg<NT>::kMinBlocks)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ FlashParams p) {
  using Smem = SmemT<NT, Cfg<NT>::kStages>;
  constexpr int kStages = Cfg<NT>::kStages;
  constexpr int kTmaWarp = 4 * NT, kMmaWarp = 4 * NT + 1;  // the producer warpgroup's roles
  extern __shared__ uint8_t smem_raw[];  // alignment not assumed: checked below
  // NT = 2 pads its dynamic shared memory to reach the 1024-byte boundary; NT = 1 has no room
  // for the pad (two CTAs per SM) and needs the allocation to start there
  const uintptr_t sbase = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
  if (NT == 1 && sbase != reinterpret_cast<uintptr_t>(smem_raw)) {
    if (threadIdx.x == 0) atomicOr(p.err, kErrLayout);
    return;
  }
  Smem& s = *reinterpret_cast<Smem*>(sbase);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Launched behind QK_PREP (programmatic dependent launch): the CTA may be resident before
  // that kernel completes, and reads nothing it writes (q, the cache rows, meta) before this.
  grid_dependency_wait();
  // Grid (heads, q pairs, images), launched in linear order: every head's q pair before the
  // next q pair, and causal q pairs longest first (the last pair sees the most keys), so the
  // block scheduler hands out the work longest-processing-time first.
  int qp, h, b, q_row0;
  bool single = false;
  if (p.lin) {
    const int bx = int(blockIdx.x);
    single = bx >= p.n_pair;
    const int item = single ? p.n_pair + ((bx - p.n_pair) >> 1) : bx;
    h = item % p.hq;
    qp = (item / p.hq) % p.n_qpairs;
    b = item / (p.hq * p.n_qpairs);
    q_row0 = qp * 2 * BM + (single ? ((bx - p.n_pair) & 1) * BM : 0);
  } else {
    qp = p.causal ? (p.n_qpairs - 1 - int(blockIdx.y)) : int(blockIdx.y);
    h = blockIdx.x;
    b = blockIdx.z;
    q_row0 = qp * NT * BM;
  }
  const int kh = h / (p.hq / p.hkv);
  const int pos0 = p.causal ? (p.meta ? int(p.meta[0]) : p.pos0_host) : 0;
  // valid q rows of the two tiles and the keys each needs (causal: 0 .. pos0 + last row)
  const int rows0 = min(BM, p.s_q - q_row0);
  if (rows0 <= 0) return;  // single mode: the second tile of a pair whose q rows end earlier
  const int rows1 = (NT == 1 || single) ? 0 : max(0, min(BM, p.s_q - q_row0 - BM));
  const int64_t kend0 = p.causal ? int64_t(pos0) + q_row0 + rows0 : int64_t(p.s_kv);
  const int64_t kend1 =
      rows1 == 0 ? 0 : (p.causal ? int64_t(pos0) + q_row0 + BM + rows1 : int64_t(p.s_kv));
  const int64_t key_end = kend0 > kend1 ? kend0 : kend1;
  if (p.causal && key_end > p.kv_rows_total) {  // the cache does not hold these keys
    if (threadIdx.x == 0) atomicOr(p.err, kErrPosBeyondCache);
    return;
  }
  // KV tiles each q tile needs (no runtime-indexed local arrays: they would live in memory)
  const int n_kv0 = int((kend0 + BN - 1) / BN);
  const int n_kv1 = int((kend1 + BN - 1) / BN);
  const int n_max = n_kv0 > n_kv1 ? n_kv0 : n_kv1;
  const int last_valid = int(key_end - int64_t(n_max - 1) * BN);  // valid rows of last tile

  if (threadIdx.x == 0) {
    mbar_init(&s.bar_q, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    for (int i = 0; i < NT; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_free[i], 4);
      mbar_init(&s.p_full[i], 4);
      mbar_init(&s.pv_done[i], 1);
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc(&s.tmem_base, Cfg<NT>::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp >= 4 * NT) {
  regs_dec<Cfg<NT>::kProducerRegs>();  // the whole producer warpgroup, before it splits
  if (warp == kTmaWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      const int nq = rows1 > 0 ? 2 : 1;
      mbar_arrive_expect_tx(&s.bar_q, kTileBytes * nq + uint32_t(p.wait_deficit));
      for (int w = 0; w < nq; ++w)
        tma_load_2d(s.q[w], &tm_q, h * D, int32_t(int64_t(b) * p.bs_q + q_row0 + w * BM),
                    &s.bar_q);
      int issued = 0;
      for (int j = 0; j < n_max; ++j) {
        const int st = j % kStages;
        if (j >= kStages && !wait_bar(s, &s.kv_empty[st], ((j / kStages) - 1) & 1, p.err))
          break;
        const int32_t y = int32_t(int64_t(b) * p.bs_kv + int64_t(j) * BN);
        mbar_arrive_expect_tx(&s.k_full[st], kTileBytes);
        tma_load_2d(s.k[st], &tm_k, kh * D, y, &s.k_full[st]);
        mbar_arrive_expect_tx(&s.v_full[st], kTileBytes);
        tma_load_2d(s.v[st], &tm_v, kh * D, y, &s.v_full[st]);
        issued = j + 1;
      }
      if (s.abort_flag) {  // let the copies already in flight land before the CTA exits
        for (int j = max(0, issued - kStages); j < issued; ++j) {
          const uint64_t t0 = globaltimer_ns();
          const int st = j % kStages;
          while (!(mbar_try_wait(&s.k_full[st], (j / kStages) & 1) &&
                   mbar_try_wait(&s.v_full[st], (j / kStages) & 1)) &&
                 globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs this loop with warp-uniform descriptors; lane 0 alone polls the
    // mbarriers and broadcasts the outcome, and one elected lane issues each MMA group and
    // its commit.  (Issuing from a one-lane branch instead lets the softmax warps of the same
    // SM sub-partition starve the issuer of issue slots, and the tensor pipe, which queues
    // very few MMAs, idles.)  All shared-memory descriptors are built once; a k-step only
    // adds to the 14-bit start-address field (16-byte units: +2 per 32-byte K16 step of a
    // 128B-swizzled K-major tile, +128 per 16-row step of the MN-major V tile), which cannot
    // carry out of the field because shared addresses stay below 228 KB.
    {
      constexpr uint32_t idesc_s = idesc_f16_f32(BM, BN, 0, 0);
      constexpr uint32_t idesc_pv = idesc_f16_f32(BM, D, 0, 1);
      // consecutive tiles (Q0/Q1, ring stages) are 16 KB apart: 1024 address units
      static_assert(sizeof(s.q[0]) == 16384 && sizeof(s.k[0]) == 16384, "16 KB tiles");
      const uint64_t qdesc0 = smem_desc_sw128(smem_u32(s.q[0]), 16, 1024);
      const uint64_t kdesc0 = smem_desc_sw128(smem_u32(s.k[0]), 16, 1024);
      const uint64_t vdesc0 = smem_desc_sw128(smem_u32(s.v[0]), 0, 1024);
      auto issue_s = [&](int w, int st) {  // S_w = Q_w K_st^T
        if (elect_one()) {
          const uint64_t qd = qdesc0 + uint64_t(w) * 1024, kd = kdesc0 + uint64_t(st) * 1024;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_f16_ss(tmem + col_s(w), qd + 2 * kk, kd + 2 * kk, idesc_s, kk > 0);
          mma_commit(&s.s_full[w]);
        }
        __syncwarp();
      };
      auto issue_pv = [&](int w, int st, bool acc) {  // O_w += P_w V_st
        if (elect_one()) {
          const uint64_t vd = vdesc0 + uint64_t(st) * 1024;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)  // 16 keys = 8 packed TMEM columns of P
            mma_f16_ts(tmem + col_o(w), tmem + col_p(w) + kk * 8, vd + 128 * kk, idesc_pv,
                       (acc || kk > 0) ? 1u : 0u);
          mma_commit(&s.pv_done[w]);
        }
        __syncwarp();
      };
      auto wait_warp = [&](uint64_t* bar, uint32_t parity) {
        bool r = true;
        if (lane == 0) r = wait_bar(s, bar, parity, p.err);
        return __shfl_sync(0xffffffffu, r ? 1 : 0, 0) != 0;
      };
      bool ok = wait_warp(&s.bar_q, 0) && wait_warp(&s.k_full[0], 0);
      if (ok) {
        tc_fence_after();
        if (n_kv0 > 0) issue_s(0, 0);
        if (NT > 1 && n_kv1 > 0) issue_s(NT - 1, 0);
      }
      for (int j = 0; ok && j < n_max; ++j) {
        const int st = j % kStages;
        // next tile's scores, as soon as each warpgroup has read its S buffer
        if (j + 1 < n_max) {
          const int st1 = (j + 1) % kStages;
          if (!wait_warp(&s.k_full[st1], ((j + 1) / kStages) & 1)) break;
          if (j + 1 < n_kv0) {
            if (!wait_warp(&s.s_free[0], j & 1)) break;
            tc_fence_after();
            issue_s(0, st1);
          }
          if (NT > 1 && j + 1 < n_kv1) {
            if (!wait_warp(&s.s_free[NT - 1], j & 1)) break;
            tc_fence_after();
            issue_s(NT - 1, st1);
          }
        }
        if (!wait_warp(&s.v_full[st], (j / kStages) & 1)) break;
        if (j == n_max - 1 && last_valid < BN) {
          // Rows past the last valid key may hold anything (the cache is not cleared); P is
          // 0 there, but 0 * NaN is NaN, so those V rows are zeroed before the P.V MMA.
          uint4* vrow = reinterpret_cast<uint4*>(s.v[st]);
          for (int i = last_valid * 8 + lane; i < BN * 8; i += 32) vrow[i] = make_uint4(0, 0, 0, 0);
          fence_proxy_async_smem();
          __syncwarp();
        }
        if (j < n_kv0) {
          if (!wait_warp(&s.p_full[0], j & 1)) break;
          tc_fence_after();
          issue_pv(0, st, j > 0);
        }
        if (NT > 1 && j < n_kv1) {
          if (!wait_warp(&s.p_full[NT - 1], j & 1)) break;
          tc_fence_after();
          issue_pv(NT - 1, st, j > 0);
        }
        if (elect_one()) mma_commit(&s.kv_empty[st]);
        __syncwarp();
      }
    }
  }
  } else {
    // ------------------------------------------------------------------ softmax warpgroups
    regs_inc<Cfg<NT>::kSoftmaxRegs>();
    const int w = warp >> 2;           // q tile of this warpgroup
    const int r = threadIdx.x & 127;   // q row within the tile = TMEM lane
    const uint32_t lane_addr = tmem + (uint32_t((warp & 3) * 32) << 16);
    const int nk = w ? n_kv1 : n_kv0;
    const int q_first = q_row0 + w * BM;  // first q row of this tile
    // keys < key_lim are visible to this row
    const int key_lim = p.causal ? pos0 + q_first + r + 1 : p.s_kv;
    const float sl2 = p.scale_log2;
    float m_raw = -INFINITY;  // reference max (raw score units) used for the exponent
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      if (!wait_bar(s, &s.s_full[w], j & 1, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_addr + col_s(w) + c * 32, sv[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.s_free[w]);

      const int key0 = j * BN;
      const bool diag = p.causal ? (key0 + BN - 1 > pos0 + q_first) : (key0 + BN > p.s_kv);
      if (diag) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (key0 + c * 32 + i >= key_lim) sv[c][i] = __float_as_uint(-INFINITY);
      }
      // row max: four independent chains of 3-input max
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          m4[(i >> 1) & 3] = fmax3(m4[(i >> 1) & 3], __uint_as_float(sv[c][i]),
                                   __uint_as_float(sv[c][i + 1]));
      const float mx = fmax3(fmaxf(m4[0], m4[1]), m4[2], m4[3]);
      // lazy rescale: keep the reference max unless this tile exceeds it by > 2^8
      const bool grow = (mx - m_raw) * sl2 > kRescaleLog2;
      const float alpha = grow ? fast_exp2((m_raw - mx) * sl2) : 1.0f;  // 0 on the first tile
      if (grow) m_raw = mx;
      const float neg = (m_raw == -INFINITY) ? 0.f : -m_raw * sl2;
      // P(j) = exp2(s * scale_log2 - m * scale_log2) as 64 packed f16 pairs in registers, all
      // computed before waiting for the P buffer: of every 16 pairs, kPolyPairs go through the
      // FMA-pipe cubic and the rest through the MUFU, so that neither pipe alone bounds the tile.
      uint32_t pk[2][32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = half * 2 + cc;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x0, x1;  // s * scale_log2 - m * scale_log2 for two keys (one FFMA2)
            fma2(__uint_as_float(sv[c][2 * i]), __uint_as_float(sv[c][2 * i + 1]), sl2, neg, x0,
                 x1);
            pk[half][cc * 16 + i] = i < kPolyPairs ? ex2_poly_f16x2(x0, x1) : ex2_f16x2(x0, x1);
          }
        }
      }
      // row sum: f16x2 partial sums of 4 pairs, then two mixed-precision adds into f32
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int half = 0; half < 2; ++half)
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const uint32_t* q4 = &pk[half][4 * g];
          ps[g & 3] = add_f16x2_to_f32(hadd2(hadd2(q4[0], q4[1]), hadd2(q4[2], q4[3])), ps[g & 3]);
        }
      // P buffer w is free (and O holds P(j-1).V) once P(j-1).V has completed
      if (j > 0 && !wait_bar(s, &s.pv_done[w], (j - 1) & 1, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tmem_st32(lane_addr + col_p(w), pk[0]);
      tmem_st32(lane_addr + col_p(w) + 32, pk[1]);
      tmem_st_wait();
      l_run = fmaf(l_run, alpha, (ps[0] + ps[1]) + (ps[2] + ps[3]));
      // rescale O (it holds P(j-1).V) before P(j).V accumulates into it; warp-uniform because
      // tcgen05.ld/st are warp-collective
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        uint32_t ov[2][32];
        tmem_ld32(lane_addr + col_o(w), ov[0]);
        tmem_ld32(lane_addr + col_o(w) + 32, ov[1]);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          ov[0][i] = __float_as_uint(__uint_as_float(ov[0][i]) * alpha);
          ov[1][i] = __float_as_uint(__uint_as_float(ov[1][i]) * alpha);
        }
        tmem_st32(lane_addr + col_o(w), ov[0]);
        tmem_st32(lane_addr + col_o(w) + 32, ov[1]);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[w]);
    }
    // epilogue: O / l -> f16 rows
    if (ok && nk > 0 && wait_bar(s, &s.pv_done[w], (nk - 1) & 1, p.err)) {
      tc_fence_after();
      uint32_t ov[2][32];
      tmem_ld32(lane_addr + col_o(w), ov[0]);
      tmem_ld32(lane_addr + col_o(w) + 32, ov[1]);
      tmem_ld_wait();
      const int rows = w == 0 ? rows0 : rows1;
      if (r < rows) {
        const float inv = 1.0f / l_run;
        uint4 row[D / 8];
#pragma unroll
        for (int i = 0; i < D; i += 8) {
          const int c = i >> 5, e = i & 31;
          row[i / 8] = make_uint4(
              pack_half2(__uint_as_float(ov[c][e]) * inv, __uint_as_float(ov[c][e + 1]) * inv),
              pack_half2(__uint_as_float(ov[c][e + 2]) * inv, __uint_as_float(ov[c][e + 3]) * inv),
              pack_half2(__uint_as_float(ov[c][e + 4]) * inv, __uint_as_float(ov[c][e + 5]) * inv),
              pack_half2(__uint_as_float(ov[c][e + 6]) * inv, __uint_as_float(ov[c][e + 7]) * inv));
        }
        const int64_t off =
            (int64_t(b) * p.bs_q + q_first + r) * p.ld_o + int64_t(p.out_head0 + h) * D;
        if (p.mc_out) {
          // head-sharded prefill with NVLink multicast: each store leaves this GPU once and
          // NVSwitch writes it into every GPU's output buffer
          uint4* dst = reinterpret_cast<uint4*>(p.mc_out + off);
#pragma unroll
          for (int i = 0; i < D / 8; ++i) multimem_st16(dst + i, row[i]);
        } else {
          // this GPU's output first, then every peer's (head-sharded prefill: the rows reach
          // the other GPUs over NVLink here, instead of through a separate all-gather)
          for (int t = 0; t < p.n_out; ++t) {
            uint4* dst = reinterpret_cast<uint4*>(p.out[t] + off);
#pragma unroll
            for (int i = 0; i < D / 8; ++i) dst[i] = row[i];
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg<NT>::kTmemCols);
  }
}

// ---- host side ------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D f16 view [rows][width] (row pitch ld elements), 64 x 128 boxes, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, int64_t width, int64_t ld, int64_t rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {cuuint64_t(width), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One launch of flash_fwd_kernel<NT> (programmatic stream serialization: it may become
// resident while the previous kernel of the stream finishes; see grid_dependency_wait).
template <int NT>
cudaError_t launch_nt(FlashParams& p, CUtensorMap& tq, CUtensorMap& tk, CUtensorMap& tv,
                      dim3 grid, cudaStream_t stream) {
  // NT = 2 pads its shared memory to a 1024-byte boundary; NT = 1 must fit twice per SM
  const size_t smem = sizeof(SmemT<NT, Cfg<NT>::kStages>) + (NT == 2 ? 1024 : 0);
  static PerDeviceOnce attrs;
  const cudaError_t attr_err = per_device_once(attrs, [&](int&) {
    cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel<NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(flash_fwd_kernel<NT>,
                               cudaFuncAttributePreferredSharedMemoryCarveout,
                               int(cudaSharedmemCarveoutMaxShared));
    return e;
  });
  if (attr_err != cudaSuccess) return attr_err;
  void* args[] = {&tq, &tk, &tv, &p};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(Cfg<NT>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at{};
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(&flash_fwd_kernel<NT>), args);
}

// q tiles per CTA: 1 (two independent CTAs per SM; measured faster on every shape: vision
// 97.7 vs 111.3 us, causal S = 2048 37.0 vs 38.1 us, S = 16384 1423 vs 1518 us), or 2 with
// P2P_FLASH_TILES=2 for comparison measurements.
int flash_tiles_per_cta(const FlashArgs&) {
  static const int forced = [] {
    const char* e = getenv("P2P_FLASH_TILES");
    return e ? atoi(e) : 0;
  }();
  return forced == 2 ? 2 : 1;
}

}  // namespace

cudaError_t launch_flash(const FlashArgs& a, cudaStream_t stream) {
  if (a.s_q <= 0 || a.batch <= 0) return cudaSuccess;
  if (a.q_rows_total > INT32_MAX || a.kv_rows_total > INT32_MAX) return cudaErrorInvalidValue;
  CUtensorMap tq, tk, tv;
  const int64_t qw = int64_t(a.hq) * D, kvw = int64_t(a.hkv) * D;
  if (!make_map(&tq, a.q, qw, a.ld_q, a.q_rows_total) ||
      !make_map(&tk, a.k, kvw, a.ld_kv, a.kv_rows_total) ||
      !make_map(&tv, a.v, kvw, a.ld_kv, a.kv_rows_total))
    return cudaErrorInvalidValue;
  FlashParams p{};
  if (a.n_extra_out < 0 || a.n_extra_out > kMaxFlashOuts - 1) return cudaErrorInvalidValue;
  p.out[0] = static_cast<__half*>(a.out);
  for (int t = 0; t < a.n_extra_out; ++t) p.out[1 + t] = static_cast<__half*>(a.extra_out[t]);
  p.n_out = 1 + a.n_extra_out;
  p.out_head0 = a.out_head0;
  p.mc_out = static_cast<__half*>(a.mc_out);
  p.ld_o = a.ld_o;
  p.bs_q = a.batch_stride_q_rows;
  p.bs_kv = a.batch_stride_kv_rows;
  p.kv_rows_total = a.kv_rows_total;
  p.meta = a.meta;
  p.err = a.err;
  p.pos0_host = a.pos0_host;
  p.s_q = a.s_q;
  p.s_kv = a.s_kv;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.causal = a.causal;
  p.scale_log2 = a.scale_log2;
  p.wait_deficit = a.wait_deficit;
  const int nt = flash_tiles_per_cta(a);
  if (nt == 1) {
    p.n_qpairs = (a.s_q + BM - 1) / BM;  // one q tile per CTA
    if (p.n_qpairs > 65535) return cudaErrorInvalidValue;
    return launch_nt<1>(p, tq, tk, tv, dim3(a.hq, p.n_qpairs, a.batch), stream);
  }
  p.n_qpairs = (a.s_q + 2 * BM - 1) / (2 * BM);
  // Non-causal (all items equal): when the items do not fill the last wave of one CTA per SM,
  // the last R pairs run as 2R one-tile CTAs at the end of the same grid (the block scheduler
  // hands them out last, to the SMs that free up first).  A one-tile CTA has its softmax
  // warpgroup alone on the XU pipe and finishes sooner than a pair, so the last wave shortens
  // (this needs 2R <= SMs).
  if (!a.causal && a.num_sms > 0) {
    const int64_t n_items = int64_t(a.hq) * p.n_qpairs * a.batch;
    const int64_t tail = n_items % a.num_sms;
    if (tail > 0 && 2 * tail <= a.num_sms && n_items + tail <= INT32_MAX) {
      p.lin = 1;
      p.n_pair = int32_t(n_items - tail);
      return launch_nt<2>(p, tq, tk, tv, dim3(unsigned(n_items + tail)), stream);
    }
  }
  if (p.n_qpairs > 65535) return cudaErrorInvalidValue;
  return launch_nt<2>(p, tq, tk, tv, dim3(a.hq, p.n_qpairs, a.batch), stream);
}

}  // namespace p2p
