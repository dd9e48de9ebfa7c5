// gemm_q4.cu -- the 4-bit MatMulNBits projection of a prompt chunk (M > 1 tokens) on the
// 5th-generation tensor cores, and the q/k/v form with QK_PREP in its epilogue.
//
// Replaces the GEMM shader (src/scripts/lfm-engine/kernels.js:70-145) that engine.js runs for
// the q/k/v projections of a prompt chunk (engine.js:202-204) and for o_proj (engine.js:224).
// The shader dequantises each 32-value block to f32, w = (q - zp) * scale, and sums
// f32(x) * w over k in f32.  Here:
//   dequant_q4_kernel  the weights once per call to f16 [n][k] in a workspace (the one
//                      deviation from the shader: w rounded to f16, relative error <= 2^-12);
//   gemm_kernel        y = x . W^T on tcgen05, persistent (one CTA per SM walking 128 x BN
//                      output tiles, BN = 256, 192 or 128; or gemm_pair_kernel, a cluster of two
//                      CTAs per 256 x BN tile sharing one tcgen05.mma.cta_group::2 stream; the
//                      form and width chosen per shape for the shortest makespan over the
//                      SMs): K in 64-wide stages through a 4- to 8-deep TMA
//                      ring (128-byte swizzle, both operands K-major) that runs on across tile
//                      boundaries, f32 accumulation in two BN-column TMEM buffers so that the
//                      epilogue of one tile overlaps the MMAs of the next, one elected lane
//                      issuing the MMAs; eight epilogue warps (two per TMEM lane quarter, heads
//                      of 64 columns dealt alternately; thread = output row) copy their
//                      accumulators out, hand the buffer back, round to
//                      f16 and either store the rows, or run QK_PREP on each 64-column head of
//                      the row (the qkv block never reaches memory): q / k heads normed and
//                      rotated exactly as the QK_PREP shader does (bit-identical given the same
//                      f16 projection), rotated q to q_out, k and v to the cache rows pos0 + m.
// Every mbarrier wait is bounded (about one second): a wait that gives up sets the device error
// word, every role of the CTA stops, the copies and MMAs in flight are waited for, the TMEM is
// freed and the CTA returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "qk_row.cuh"
#include "sm100.cuh"

namespace p2p {
namespace {

using namespace sm100;

constexpr int GBM = 128;  // output rows (tokens) per tile
constexpr int GBK = 64;   // k per stage (one 128-byte swizzled row per operand row)
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, each owning 128 of the 256 columns
constexpr int kTmaWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1;
constexpr int kGemmThreads = 32 * (kEpiWarps + 2);
constexpr uint32_t kATile = GBM * GBK * 2;  // 16 KB
constexpr uint64_t kGemmWaitNs = 1000000000ull;

// Output tile width BN (a multiple of the 64-column head).  PAIR = false: one CTA computes a
// 128 x BN tile; PAIR = true: a cluster of two CTAs computes a 256 x BN tile with one
// tcgen05.mma.cta_group::2 stream, each CTA holding 128 rows of x and BN/2 rows of the weights
// (so each SM moves 2/3 (BN = 256) of the operand bytes per FLOP of the single-CTA tile).  The
// ring takes as many stages as fit in 200 KB of shared memory; two BN-column accumulators per
// CTA, TMEM allocated in powers of 2.
template <int BN, bool PAIR>
struct GemmCfg {
  static_assert(BN == 256 || BN == 192 || BN == 128, "tile width");
  static constexpr int kBRows = PAIR ? BN / 2 : BN;
  static constexpr uint32_t kBTile = kBRows * GBK * 2;
  static constexpr int kStages = int((200u * 1024u) / (kATile + kBTile));
  static constexpr uint32_t kAccCols = 2 * BN <= 256 ? 256 : 512;
  static_assert(kBTile % 1024 == 0, "stage alignment of the 128-byte swizzle");
};

template <int BN, bool PAIR>
struct __align__(1024) GemmSmem {
  static constexpr int ST = GemmCfg<BN, PAIR>::kStages;
  __half a[ST][GBM * GBK];
  __half b[ST][GemmCfg<BN, PAIR>::kBRows * GBK];
  uint64_t full[ST], empty[ST];     // TMA -> MMA, MMA -> TMA (per ring stage)
  uint64_t acc_full[2], acc_empty[2];  // MMA -> epilogue, epilogue(s) -> MMA (per TMEM buffer)
  uint64_t mma_done;                // every MMA of the CTA has completed (teardown)
  uint32_t tmem_base;
  volatile int abort_flag;
  float nw[2 * kHeadDim];  // fused QK_PREP: [q norm | k norm] as f32
};

struct GemmParams {
  int32_t m, n, k;
  int32_t tiles_n, tiles;  // output tiles along n, in all
  __half* y;
  int64_t ld_y, y_off;
  int32_t prep;
  int32_t hq, hkv;
  const __half* norm_w;
  const __half* rope;
  float eps;
  __half* q_out;
  int64_t ld_q;
  __half* k_cache;
  __half* v_cache;
  int64_t kv_cap;
  const uint32_t* meta;
  int32_t pos0;
  int32_t* err;
};

__device__ __forceinline__ bool gemm_wait(volatile int& abort_flag, uint64_t* bar,
                                          uint32_t parity, int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag) return false;
    if (globaltimer_ns() - t0 > kGemmWaitNs) {
      abort_flag = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
}

// A wait of a warp: lane 0 polls, the verdict is shared.
__device__ __forceinline__ bool gemm_wait_warp(volatile int& abort_flag, uint64_t* bar,
                                               uint32_t parity, int32_t* err, int lane) {
  bool r = true;
  if (lane == 0) r = gemm_wait(abort_flag, bar, parity, err);
  return __shfl_sync(0xffffffffu, r ? 1 : 0, 0) != 0;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The epilogue of one tile, by epilogue warp `warp` (0-7): TMEM lane quarter warp & 3 (row
// m0 + quarter * 32 + lane of the output), heads warp >> 2 and (warp >> 2) + 2 of the tile's
// BN / 64.  `acc` is the accumulator buffer's TMEM address.  Once the warp's accumulators are
// in registers `release()` hands the buffer back to the MMA; then the f16 rows are stored, or
// run through QK_PREP (the fused q/k/v form).
template <int BN, class Release>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const float* nw, uint32_t acc,
                                              int m0, int n0, int warp, int lane,
                                              Release release) {
  constexpr int kHeads = BN / kHeadDim;
  const int quarter = warp & 3, half = warp >> 2;
  const uint32_t lane_addr = acc + (uint32_t(quarter * 32) << 16);
  Row64<__half> x[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int hc = half + 2 * j;
    if (hc >= kHeads) break;
    uint32_t v[2][32];
    const uint32_t a = lane_addr + uint32_t(hc * kHeadDim);
    tmem_ld32(a, v[0]);
    tmem_ld32(a + 32, v[1]);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      x[j].w[e] = pack2(__uint_as_float(v[0][2 * e]), __uint_as_float(v[0][2 * e + 1]));
      x[j].w[16 + e] = pack2(__uint_as_float(v[1][2 * e]), __uint_as_float(v[1][2 * e + 1]));
    }
  }
  tc_fence_before();
  __syncwarp();
  release();

  const int m = m0 + quarter * 32 + lane;
  if (m >= p.m) return;
  int64_t pos = 0;
  if (p.prep) {
    pos = int64_t(p.meta ? int(p.meta[0]) : p.pos0) + m;
    if (pos >= p.kv_cap) {  // the cache cannot hold this row: touch nothing, report it
      atomicOr(p.err, kErrPosBeyondCache);
      return;
    }
  }
  const int64_t kv_stride = int64_t(p.hkv) * kHeadDim;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int hc = half + 2 * j;
    const int n = n0 + hc * kHeadDim;
    if (hc >= kHeads || n >= p.n) break;
    __half* dst;
    const int unit = n / kHeadDim;
    if (!p.prep) {
      dst = p.y + int64_t(m) * p.ld_y + p.y_off + n;
    } else if (unit >= p.hq + p.hkv) {  // v head: the cache row, unchanged
      dst = p.v_cache + pos * kv_stride + int64_t(unit - p.hq - p.hkv) * kHeadDim;
    } else {
      const bool isq = unit < p.hq;
      __half* out = isq ? p.q_out + int64_t(m) * p.ld_q + int64_t(unit) * kHeadDim
                        : p.k_cache + pos * kv_stride + int64_t(unit - p.hq) * kHeadDim;
      rotate_row<__half>(x[j], p.norm_w ? nw + (isq ? 0 : kHeadDim) : nullptr, p.eps,
                         p.rope + pos * kHeadDim,
                         [&](int kc, const float(&vals)[8]) { store8(out + 8 * kc, vals); });
      continue;
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      d4[q] = make_uint4(x[j].w[4 * q], x[j].w[4 * q + 1], x[j].w[4 * q + 2], x[j].w[4 * q + 3]);
  }
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  using Cfg = GemmCfg<BN, false>;
  constexpr int GST = Cfg::kStages;
  GemmSmem<BN, false>& s = *reinterpret_cast<GemmSmem<BN, false>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Launched behind the previous kernel of the stream (programmatic dependent launch): nothing
  // it writes (x, the weights, the caches) is read or written before that kernel has completed.
  grid_dependency_wait();
  const int nk = (p.k + GBK - 1) / GBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GST; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], kEpiWarps);
    }
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (p.prep && threadIdx.x < 2 * kHeadDim)
    s.nw[threadIdx.x] = p.norm_w ? to_f32(p.norm_w[threadIdx.x]) : 0.f;
  if (warp == kMmaWarp) tmem_alloc(&s.tmem_base, Cfg::kAccCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == kTmaWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tm_a);
      prefetch_tensormap(&tm_b);
      uint32_t g = 0;  // ring slot counter, continuous across tiles
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.tiles_n) * GBM, n0 = (t % p.tiles_n) * BN;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const uint32_t st = g % GST;
          if (g >= GST && !gemm_wait(s.abort_flag, &s.empty[st], ((g / GST) - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[st], kATile + Cfg::kBTile);
          tma_load_2d(s.a[st], &tm_a, kt * GBK, m0, &s.full[st]);
          tma_load_2d(s.b[st], &tm_b, kt * GBK, n0, &s.full[st]);
        }
      }
      if (!ok) {  // let the copies already in flight land before the CTA exits
        for (uint32_t h = g > GST ? g - GST : 0; h < g; ++h) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s.full[h % GST], (h / GST) & 1) &&
                 globaltimer_ns() - t0 < kGemmWaitNs) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_f16_f32(GBM, BN, 0, 0);
    static_assert(sizeof(s.a[0]) == kATile && sizeof(s.b[0]) == Cfg::kBTile, "tile sizes");
    const uint64_t adesc0 = smem_desc_sw128(smem_u32(s.a[0]), 16, 1024);
    const uint64_t bdesc0 = smem_desc_sw128(smem_u32(s.b[0]), 16, 1024);
    bool ok = true, issued = false;
    uint32_t g = 0;
    int i = 0;  // tiles of this CTA
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++i) {
      const int b = i & 1, u = i >> 1;  // accumulator buffer, its use count
      if (u > 0 && !(ok = gemm_wait_warp(s.abort_flag, &s.acc_empty[b], (u - 1) & 1, p.err, lane))) break;
      tc_fence_after();
      const uint32_t acc = tmem + uint32_t(b * BN);
      for (int kt = 0; kt < nk; ++kt, ++g) {
        const uint32_t st = g % GST;
        if (!(ok = gemm_wait_warp(s.abort_flag, &s.full[st], (g / GST) & 1, p.err, lane))) break;
        tc_fence_after();
        if (elect_one()) {
          // a K16 step is +32 bytes (2 address units) inside the 128-byte swizzled rows; a
          // stage is one tile (bytes / 16 address units) further
          const uint64_t ad = adesc0 + uint64_t(st) * (kATile >> 4),
                         bd = bdesc0 + uint64_t(st) * (Cfg::kBTile >> 4);
#pragma unroll
          for (int kk = 0; kk < GBK / 16; ++kk)
            mma_f16_ss(acc, ad + 2 * kk, bd + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&s.empty[st]);
        }
        issued = true;
        __syncwarp();
      }
      if (ok && elect_one()) mma_commit(&s.acc_full[b]);
      __syncwarp();
    }
    // teardown: no MMA of this CTA may still be running when its TMEM is freed
    if (issued) {
      if (elect_one()) mma_commit(&s.mma_done);
      __syncwarp();
      if (lane == 0) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&s.mma_done, 0) && globaltimer_ns() - t0 < kGemmWaitNs) {
        }
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    int i = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++i) {
      const int b = i & 1, u = i >> 1;
      __syncwarp();  // lanes that skipped the previous tile's rows rejoin before the TMEM loads
      if (!gemm_wait_warp(s.abort_flag, &s.acc_full[b], u & 1, p.err, lane)) break;
      tc_fence_after();
      epilogue_tile<BN>(p, s.nw, tmem + uint32_t(b * BN), (t / p.tiles_n) * GBM,
                        (t % p.tiles_n) * BN, warp, lane, [&] {
                          if (lane == 0) mbar_arrive(&s.acc_empty[b]);
                        });
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kAccCols);
  }
}

// The pair form: a cluster of two CTAs per 256 x BN tile.  The even CTA (rank 0) issues the
// MMAs of both; each CTA's TMA loads its own 128 rows of x and BN/2 rows of the weights into
// its own shared memory, all completing on the even CTA's ring barriers (which expect both
// CTAs' bytes); the even CTA's commits arrive on the ring and accumulator barriers of both
// CTAs (multicast commit); both CTAs' epilogue warps hand an accumulator buffer back on the
// even CTA's barrier (16 arrivals).  Cluster barriers after the barrier setup and before the
// TMEM is freed keep either CTA from touching the other's shared memory out of its lifetime.
template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ GemmParams p) {
  using Cfg = GemmCfg<BN, true>;
  constexpr int GST = Cfg::kStages;
  constexpr uint32_t kStageBytes = kATile + Cfg::kBTile;  // one CTA's share of a ring stage
  extern __shared__ uint8_t smem_raw[];
  GemmSmem<BN, true>& s = *reinterpret_cast<GemmSmem<BN, true>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = int(cluster_id_x()), pairs = int(cluster_count_x());
  grid_dependency_wait();
  const int nk = (p.k + GBK - 1) / GBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GST; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 2 * kEpiWarps);
    }
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (p.prep && threadIdx.x < 2 * kHeadDim)
    s.nw[threadIdx.x] = p.norm_w ? to_f32(p.norm_w[threadIdx.x]) : 0.f;
  if (warp == kMmaWarp) tmem_alloc_pair(&s.tmem_base, Cfg::kAccCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and visible, the pair's TMEM allocated
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == kTmaWarp) {
    // ------------------------------------------------------------------ TMA producer (both)
    if (lane == 0) {
      prefetch_tensormap(&tm_a);
      prefetch_tensormap(&tm_b);
      uint32_t g = 0;
      bool ok = true;
      for (int t = pair; t < p.tiles && ok; t += pairs) {
        const int m0 = (t / p.tiles_n) * (2 * GBM) + int(rank) * GBM;
        const int n0 = (t % p.tiles_n) * BN + int(rank) * Cfg::kBRows;
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const uint32_t st = g % GST;
          if (g >= GST && !gemm_wait(s.abort_flag, &s.empty[st], ((g / GST) - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          const uint32_t full0 = cluster_map(smem_u32(&s.full[st]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&s.full[st], 2 * kStageBytes);
          tma_load_2d_pair(s.a[st], &tm_a, kt * GBK, m0, full0);
          tma_load_2d_pair(s.b[st], &tm_b, kt * GBK, n0, full0);
        }
      }
      if (!ok) {  // let the copies already in flight land before the CTA exits
        if (rank == 0) {
          for (uint32_t h = g > GST ? g - GST : 0; h < g; ++h) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&s.full[h % GST], (h / GST) & 1) &&
                   globaltimer_ns() - t0 < kGemmWaitNs) {
            }
          }
        } else {  // its loads complete on the even CTA's barriers: give them time to land
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 100000) {
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer (even CTA)
    if (rank == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * GBM, BN, 0, 0);
      static_assert(sizeof(s.a[0]) == kATile && sizeof(s.b[0]) == Cfg::kBTile, "tile sizes");
      const uint64_t adesc0 = smem_desc_sw128(smem_u32(s.a[0]), 16, 1024);
      const uint64_t bdesc0 = smem_desc_sw128(smem_u32(s.b[0]), 16, 1024);
      bool ok = true, issued = false;
      uint32_t g = 0;
      int i = 0;
      for (int t = pair; t < p.tiles && ok; t += pairs, ++i) {
        const int b = i & 1, u = i >> 1;
        if (u > 0 &&
            !(ok = gemm_wait_warp(s.abort_flag, &s.acc_empty[b], (u - 1) & 1, p.err, lane)))
          break;
        tc_fence_after();
        const uint32_t acc = tmem + uint32_t(b * BN);
        for (int kt = 0; kt < nk; ++kt, ++g) {
          const uint32_t st = g % GST;
          if (!(ok = gemm_wait_warp(s.abort_flag, &s.full[st], (g / GST) & 1, p.err, lane)))
            break;
          tc_fence_after();
          if (elect_one()) {
            const uint64_t ad = adesc0 + uint64_t(st) * (kATile >> 4),
                           bd = bdesc0 + uint64_t(st) * (Cfg::kBTile >> 4);
#pragma unroll
            for (int kk = 0; kk < GBK / 16; ++kk)
              mma_pair_f16_ss(acc, ad + 2 * kk, bd + 2 * kk, idesc,
                              (kt > 0 || kk > 0) ? 1u : 0u);
            mma_pair_commit(&s.empty[st], 0x3);
          }
          issued = true;
          __syncwarp();
        }
        if (ok && elect_one()) mma_pair_commit(&s.acc_full[b], 0x3);
        __syncwarp();
      }
      if (issued) {  // no MMA of the pair may still run when the TMEM is freed
        if (elect_one()) mma_pair_commit(&s.mma_done, 0x1);
        __syncwarp();
        if (lane == 0) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s.mma_done, 0) && globaltimer_ns() - t0 < kGemmWaitNs) {
          }
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both)
    int i = 0;
    for (int t = pair; t < p.tiles; t += pairs, ++i) {
      const int b = i & 1, u = i >> 1;
      __syncwarp();
      if (!gemm_wait_warp(s.abort_flag, &s.acc_full[b], u & 1, p.err, lane)) break;
      tc_fence_after();
      const uint32_t empty0 = cluster_map(smem_u32(&s.acc_empty[b]), 0);
      epilogue_tile<BN>(p, s.nw, tmem + uint32_t(b * BN),
                        (t / p.tiles_n) * (2 * GBM) + int(rank) * GBM, (t % p.tiles_n) * BN,
                        warp, lane, [&] {
                          if (lane == 0) mbar_arrive_cluster(empty0);
                        });
    }
  }

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while the other may still reach into it
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, Cfg::kAccCols);
  }
}

// Dequantised weights of up to three matrices stacked along n (the q, k and v projections in
// one launch): dst[n][k] = f16((f32(q) - zp) * scale), one 8-value word per thread and step of
// a grid-stride loop, so that a warp stores 512 contiguous bytes per instruction.  Every
// matrix has the same k, so word idx of the stack is element 8 idx of dst.
struct Q4Stack {
  Q4Matrix w[3];
  int64_t end[3];  // cumulative words
  int count;
};

__global__ void __launch_bounds__(256)
    dequant_q4_kernel(const __grid_constant__ Q4Stack st, int32_t k, __half* dst) {
  const int wpr = k >> 3, nb = k >> 5, zr = (nb + 1) >> 1;
  const int64_t total = st.end[st.count - 1];
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int j = idx < st.end[0] ? 0 : idx < st.end[1] ? 1 : 2;
    const Q4Matrix& w = st.w[j];
    const int64_t local = j ? idx - st.end[j - 1] : idx;
    const int64_t n = local / wpr;
    const int wi = int(local - n * wpr), blk = wi >> 2;
    const uint32_t word = w.qweight[local];
    const float sc = __half2float(w.scales[n * nb + blk]);
    const unsigned char* zp = reinterpret_cast<const unsigned char*>(w.zero_points);
    const float z = float((zp[n * zr + (blk >> 1)] >> ((blk & 1) * 4)) & 15u);
    float vals[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) vals[i] = (float((word >> (4 * i)) & 15u) - z) * sc;
    store8(dst + idx * 8, vals);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// f16 [rows][width] with row pitch ld elements, boxes of 64 (k) x box_rows, 128-byte swizzle.
bool map_k_major(CUtensorMap* m, const void* base, int64_t width, int64_t ld, int64_t rows,
                 uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cuuint64_t(width), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {GBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_dequant_q4(const Q4Matrix* ws, int count, int32_t k, void* dst,
                              cudaStream_t s) {
  if (count < 1 || count > 3 || (k % 32) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return cudaErrorInvalidValue;
  Q4Stack st{};
  int64_t words = 0;
  for (int i = 0; i < count; ++i) {
    st.w[i] = ws[i];
    words += int64_t(ws[i].n) * (k / 8);
    st.end[i] = words;
  }
  for (int i = count; i < 3; ++i) st.end[i] = words;
  st.count = count;
  if (words <= 0) return cudaSuccess;
  const int threads = 256;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  // eight resident CTAs of 256 per SM (measured best of 4 / 8 / 16 / 64 per SM)
  const unsigned grid =
      unsigned(std::min<int64_t>((words + threads - 1) / threads, int64_t(std::max(sms, 1)) * 8));
  dequant_q4_kernel<<<grid, threads, 0, s>>>(st, k, static_cast<__half*>(dst));
  return cudaGetLastError();
}

namespace {

GemmParams gemm_params(const GemmArgs& a) {
  GemmParams p{};
  p.m = a.m;
  p.n = a.n;
  p.k = a.k;
  p.y = static_cast<__half*>(a.y);
  p.ld_y = a.ld_y;
  p.y_off = a.y_off;
  p.prep = a.prep;
  p.hq = a.hq;
  p.hkv = a.hkv;
  p.norm_w = static_cast<const __half*>(a.norm_w);
  p.rope = static_cast<const __half*>(a.rope);
  p.eps = a.eps;
  p.q_out = static_cast<__half*>(a.q_out);
  p.ld_q = a.ld_q;
  p.k_cache = static_cast<__half*>(a.k_cache);
  p.v_cache = static_cast<__half*>(a.v_cache);
  p.kv_cap = a.kv_cap;
  p.meta = a.meta;
  p.pos0 = a.pos0;
  p.err = a.err;
  return p;
}

template <int BN>
cudaError_t launch_gemm_bn(const GemmArgs& a, int sms, cudaStream_t stream) {
  CUtensorMap ta, tb;
  if (!map_k_major(&ta, a.x, a.k, a.ld_x, a.m, GBM) ||
      !map_k_major(&tb, a.w16, a.k, a.k, a.n, BN))
    return cudaErrorInvalidValue;
  const int64_t tiles_n = (a.n + BN - 1) / BN, tiles = tiles_n * ((a.m + GBM - 1) / GBM);
  if (tiles > INT32_MAX) return cudaErrorInvalidValue;
  GemmParams p = gemm_params(a);
  p.tiles_n = int32_t(tiles_n);
  p.tiles = int32_t(tiles);
  const size_t smem = sizeof(GemmSmem<BN, false>) + 1024;
  static PerDeviceOnce attrs;
  const cudaError_t attr_err = per_device_once(attrs, [&](int&) {
    return cudaFuncSetAttribute(gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(smem));
  });
  if (attr_err != cudaSuccess) return attr_err;
  // persistent: one CTA per SM (the shared ring admits no second), tiles strided over them
  const dim3 grid(unsigned(std::min<int64_t>(tiles, sms)));
  void* args[] = {&ta, &tb, &p};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at{};
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(&gemm_kernel<BN>), args);
}

template <int BN>
cudaError_t launch_gemm_pair(const GemmArgs& a, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, true>;
  CUtensorMap ta, tb;
  if (!map_k_major(&ta, a.x, a.k, a.ld_x, a.m, GBM) ||
      !map_k_major(&tb, a.w16, a.k, a.k, a.n, Cfg::kBRows))
    return cudaErrorInvalidValue;
  const int64_t tiles_n = (a.n + BN - 1) / BN,
                tiles = tiles_n * ((a.m + 2 * GBM - 1) / (2 * GBM));
  if (tiles > INT32_MAX) return cudaErrorInvalidValue;
  GemmParams p = gemm_params(a);
  p.tiles_n = int32_t(tiles_n);
  p.tiles = int32_t(tiles);
  const size_t smem = sizeof(GemmSmem<BN, true>) + 1024;
  const void* fn = reinterpret_cast<const void*>(&gemm_pair_kernel<BN>);
  cudaLaunchAttribute at[2] = {};
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // persistent: as many pairs as can be resident at once (the SM pairs of the TPCs), tiles
  // strided over them
  static PerDeviceOnce setup;
  int max_pairs = 0;
  const cudaError_t setup_err = per_device_once(setup, [&](int& pairs) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
    if (e != cudaSuccess) return e;
    cfg.gridDim = dim3(2);
    return cudaOccupancyMaxActiveClusters(&pairs, fn, &cfg);
  }, &max_pairs);
  if (setup_err != cudaSuccess) return setup_err;
  if (max_pairs <= 0) return cudaErrorInvalidConfiguration;
  cfg.gridDim = dim3(unsigned(2 * std::min<int64_t>(tiles, max_pairs)));
  cfg.numAttrs = 2;
  void* args[] = {&ta, &tb, &p};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

GemmTiling gemm_tiling(int64_t m, int64_t n, int sms, int force_bn, int force_pair) {
  // The makespan of a persistent launch is its busiest SM's tiles: ceil(tiles / slots) x BN
  // columns of 128 rows per SM (slots = SMs, or SM pairs for the pair form).  The weights
  // carry what the count misses, the operand bytes each SM's TMA must move per FLOP (about 80
  // bytes per clock per SM are sustained; at full MMA rate the single-CTA tile needs 96 (BN
  // 256), 107 (192) and 128 (128), the pair tile 64, 75 and 96), and the pair's fixed cost
  // (cluster barriers, cross-CTA handshakes: about 40 units, 1.5 us).  Fitted to the measured
  // times of every form at 512 / 2048 / 8192 x 2048 / 3072 x 2048.
  const int widths[3] = {256, 192, 128};
  const double weight[2][3] = {{1.0, 1.15, 1.3}, {0.92, 0.97, 1.05}};
  const double fixed[2] = {0.0, 40.0};
  GemmTiling best{256, false};
  double best_cost = -1;
  for (int pair = 0; pair < 2; ++pair) {
    if (force_pair >= 0 && pair != force_pair) continue;
    const int64_t rows = pair ? 2 * GBM : GBM, slots = pair ? std::max(sms / 2, 1) : sms;
    for (int i = 0; i < 3; ++i) {
      if (force_bn && widths[i] != force_bn) continue;
      const int64_t tiles = ((n + widths[i] - 1) / widths[i]) * ((m + rows - 1) / rows);
      const double cost =
          double((tiles + slots - 1) / slots) * widths[i] * weight[pair][i] + fixed[pair];
      if (best_cost < 0 || cost < best_cost) {
        best = GemmTiling{widths[i], pair != 0};
        best_cost = cost;
      }
    }
  }
  return best;
}

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.m <= 0 || a.n <= 0) return cudaSuccess;
  if (a.k <= 0 || (a.k % 8) || (a.ld_x % 8) || (reinterpret_cast<uintptr_t>(a.x) & 15) ||
      (reinterpret_cast<uintptr_t>(a.w16) & 15) || (a.n % kHeadDim))
    return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  sms = std::max(sms, 1);
  const GemmTiling t = gemm_tiling(a.m, a.n, sms, a.bn, a.pair);
  if (t.pair) {
    switch (t.bn) {
      case 256: return launch_gemm_pair<256>(a, stream);
      case 192: return launch_gemm_pair<192>(a, stream);
      case 128: return launch_gemm_pair<128>(a, stream);
    }
  } else {
    switch (t.bn) {
      case 256: return launch_gemm_bn<256>(a, sms, stream);
      case 192: return launch_gemm_bn<192>(a, sms, stream);
      case 128: return launch_gemm_bn<128>(a, sms, stream);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace p2p
