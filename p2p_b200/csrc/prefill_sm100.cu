// prefill_sm100.cu -- flash attention forward on the 5th-generation tensor cores (sm_100a).
//
// Replaces ATTN for M > 1 (causal GQA prefill over the KV cache,
// src/scripts/lfm-engine/kernels.js:268-319) and VISION_ATTN (bidirectional MHA,
// src/scripts/lfm-engine/vision-kernels.js:176-258).  Same math as the shaders -- scores
// q.k * scale, running max / sum online softmax, P.V accumulated in f32, out = acc / sum in
// f16 -- reorganised into 128 x 128 tiles:
//
//   CTA = one (image, q head, 128-row q tile); 6 warps.
//   warp 4     TMA producer: Q tile once, then K/V tiles of 128 keys (SWIZZLE_128B) into a
//              3-stage ring; mbarrier complete_tx signalling.  No multicast.
//   warp 5     allocates 512 TMEM columns; one lane issues tcgen05.mma:
//                S_j = Q K_j^T  -> TMEM S[j%2]   (M=128, N=128, K=64: 4 x K16 MMAs)
//                O_j = P_j V_j  -> TMEM PV[j%2]  (M=128, N=64,  K=128: 8 x K16 MMAs)
//              S_{j+1} is issued before O_j so QK^T of the next tile overlaps the softmax.
//   warps 0-3  softmax, one thread per q row (= TMEM lane): tcgen05.ld of its S row, causal /
//              length mask, running max, exp2, running sum, P_j rounded to f16 into shared
//              memory in the 128B-swizzled K-major layout the MMA reads, then O kept in
//              registers: O = O * alpha + PV_j.  Epilogue: O / sum -> f16 row store.
//
// Every mbarrier wait is bounded (about one second); a wait that gives up sets the device
// error word, tells the other roles to stop, and the CTA still frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

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
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr uint32_t kTileBytes = BM * D * 2;  // one Q, K or V tile: 16 KB
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S[0] 0..127, S[1] 128..255, PV[0] 256..319, PV[1] 320..383.
__device__ __forceinline__ uint32_t col_s(int bf) { return bf ? 128u : 0u; }
__device__ __forceinline__ uint32_t col_pv(int bf) { return bf ? 320u : 256u; }
constexpr int kErrTimeout = 2;
constexpr uint64_t kWaitLimitNs = 1000000000ull;

struct __align__(1024) Smem {
  __half q[BM * D];
  __half k[kStages][BN * D];
  __half v[kStages][BN * D];
  __half p[2][2][BM * 64];  // [buffer][key chunk of 64][128 rows x 64 keys], SW128 K-major
  uint64_t bar_q;
  uint64_t k_full[kStages], v_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], s_empty[2], p_full[2], pv_full[2];
  uint32_t tmem_base;
  volatile int abort_flag;
};

struct FlashParams {
  __half* out;
  int64_t ld_o;
  int64_t bs_q, bs_kv;  // rows between images
  int64_t kv_rows_total;
  const uint32_t* meta;
  int32_t* err;
  int32_t pos0_host;
  int32_t s_q, s_kv;
  int32_t hq, hkv;
  int32_t causal;
  int32_t n_qtiles;
  float scale_log2;
};

// Bounded wait on an mbarrier phase; false when the limit passed or another role gave up.
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

__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ FlashParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.causal ? (p.n_qtiles - 1 - int(blockIdx.x)) : int(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (p.hq / p.hkv);
  const int pos0 = p.causal ? (p.meta ? int(p.meta[0]) : p.pos0_host) : 0;
  const int q_row0 = qt * BM;
  const int q_rows = min(BM, p.s_q - q_row0);
  // keys this tile needs: causal -> 0 .. pos0 + last row; bidirectional -> 0 .. s_kv - 1
  const int64_t key_end = p.causal ? int64_t(pos0) + q_row0 + q_rows : int64_t(p.s_kv);
  if (p.causal && key_end > p.kv_rows_total) {  // the cache does not hold these keys
    if (threadIdx.x == 0) atomicOr(p.err, kErrPosBeyondCache);
    return;
  }
  const int n_kv = int((key_end + BN - 1) / BN);
  const int last_valid = int(key_end - int64_t(n_kv - 1) * BN);  // valid rows of last tile

  if (threadIdx.x == 0) {
    mbar_init(&s.bar_q, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 4);
      mbar_init(&s.p_full[i], 4);
      mbar_init(&s.pv_full[i], 1);
    }
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(&s.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      mbar_arrive_expect_tx(&s.bar_q, kTileBytes);
      tma_load_2d(s.q, &tm_q, h * D, int32_t(int64_t(b) * p.bs_q + q_row0), &s.bar_q);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
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
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = idesc_f16_f32(BM, BN, 0, 0);
    constexpr uint32_t idesc_pv = idesc_f16_f32(BM, D, 0, 1);
    const uint32_t q_addr = smem_u32(s.q);
    bool ok = wait_bar(s, &s.bar_q, 0, p.err);
    auto issue_s = [&](int j) -> bool {
      const int st = j % kStages, bf = j & 1;
      if (!wait_bar(s, &s.k_full[st], (j / kStages) & 1, p.err)) return false;
      if (j >= 2 && !wait_bar(s, &s.s_empty[bf], ((j >> 1) - 1) & 1, p.err)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_addr = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_f16_ss(tmem + col_s(bf), smem_desc_sw128(q_addr + kk * 32, 16, 1024),
                     smem_desc_sw128(k_addr + kk * 32, 16, 1024), idesc_s, kk > 0);
        mma_commit(&s.s_full[bf]);
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = issue_s(0);
    for (int j = 0; ok && j < n_kv; ++j) {
      if (j + 1 < n_kv && !issue_s(j + 1)) break;
      const int st = j % kStages, bf = j & 1;
      if (!wait_bar(s, &s.v_full[st], (j / kStages) & 1, p.err)) break;
      if (j == n_kv - 1 && last_valid < BN) {
        // Rows past the last valid key may hold anything (the cache is not cleared); P is 0
        // there, but 0 * NaN is NaN, so those V rows are zeroed before the P.V MMA.
        uint4* vrow = reinterpret_cast<uint4*>(s.v[st]);
        for (int i = last_valid * 8 + lane; i < BN * 8; i += 32) vrow[i] = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (!wait_bar(s, &s.p_full[bf], (j >> 1) & 1, p.err)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_addr = smem_u32(s.v[st]);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t pa = smem_u32(s.p[bf][kk >> 2]) + (kk & 3) * 32;
          mma_f16_ss(tmem + col_pv(bf), smem_desc_sw128(pa, 16, 1024),
                     smem_desc_sw128(v_addr + kk * 2048, 0, 1024), idesc_pv, kk > 0);
        }
        mma_commit(&s.pv_full[bf]);
        mma_commit(&s.kv_empty[st]);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------ softmax warps 0-3
    const int r = threadIdx.x;  // q row within the tile = TMEM lane
    const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
    const int64_t qpos = int64_t(pos0) + q_row0 + r;
    float m_run = -1e30f, l_run = 0.f, alpha_prev = 0.f;
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    bool ok = true;
    auto fold_pv = [&](int j) -> bool {  // O = O * alpha_j + PV_j
      const int bf = j & 1;
      if (!wait_bar(s, &s.pv_full[bf], (j >> 1) & 1, p.err)) return false;
      tc_fence_after();
      uint32_t pv[2][32];
      tmem_ld32(lane_addr + col_pv(bf), pv[0]);
      tmem_ld32(lane_addr + col_pv(bf) + 32, pv[1]);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        o[i] = fmaf(o[i], alpha_prev, __uint_as_float(pv[0][i]));
        o[32 + i] = fmaf(o[32 + i], alpha_prev, __uint_as_float(pv[1][i]));
      }
      return true;
    };
    for (int j = 0; j < n_kv; ++j) {
      const int bf = j & 1;
      if (!wait_bar(s, &s.s_full[bf], (j >> 1) & 1, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_addr + col_s(bf) + c * 32, sv[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.s_empty[bf]);

      const int64_t key0 = int64_t(j) * BN;
      const bool need_mask = p.causal ? (key0 + BN - 1 > int64_t(pos0) + q_row0)
                                      : (key0 + BN > int64_t(p.s_kv));
      const int64_t key_lim = p.causal ? qpos + 1 : int64_t(p.s_kv);  // keys < key_lim
      float mx = m_run;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = __uint_as_float(sv[c][i]) * p.scale_log2;
          if (need_mask && key0 + c * 32 + i >= key_lim) x = -INFINITY;
          sv[c][i] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      const float alpha = fast_exp2(m_run - mx);
      m_run = mx;
      float psum = 0.f;
      uint8_t* prow = reinterpret_cast<uint8_t*>(s.p[bf][0]) + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = fast_exp2(__uint_as_float(sv[c][2 * i]) - mx);
          const float p1 = fast_exp2(__uint_as_float(sv[c][2 * i + 1]) - mx);
          psum += p0 + p1;
          packed[i] = pack_half2(p0, p1);
        }
        // keys c*32 .. c*32+31 -> chunk c/2, 16-byte pieces (c%2)*4 .. +3, swizzled by row
        uint8_t* chunk = prow + (c >> 1) * (BM * 128);
#pragma unroll
        for (int pc = 0; pc < 4; ++pc) {
          const int piece = (c & 1) * 4 + pc;
          *reinterpret_cast<uint4*>(chunk + ((piece ^ (r & 7)) << 4)) =
              make_uint4(packed[4 * pc], packed[4 * pc + 1], packed[4 * pc + 2],
                         packed[4 * pc + 3]);
        }
      }
      l_run = fmaf(l_run, alpha, psum);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[bf]);
      if (j > 0 && !fold_pv(j - 1)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok && fold_pv(n_kv - 1) && r < q_rows) {
      const float inv = 1.0f / l_run;
      __half* dst = p.out + (int64_t(b) * p.bs_q + q_row0 + r) * p.ld_o + int64_t(h) * D;
#pragma unroll
      for (int i = 0; i < D; i += 8)
        *reinterpret_cast<uint4*>(dst + i) =
            make_uint4(pack_half2(o[i] * inv, o[i + 1] * inv),
                       pack_half2(o[i + 2] * inv, o[i + 3] * inv),
                       pack_half2(o[i + 4] * inv, o[i + 5] * inv),
                       pack_half2(o[i + 6] * inv, o[i + 7] * inv));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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
  p.out = static_cast<__half*>(a.out);
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
  p.n_qtiles = (a.s_q + BM - 1) / BM;
  p.scale_log2 = a.scale_log2;
  const size_t smem = sizeof(Smem) + 1024;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(flash_fwd_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  });
  if (attr_err != cudaSuccess) return attr_err;
  dim3 grid(p.n_qtiles, a.hq, a.batch);
  void* args[] = {&tq, &tk, &tv, &p};
  return cudaLaunchKernel(reinterpret_cast<const void*>(&flash_fwd_kernel), grid,
                          dim3(kThreads), args, smem, stream);
}

}  // namespace p2p
