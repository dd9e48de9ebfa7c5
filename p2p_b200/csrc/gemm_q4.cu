// gemm_q4.cu -- the 4-bit MatMulNBits projection of a prompt chunk (M > 1 tokens) on the
// 5th-generation tensor cores, and the q/k/v form with QK_PREP in its epilogue.
//
// Replaces the GEMM shader (src/scripts/lfm-engine/kernels.js:70-145) that engine.js runs for
// the q/k/v projections of a prompt chunk (engine.js:202-204) and for o_proj (engine.js:224).
// The shader dequantises each 32-value block to f32, w = (q - zp) * scale, and sums
// f32(x) * w over k in f32.  Here:
//   dequant_q4_kernel  the weights once per call to f16 [n][k] in a workspace (the one
//                      deviation from the shader: w rounded to f16, relative error <= 2^-12);
//   gemm_kernel        y = x . W^T on tcgen05: 128 x 256 output tiles, K in 64-wide stages
//                      through a 4-deep TMA ring (128-byte swizzle, both operands K-major),
//                      f32 accumulation in 256 TMEM columns, one elected lane issuing the MMAs;
//                      the epilogue warps (thread = output row = TMEM lane) round to f16 and
//                      either store the rows, or run QK_PREP on each 64-column head of the row
//                      (the qkv block never reaches memory): q / k heads normed and rotated
//                      exactly as the QK_PREP shader does (bit-identical given the same f16
//                      projection), rotated q to q_out, k and v to the cache rows pos0 + m.
// Every mbarrier wait is bounded (about one second): a wait that gives up sets the device error
// word, the CTA stops its roles, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "qk_row.cuh"
#include "sm100.cuh"

namespace p2p {
namespace {

using namespace sm100;

constexpr int GBM = 128;  // output rows (tokens) per tile
constexpr int GBN = 256;  // output columns per tile (four 64-column heads)
constexpr int GBK = 64;   // k per stage (one 128-byte swizzled row per operand row)
constexpr int GST = 4;    // ring depth
constexpr int kGemmThreads = 192;  // warps 0-3 epilogue (TMEM lane quarters), 4 TMA, 5 MMA
constexpr uint32_t kATile = GBM * GBK * 2;  // 16 KB
constexpr uint32_t kBTile = GBN * GBK * 2;  // 32 KB
constexpr uint32_t kAccCols = GBN;          // f32 accumulator columns
constexpr uint64_t kGemmWaitNs = 1000000000ull;

struct __align__(1024) GemmSmem {
  __half a[GST][GBM * GBK];
  __half b[GST][GBN * GBK];
  uint64_t full[GST], empty[GST], acc_full;
  uint32_t tmem_base;
  volatile int abort_flag;
  float nw[2 * kHeadDim];  // fused QK_PREP: [q norm | k norm] as f32
};

struct GemmParams {
  int32_t m, n, k;
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

__device__ __forceinline__ bool gemm_wait(GemmSmem& s, uint64_t* bar, uint32_t parity,
                                          int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (s.abort_flag) return false;
    if (globaltimer_ns() - t0 > kGemmWaitNs) {
      s.abort_flag = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  GemmSmem& s = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Launched behind the previous kernel of the stream (programmatic dependent launch): nothing
  // it writes (x, the caches) is read or written before that kernel has completed.
  grid_dependency_wait();
  const int n0 = int(blockIdx.x) * GBN, m0 = int(blockIdx.y) * GBM;
  const int nk = (p.k + GBK - 1) / GBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < GST; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.acc_full, 1);
    s.abort_flag = 0;
    fence_barrier_init();
  }
  if (p.prep && threadIdx.x < 2 * kHeadDim)
    s.nw[threadIdx.x] = p.norm_w ? to_f32(p.norm_w[threadIdx.x]) : 0.f;
  if (warp == 5) tmem_alloc(&s.tmem_base, kAccCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tm_a);
      prefetch_tensormap(&tm_b);
      int issued = 0;
      for (int kt = 0; kt < nk; ++kt) {
        const int st = kt % GST;
        if (kt >= GST && !gemm_wait(s, &s.empty[st], ((kt / GST) - 1) & 1, p.err)) break;
        mbar_arrive_expect_tx(&s.full[st], kATile + kBTile);
        tma_load_2d(s.a[st], &tm_a, kt * GBK, m0, &s.full[st]);
        tma_load_2d(s.b[st], &tm_b, kt * GBK, n0, &s.full[st]);
        issued = kt + 1;
      }
      if (s.abort_flag) {  // let the copies already in flight land before the CTA exits
        for (int kt = max(0, issued - GST); kt < issued; ++kt) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s.full[kt % GST], (kt / GST) & 1) &&
                 globaltimer_ns() - t0 < kGemmWaitNs) {
          }
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_f16_f32(GBM, GBN, 0, 0);
    static_assert(sizeof(s.a[0]) == 16384 && sizeof(s.b[0]) == 32768, "tile sizes");
    const uint64_t adesc0 = smem_desc_sw128(smem_u32(s.a[0]), 16, 1024);
    const uint64_t bdesc0 = smem_desc_sw128(smem_u32(s.b[0]), 16, 1024);
    bool ok = true;
    for (int kt = 0; kt < nk && ok; ++kt) {
      const int st = kt % GST;
      bool r = true;
      if (lane == 0) r = gemm_wait(s, &s.full[st], (kt / GST) & 1, p.err);
      ok = __shfl_sync(0xffffffffu, r ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        // a K16 step is +32 bytes (2 address units) inside the 128-byte swizzled rows; a
        // stage is 1024 (A) / 2048 (B) address units further
        const uint64_t ad = adesc0 + uint64_t(st) * 1024, bd = bdesc0 + uint64_t(st) * 2048;
#pragma unroll
        for (int kk = 0; kk < GBK / 16; ++kk)
          mma_f16_ss(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kt > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&s.empty[st]);
      }
      __syncwarp();
    }
    if (ok && elect_one()) mma_commit(&s.acc_full);
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int row = warp * 32 + lane;  // = TMEM lane
    const int m = m0 + row;
    const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
    bool ok = gemm_wait(s, &s.acc_full, 0, p.err);
    ok = __all_sync(0xffffffffu, ok);
    int64_t pos = 0;
    bool row_ok = m < p.m;
    if (p.prep && row_ok) {
      pos = int64_t(p.meta ? int(p.meta[0]) : p.pos0) + m;
      if (pos >= p.kv_cap) {  // the cache cannot hold this row: touch nothing, report it
        atomicOr(p.err, kErrPosBeyondCache);
        row_ok = false;
      }
    }
    if (ok) {
      tc_fence_after();
      const int64_t kv_stride = int64_t(p.hkv) * kHeadDim;
      for (int hc = 0; hc < GBN / kHeadDim; ++hc) {
        const int n = n0 + hc * kHeadDim;
        if (n >= p.n) break;  // the same for every thread of the CTA
        uint32_t v[2][32];
        tmem_ld32(lane_addr + hc * kHeadDim, v[0]);
        tmem_ld32(lane_addr + hc * kHeadDim + 32, v[1]);
        tmem_ld_wait();
        if (!row_ok) continue;
        // the f16 projection row (what the GEMM shader stores)
        Row64<__half> x;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          x.w[e] = pack2(__uint_as_float(v[0][2 * e]), __uint_as_float(v[0][2 * e + 1]));
          x.w[16 + e] = pack2(__uint_as_float(v[1][2 * e]), __uint_as_float(v[1][2 * e + 1]));
        }
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
          rotate_row<__half>(x, p.norm_w ? s.nw + (isq ? 0 : kHeadDim) : nullptr, p.eps,
                             p.rope + pos * kHeadDim,
                             [&](int kc, const float(&vals)[8]) { store8(out + 8 * kc, vals); });
          continue;
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          d4[i] = make_uint4(x.w[4 * i], x.w[4 * i + 1], x.w[4 * i + 2], x.w[4 * i + 3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kAccCols);
  }
}

// Dequantised weights: dst[n][k] = f16((f32(q) - zp) * scale), one 8-value word per thread.
__global__ void dequant_q4_kernel(const Q4Matrix w, int32_t k, __half* dst) {
  const int wpr = k >> 3, nb = k >> 5, zr = (nb + 1) >> 1;
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= int64_t(w.n) * wpr) return;
  const int64_t n = idx / wpr;
  const int wi = int(idx % wpr), blk = wi >> 2;
  const uint32_t word = w.qweight[idx];
  const float sc = __half2float(w.scales[n * nb + blk]);
  const uint32_t zb =
      reinterpret_cast<const unsigned char*>(w.zero_points)[n * zr + (blk >> 1)];
  const float z = float((zb >> ((blk & 1) * 4)) & 15u);
  float vals[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) vals[i] = (float((word >> (4 * i)) & 15u) - z) * sc;
  store8(dst + n * k + wi * 8, vals);
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

cudaError_t launch_dequant_q4(const Q4Matrix& w, int32_t k, void* dst, cudaStream_t s) {
  const int64_t words = int64_t(w.n) * (k / 8);
  if (words <= 0) return cudaSuccess;
  const int threads = 256;
  dequant_q4_kernel<<<unsigned((words + threads - 1) / threads), threads, 0, s>>>(
      w, k, static_cast<__half*>(dst));
  return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  if (a.m <= 0 || a.n <= 0) return cudaSuccess;
  if (a.k <= 0 || (a.k % 8) || (a.ld_x % 8) || (reinterpret_cast<uintptr_t>(a.x) & 15) ||
      (reinterpret_cast<uintptr_t>(a.w16) & 15) || (a.n % kHeadDim))
    return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  if (!map_k_major(&ta, a.x, a.k, a.ld_x, a.m, GBM) ||
      !map_k_major(&tb, a.w16, a.k, a.k, a.n, GBN))
    return cudaErrorInvalidValue;
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
  const size_t smem = sizeof(GemmSmem) + 1024;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem));
  });
  if (attr_err != cudaSuccess) return attr_err;
  const dim3 grid(unsigned((a.n + GBN - 1) / GBN), unsigned((a.m + GBM - 1) / GBM));
  if (grid.y > 65535) return cudaErrorInvalidValue;
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
  return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(&gemm_kernel), args);
}

}  // namespace p2p
