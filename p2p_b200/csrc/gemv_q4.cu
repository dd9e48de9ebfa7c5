// gemv_q4.cu -- the 4-bit MatMulNBits GEMV on either side of the attention path, for one token.
//
// The reference engine projects the normed hidden row to q, k and v with three GEMV dispatches
// (kernels.js:22-68, engine.js:202-204: q_proj, k_proj, v_proj into one qkv row), runs QK_PREP
// and ATTN, and projects the attention row back with o_proj (engine.js:224).  Weights are ONNX
// MatMulNBits (kernels.js:4-9): u32 words of eight 4-bit values per row, one f16 scale and one
// 4-bit zero point per 32-element block, w = (q - zp) * scale.
//
//   gemv_q4_kernel   y[y_off + n] = f16(x . W[n]): the o_proj consumer (any projection).
//   qkv_prep_kernel  the q/k/v projections of one token with QK_PREP in the epilogue: a cluster
//                    of 4 CTAs per head unit computes its 64 outputs (16 each, gathered in the
//                    first CTA's shared memory), rounds them to f16 (the qkv row the shader
//                    would store), then norms and rotates q / k (kernels.js:244-264) and
//                    writes rotated q to q_out and k / v to the cache row at the position -- the
//                    qkv row never goes through HBM and no separate QK_PREP launch runs.
//
// Both compute every output exactly as the GEMV shader does, so their outputs are bit-identical
// to it: 32 lanes per row, lane l walks words l, l+32, ..., a = sum over the word's 8 values of
// f32(x) * (q - zp) in order, acc += a * scale, then the shader's tree over the lanes
// (red[l] += red[l + s], s = 16..1), all f32 operations separately rounded.  HBM-bound: the
// weights stream once (3.1 MB of qkv weights and 2.1 MB of o_proj weights per LFM2.5-1.2B
// attention layer).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace p2p {
namespace {

constexpr int kThreads = 512;  // 16 warps
constexpr int kWarps = kThreads / 32;

// Arrive on the cluster barrier now (relaxed: the leader's barrier init is released by its own
// fence) and wait for every CTA's arrival later, just before the first remote store.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t smem_u32addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32addr(p)),
               "r"(rank));
  return r;
}
// One f32 into a cluster CTA's shared memory, counted (4 bytes) on that CTA's mbarrier.
__device__ __forceinline__ void st_async_f32(uint32_t dst, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(
                   dst),
               "f"(v), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void rows_bar_init(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32addr(bar)));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool rows_bar_try_wait(uint64_t* bar) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32addr(bar))
      : "memory");
  return ok != 0;
}
constexpr uint64_t kRowsWaitNs = 1000000000ull;
__device__ __forceinline__ uint64_t globaltimer_ns_() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}


// One output row as the shader's 32-lane subgroup computes it (kernels.js:44-66); the row's
// value ends in lane 0.  The words of a lane are fetched 8 at a time (all loads of a batch in
// flight together) and then accumulated in the shader's order.
__device__ __forceinline__ float row_dot(const Q4Matrix& w, int n, int k, const __half* xs,
                                         int lane) {
  const int nb = k >> 5, zr = (nb + 1) >> 1, wpr = k >> 3;
  const uint32_t* wrow = w.qweight + int64_t(n) * wpr;
  const __half* srow = w.scales + int64_t(n) * nb;
  const unsigned char* zrow =
      reinterpret_cast<const unsigned char*>(w.zero_points) + int64_t(n) * zr;
  float acc = 0.f;
  for (int base = lane; base < wpr; base += 32 * 8) {
    uint32_t word[8];
    __half sc[8];
    uint32_t zb[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int wi = base + 32 * j;
      if (wi < wpr) {
        word[j] = __ldg(wrow + wi);
        sc[j] = __ldg(srow + (wi >> 2));
        zb[j] = __ldg(zrow + (wi >> 3));  // kernels.js:16-19 (byte (blk >> 1) of the row)
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int wi = base + 32 * j;
      if (wi < wpr) {
        const int blk = wi >> 2;
        const float z = float((zb[j] >> ((blk & 1) * 4)) & 15u);
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + wi * 8);
        const __half* xh = reinterpret_cast<const __half*>(&xv);
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float q = float((word[j] >> (4 * i)) & 15u);
          a = __fadd_rn(a, __fmul_rn(__half2float(xh[i]), __fsub_rn(q, z)));
        }
        acc = __fadd_rn(acc, __fmul_rn(a, __half2float(sc[j])));
      }
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, s));
  return acc;
}

__device__ __forceinline__ void stage_x(const __half* x, int k, __half* xs) {
  for (int i = threadIdx.x * 8; i < k; i += kThreads * 8)
    *reinterpret_cast<uint4*>(xs + i) = *reinterpret_cast<const uint4*>(x + i);
}

__global__ void __launch_bounds__(kThreads) gemv_q4_kernel(const __grid_constant__ GemvArgs a) {
  __shared__ __align__(16) __half xs[kGemvMaxK];
  grid_dependency_wait();  // x may come from the previous kernel of the stream
  stage_x(static_cast<const __half*>(a.x), a.k, xs);
  __syncthreads();
  launch_dependents();  // the next kernel still waits for this one to complete
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (n >= a.w.n) return;
  const float v = row_dot(a.w, n, a.k, xs, lane);
  if (lane == 0) static_cast<__half*>(a.y)[a.y_off + n] = __float2half_rn(v);  // kernels.js:66
}

// One head unit per cluster of kUnitCtas CTAs: CTA r computes rows 16r..16r+15 of the head
// (one per warp) and pushes them into the first CTA's shared memory (st.async, counted on its
// mbarrier), whose epilogue warp alone waits for them; the other CTAs never wait on a peer.
constexpr int kUnitCtas = 4;

__global__ void __cluster_dims__(kUnitCtas, 1, 1) __launch_bounds__(kThreads)
    qkv_prep_kernel(const __grid_constant__ QkvPrepArgs a) {
  constexpr int D = kHeadDim;
  static_assert(D == kUnitCtas * kWarps, "one row per warp");
  __shared__ __align__(16) __half xs[kGemvMaxK];
  __shared__ float y_s[D];
  __shared__ uint64_t rows_bar;
  grid_dependency_wait();
  const int unit = blockIdx.x / kUnitCtas;
  const int part = blockIdx.x % kUnitCtas;  // rank in the cluster
  if (part == 0 && threadIdx.x == 0) rows_bar_init(&rows_bar, uint32_t(D * sizeof(float)));
  cluster_arrive_relaxed();
  // The position (meta) is needed only once the rows are computed: its load overlaps the
  // weight loads instead of preceding them.
  const int pos = a.meta ? int(a.meta[0]) : a.pos_host;
  stage_x(static_cast<const __half*>(a.x), a.k, xs);
  __syncthreads();
  launch_dependents();
  const int kind = unit < a.hq ? 0 : unit < a.hq + a.hkv ? 1 : 2;  // q, k or v head
  const int head = kind == 0 ? unit : kind == 1 ? unit - a.hq : unit - a.hq - a.hkv;
  const Q4Matrix& w = kind == 0 ? a.wq : kind == 1 ? a.wk : a.wv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // this CTA's 16 rows of the head; the value the GEMV shader would store is the f16 one,
  // written into the cluster leader's y_s
  const int row = part * kWarps + warp;
  const float v = row_dot(w, head * D + row, a.k, xs, lane);
  cluster_wait();  // every CTA has arrived: the leader's rows_bar is initialised
  if (pos < 0 || int64_t(pos) >= a.kv_cap) {  // the same for every CTA: nothing is written
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, kErrPosBeyondCache);
    return;
  }
  if (lane == 0)
    st_async_f32(cluster_addr(&y_s[row], 0), __half2float(__float2half_rn(v)),
                 cluster_addr(&rows_bar, 0));
  if (part != 0 || warp != 0) return;
  // the leader's epilogue warp fetches the position's rope row and the norm weights while the
  // cluster gathers the rows
  const bool epi = kind != 2;  // (only the leader's warp 0 reaches here)
  const __half* nw = static_cast<const __half*>(a.norm_w);
  float cs = 0.f, sn = 0.f, w0 = 0.f, w1 = 0.f;
  if (epi) {
    const __half* rope = static_cast<const __half*>(a.rope) + int64_t(pos) * D;
    cs = __half2float(rope[lane]);
    sn = __half2float(rope[32 + lane]);
    if (nw) {
      w0 = __half2float(nw[(kind == 1 ? D : 0) + lane]);
      w1 = __half2float(nw[(kind == 1 ? D : 0) + lane + 32]);
    }
  }
  // the 64 rows of the unit: every lane waits (its own acquire orders its reads of y_s), bounded;
  // a peer that never delivers is reported and nothing is written
  bool got = rows_bar_try_wait(&rows_bar);
  if (!got) {
    const uint64_t t0 = globaltimer_ns_();
    while (!(got = rows_bar_try_wait(&rows_bar)) && globaltimer_ns_() - t0 < kRowsWaitNs) {
    }
  }
  if (!__all_sync(0xffffffffu, got)) {
    if (lane == 0) atomicOr(a.err, kErrTimeout);
    return;
  }
  const int64_t crow = (int64_t(pos) * a.hkv + head) * D;  // cache row `pos`, kv head `head`
  if (kind == 2) {  // QK_PREP v unit (kernels.js:237-241): raw copy
    __half* vc = static_cast<__half*>(a.v_cache) + crow;
    vc[lane] = __float2half_rn(y_s[lane]);
    vc[lane + 32] = __float2half_rn(y_s[lane + 32]);
    return;
  }
  float r0, r1;  // QK_PREP q / k unit (kernels.js:244-264)
  norm_rope_vals<__half>(y_s[lane], y_s[lane + 32], w0, w1, nw != nullptr, a.eps, cs, sn, r0,
                         r1);
  __half* dst = kind == 0 ? static_cast<__half*>(a.q_out) + int64_t(head) * D
                          : static_cast<__half*>(a.k_cache) + crow;
  dst[lane] = __float2half_rn(r0);
  dst[lane + 32] = __float2half_rn(r1);
}

cudaError_t launch_pdl(const void* fn, dim3 grid, void** args, cudaStream_t s) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute at{};
  at.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_gemv_q4(const GemvArgs& a, cudaStream_t s) {
  void* args[] = {const_cast<GemvArgs*>(&a)};
  return launch_pdl(reinterpret_cast<const void*>(&gemv_q4_kernel),
                    dim3(unsigned((a.w.n + kWarps - 1) / kWarps)), args, s);
}

cudaError_t launch_qkv_prep(const QkvPrepArgs& a, cudaStream_t s) {
  void* args[] = {const_cast<QkvPrepArgs*>(&a)};
  return launch_pdl(reinterpret_cast<const void*>(&qkv_prep_kernel),
                    dim3(unsigned((a.hq + 2 * a.hkv) * kUnitCtas)), args, s);
}

}  // namespace p2p
