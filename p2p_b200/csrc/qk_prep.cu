// qk_prep.cu -- QK_PREP (src/scripts/lfm-engine/kernels.js:216-266) for sm_100a.
//
// One warp per (head unit, token): units [0,Hq) are q heads, [Hq,Hq+Hkv) k heads,
// [Hq+Hkv,Hq+2Hkv) v heads, exactly the shader's unit numbering generalised from 16/8.
// Lane l owns elements l and l+32 (the rotate-half partners), so RoPE needs no exchange and
// the RMS sum is a 5-level butterfly that reproduces the shader's tree sum bit for bit.
#include "common.cuh"
#include "kernels.h"

namespace p2p {
namespace {

constexpr int kWarpsPerBlock = 8;

template <class T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    qk_prep_kernel(const QkPrepArgs a) {
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int m = blockIdx.y;
  const int units = a.hq + 2 * a.hkv;
  if (unit >= units) return;
  const int64_t pos = int64_t(a.meta ? a.meta[0] : uint32_t(a.pos0)) + m;
  if (pos >= a.kv_cap) {  // the cache cannot hold this row: touch nothing, report it
    if ((threadIdx.x & 31) == 0) atomicOr(a.err, kErrPosBeyondCache);
    return;
  }
  const T* row = static_cast<const T*>(a.qkv) + int64_t(m) * a.ld_qkv;
  const int64_t kv_stride = int64_t(a.hkv) * kHeadDim;
  if (unit >= a.hq + a.hkv) {  // kernels.js:237-241: v heads are copied unchanged
    const int kh = unit - a.hq - a.hkv;
    const T* src = row + int64_t(a.hq + a.hkv) * kHeadDim + kh * kHeadDim;
    T* dst = static_cast<T*>(a.v_cache) + pos * kv_stride + kh * kHeadDim;
    dst[lane] = src[lane];
    dst[lane + 32] = src[lane + 32];
    return;
  }
  const bool isq = unit < a.hq;
  const int64_t off = int64_t(unit) * kHeadDim;  // q heads then k heads are contiguous
  const float v0 = to_f32(row[off + lane]);
  const float v1 = to_f32(row[off + lane + 32]);
  const T* nw = a.norm_w ? static_cast<const T*>(a.norm_w) + (isq ? 0 : kHeadDim) : nullptr;
  const T* rope = static_cast<const T*>(a.rope) + pos * kHeadDim;
  const float cs = to_f32(rope[lane]);
  const float sn = to_f32(rope[32 + lane]);
  float r0, r1;
  norm_rope_head<T>(v0, v1, nw, nw != nullptr, a.eps, cs, sn, r0, r1);
  T* dst = isq ? static_cast<T*>(a.q_out) + int64_t(m) * a.ld_q + off
               : static_cast<T*>(a.k_cache) + pos * kv_stride + (unit - a.hq) * kHeadDim;
  dst[lane] = from_f32<T>(r0);
  dst[lane + 32] = from_f32<T>(r1);
}

}  // namespace

cudaError_t launch_qk_prep(const QkPrepArgs& a, int dtype, cudaStream_t s) {
  if (a.m_tokens <= 0) return cudaSuccess;
  const int units = a.hq + 2 * a.hkv;
  dim3 grid(ceil_div(units, kWarpsPerBlock), a.m_tokens);
  if (dtype == 0) qk_prep_kernel<__half><<<grid, kWarpsPerBlock * 32, 0, s>>>(a);
  else qk_prep_kernel<float><<<grid, kWarpsPerBlock * 32, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace p2p
