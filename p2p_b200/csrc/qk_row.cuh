// qk_row.cuh -- QK_PREP's q/k unit for one 64-element row held by ONE thread
// (src/scripts/lfm-engine/kernels.js:242-263), shared by the QK_PREP rows kernel and the
// prompt-chunk projection's fused epilogue.  The sum of squares follows the shader's tree
// (t[i] = v[i]^2 + v[i+32]^2, then pairs 16, 8, 4, 2, 1 apart: the same IEEE additions, so the
// result is bit-identical), then inverseSqrt, the f16-rounded norm with the weights and the
// rotate-half RoPE per element pair (i, i + 32).
#pragma once

#include "common.cuh"

namespace p2p {

// 64 elements of one row in registers; element e as f32.
template <class T>
struct Row64;
template <>
struct Row64<__half> {
  uint32_t w[32];  // w[k] = elements 2k, 2k+1
  __device__ __forceinline__ void load(const __half* p) {
    const uint4* s = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 v = s[i];
      w[4 * i] = v.x;
      w[4 * i + 1] = v.y;
      w[4 * i + 2] = v.z;
      w[4 * i + 3] = v.w;
    }
  }
  __device__ __forceinline__ float get(int e) const {
    const __half2 h = *reinterpret_cast<const __half2*>(&w[e >> 1]);
    return (e & 1) ? __high2float(h) : __low2float(h);
  }
};
template <>
struct Row64<float> {
  float f[64];
  __device__ __forceinline__ void load(const float* p) {
    const float4* s = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 v = s[i];
      f[4 * i] = v.x;
      f[4 * i + 1] = v.y;
      f[4 * i + 2] = v.z;
      f[4 * i + 3] = v.w;
    }
  }
  __device__ __forceinline__ float get(int e) const { return f[e]; }
};

// The rotated row of x: `put(k, v)` receives elements 8k .. 8k+7 (k = 0..7) as f32 values that
// the shader stores as T.  w: the 64 norm weights as f32, or nullptr (no norm); rope: the
// position's row [cos(32) | sin(32)].
template <class T, class Put>
__device__ __forceinline__ void rotate_row(const Row64<T>& x, const float* w, float eps,
                                           const T* rope, Put put) {
  float inv = 1.0f;
  if (w != nullptr) {
    float t[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      t[i] = __fadd_rn(__fmul_rn(x.get(i), x.get(i)), __fmul_rn(x.get(i + 32), x.get(i + 32)));
#pragma unroll
    for (int s = 16; s > 0; s >>= 1)
#pragma unroll
      for (int i = 0; i < s; ++i) t[i] = __fadd_rn(t[i], t[i + s]);
    inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(t[0], 64.0f), eps));
  }
#pragma unroll
  for (int c = 0; c < 32; c += 8) {  // element pairs (i, i + 32), i = c .. c + 7
    float cs[8], sn[8], lo[8], hi[8];
    // rope row: cos at [0, 32), sin at [32, 64)
    if constexpr (sizeof(T) == 2) {
      const uint4 vc = *reinterpret_cast<const uint4*>(rope + c);
      const uint4 vs = *reinterpret_cast<const uint4*>(rope + 32 + c);
      const uint32_t uc[4] = {vc.x, vc.y, vc.z, vc.w}, us[4] = {vs.x, vs.y, vs.z, vs.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 hc = *reinterpret_cast<const __half2*>(&uc[q]);
        const __half2 hs = *reinterpret_cast<const __half2*>(&us[q]);
        cs[2 * q] = __low2float(hc);
        cs[2 * q + 1] = __high2float(hc);
        sn[2 * q] = __low2float(hs);
        sn[2 * q + 1] = __high2float(hs);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; k += 4) {
        const float4 vc = *reinterpret_cast<const float4*>(rope + c + k);
        const float4 vs = *reinterpret_cast<const float4*>(rope + 32 + c + k);
        cs[k] = to_f32(vc.x); cs[k + 1] = to_f32(vc.y); cs[k + 2] = to_f32(vc.z); cs[k + 3] = to_f32(vc.w);
        sn[k] = to_f32(vs.x); sn[k + 1] = to_f32(vs.y); sn[k + 2] = to_f32(vs.z); sn[k + 3] = to_f32(vs.w);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      const int i = c + k;
      float n0[2] = {x.get(i), x.get(i + 1)}, n1[2] = {x.get(i + 32), x.get(i + 33)};
      if (w != nullptr) {
        float u0[2], u1[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          u0[e] = __fmul_rn(__fmul_rn(n0[e], inv), w[i + e]);
          u1[e] = __fmul_rn(__fmul_rn(n1[e], inv), w[i + 32 + e]);
        }
        if constexpr (sizeof(T) == 2) {  // the shader's f16() rounding, two values at once
          const float2 r0 = __half22float2(__floats2half2_rn(u0[0], u0[1]));
          const float2 r1 = __half22float2(__floats2half2_rn(u1[0], u1[1]));
          n0[0] = r0.x; n0[1] = r0.y; n1[0] = r1.x; n1[1] = r1.y;
        } else {
          n0[0] = u0[0]; n0[1] = u0[1]; n1[0] = u1[0]; n1[1] = u1[1];
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        lo[k + e] = __fsub_rn(__fmul_rn(n0[e], cs[k + e]), __fmul_rn(n1[e], sn[k + e]));
        hi[k + e] = __fadd_rn(__fmul_rn(n1[e], cs[k + e]), __fmul_rn(n0[e], sn[k + e]));
      }
    }
    put(c / 8, lo);
    put(4 + c / 8, hi);
  }
}

}  // namespace p2p
