// common.cuh -- shared device helpers for the sm_100a attention kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace p2p {

constexpr int kHeadDim = 64;
constexpr float kLog2e = 1.4426950408889634f;

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Programmatic dependent launch.  A kernel launched with the programmatic-stream-serialization
// attribute may start while the previous kernel of its stream still runs; grid_dependency_wait
// returns once that kernel has completed and its memory operations are visible (immediately
// when there is no such kernel), so it goes before the first global load or store.
// launch_dependents lets the next kernel of the stream start early in the same way.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- storage types ------------------------------------------------------------------------
// Every kernel reads/writes rows of 64 elements; a "chunk" is 8 consecutive elements
// (16 bytes of f16 or 32 bytes of f32).

struct F16 {
  using T = __half;
  static constexpr int kBytes = 2;
};
struct F32 {
  using T = float;
  static constexpr int kBytes = 4;
};

__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(float x) { return x; }
template <class T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
// The f16() rounding point of the shaders: identity for f32 storage.
template <class T>
__device__ __forceinline__ float round_st(float x) { return to_f32(from_f32<T>(x)); }

// Streaming 16-byte load through the non-coherent path without allocating in L1; the data is
// read exactly once per kernel.  Only for buffers the kernel does not write.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 8 elements of a row starting at `p` (16-byte aligned) widened to f32.
__device__ __forceinline__ void load8_stream(const __half* p, float (&v)[8]) {
  const uint4 r = ld_stream16(p);
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8_stream(const float* p, float (&v)[8]) {
  const uint4 a = ld_stream16(p);
  const uint4 b = ld_stream16(p + 4);
  v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y);
  v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
  v[4] = __uint_as_float(b.x); v[5] = __uint_as_float(b.y);
  v[6] = __uint_as_float(b.z); v[7] = __uint_as_float(b.w);
}

// Raw 8-element chunk kept in registers between the load and its use (software pipelining).
template <class T>
struct Chunk8;
template <>
struct Chunk8<__half> {
  uint4 r;
  __device__ __forceinline__ void load(const __half* p) { r = ld_stream16(p); }
  __device__ __forceinline__ void zero() { r = make_uint4(0, 0, 0, 0); }
  __device__ __forceinline__ void widen(float (&v)[8]) const {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};
template <>
struct Chunk8<float> {
  uint4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = ld_stream16(p);
    b = ld_stream16(p + 4);
  }
  __device__ __forceinline__ void zero() { a = b = make_uint4(0, 0, 0, 0); }
  __device__ __forceinline__ void widen(float (&v)[8]) const {
    v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y);
    v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
    v[4] = __uint_as_float(b.x); v[5] = __uint_as_float(b.y);
    v[6] = __uint_as_float(b.z); v[7] = __uint_as_float(b.w);
  }
};

// Coherent 8-element store (f16: one 16-byte store; f32: two).
__device__ __forceinline__ void store8(__half* p, const float (&v)[8]) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = r;
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- q/k RMSNorm + RoPE of one 64-wide head held by one warp ------------------------------
// Lane l holds elements l and l+32 (the rotate-half partners, kernels.js:257-262).  The
// sum of squares is folded with xor-butterflies 16, 8, 4, 2, 1 after pairing (l, l+32): every
// partial sum equals the shader's shared-memory tree (kernels.js:246-251) bit for bit, since
// each IEEE addition is commutative.  Separate __fmul_rn/__fadd_rn keep the shader's
// rounding (no FMA contraction).  norm_rope_vals takes the lane's norm weights already loaded
// (w0 = nw[lane], w1 = nw[lane + 32]); norm_rope_head loads them from nw.
template <class T>
__device__ __forceinline__ void norm_rope_vals(float v0, float v1, float w0, float w1,
                                               bool has_norm, float eps, float cs, float sn,
                                               float& r0, float& r1) {
  float n0 = v0, n1 = v1;
  if (has_norm) {
    float ss = __fadd_rn(__fmul_rn(v0, v0), __fmul_rn(v1, v1));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    const float inv = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, 64.0f), eps));
    n0 = round_st<T>(__fmul_rn(__fmul_rn(v0, inv), w0));
    n1 = round_st<T>(__fmul_rn(__fmul_rn(v1, inv), w1));
  }
  r0 = __fsub_rn(__fmul_rn(n0, cs), __fmul_rn(n1, sn));
  r1 = __fadd_rn(__fmul_rn(n1, cs), __fmul_rn(n0, sn));
}
template <class T>
__device__ __forceinline__ void norm_rope_head(float v0, float v1, const T* nw, bool has_norm,
                                               float eps, float cs, float sn, float& r0,
                                               float& r1) {
  const int l = threadIdx.x & 31;
  const float w0 = has_norm ? to_f32(nw[l]) : 0.f;
  const float w1 = has_norm ? to_f32(nw[l + 32]) : 0.f;
  norm_rope_vals<T>(v0, v1, w0, w1, has_norm, eps, cs, sn, r0, r1);
}

}  // namespace p2p

namespace p2p {

// ---- cp.async (16-byte, L2-only) ring helpers ---------------------------------------------
// When `valid` is false the 16 destination bytes are zero-filled and no source byte is read.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, bool valid) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem_src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 8 consecutive elements from shared memory, widened to f32.
__device__ __forceinline__ void load8_shared(const __half* p, float (&v)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8_shared(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

}  // namespace p2p
