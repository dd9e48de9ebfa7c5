// probe.cu -- a measurement reference for the HBM-bound kernels: one launch that streams a
// buffer once (16-byte loads, eight in flight per thread, two 512-thread CTAs per SM) and
// folds it into a 32-bit XOR checksum.  Timed on the same bytes and in the same way as a
// decode step (one launch per graph node), it gives the speed of light of "read these bytes
// in one launch" on this GPU, against which the decode kernels' fixed costs are measured.
// Not part of the reference contract.
#include <cuda_runtime.h>

#include <cstdint>

// Only the declared C ABI is exported (the library is built with -fvisibility=hidden).
#pragma GCC visibility push(default)
#include "../../include/p2p_attn.h"
#pragma GCC visibility pop
#include "host_internal.h"

namespace p2p {
namespace {

constexpr int kProbeThreads = 512;
constexpr int kProbeUnroll = 8;

__global__ void __launch_bounds__(kProbeThreads)
    stream_xor_kernel(const uint4* __restrict__ src, int64_t n_vec, uint32_t* out) {
  uint32_t acc = 0;
  const int64_t stride = int64_t(gridDim.x) * kProbeThreads;
  for (int64_t base = int64_t(blockIdx.x) * kProbeThreads * kProbeUnroll + threadIdx.x;
       base < n_vec; base += stride * kProbeUnroll) {
    uint4 v[kProbeUnroll];
#pragma unroll
    for (int u = 0; u < kProbeUnroll; ++u) {
      const int64_t i = base + int64_t(u) * kProbeThreads;
      v[u] = i < n_vec ? __ldcs(src + i) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kProbeUnroll; ++u) acc ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc ^= __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0 && acc != 0) atomicXor(out, acc);
}

}  // namespace
}  // namespace p2p

extern "C" p2p_status p2p_debug_stream_read(p2p_ctx* ctx, const void* src, int64_t bytes,
                                            uint32_t* xor_out, void* stream) {
  if (!ctx || !src || !xor_out || bytes < 0 || (bytes & 15) ||
      (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(xor_out) & 3))
    return ctx ? p2p::ctx_fail(ctx, P2P_ERR_INVALID_ARG,
                               "debug_stream_read: src 16-byte aligned, bytes a multiple of 16")
               : P2P_ERR_INVALID_ARG;
  if (bytes == 0) return P2P_OK;
  const int dev = p2p::ctx_device(ctx);
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != dev) cudaSetDevice(dev);
  const int64_t n_vec = bytes / 16;
  const int64_t per_cta = int64_t(p2p::kProbeThreads) * p2p::kProbeUnroll;
  int64_t grid = (n_vec + per_cta - 1) / per_cta;
  const int64_t cap = 2 * int64_t(p2p::ctx_num_sms(ctx));
  if (grid > cap) grid = cap;
  p2p::stream_xor_kernel<<<unsigned(grid), p2p::kProbeThreads, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), n_vec, xor_out);
  const cudaError_t e = cudaGetLastError();
  if (cur != dev && cur >= 0) cudaSetDevice(cur);
  if (e != cudaSuccess)
    return p2p::ctx_fail(ctx, P2P_ERR_CUDA, cudaGetErrorString(e));
  return P2P_OK;
}
