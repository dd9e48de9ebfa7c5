// kv_quant.cu -- f16 KV-cache rows to the int8 cache format of p2p_attn_decode_kv.
//
// The int8 cache restates the quantised-cache append of the GroupQueryAttention kernels in the
// reference's kernel bundle (public/kernels/megakernel.json, com.microsoft.GroupQueryAttention
// gqa-present.wgsl.jinja, bits == 8): q = i32(clamp(round(x / scale), -128, 127)), with
// round() to nearest even and one f32 scale per tensor or per (kv head, dim) channel; the
// attention dequantises f32(q) * scale (attn-flash-decode-splitk.wgsl.jinja's load_key4 /
// load_value4).  HBM-bound elementwise pass: one thread per 8 values (16 bytes in, 8 out).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace p2p {
namespace {

__global__ void quantize_q8_kernel(const uint4* __restrict__ src, uint2* __restrict__ dst,
                                   int64_t n8, int chan, const float* __restrict__ scale,
                                   int per_channel) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8;
       i += int64_t(gridDim.x) * blockDim.x) {
    const uint4 w = src[i];
    const __half* h = reinterpret_cast<const __half*>(&w);
    const int c0 = int((i * 8) % chan);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sc = per_channel ? scale[c0 + k] : scale[0];
      const float q = fminf(fmaxf(rintf(__fdiv_rn(__half2float(h[k]), sc)), -128.f), 127.f);
      const uint32_t b = uint32_t(int32_t(q)) & 0xffu;
      if (k < 4) lo |= b << (8 * k);
      else hi |= b << (8 * (k - 4));
    }
    dst[i] = make_uint2(lo, hi);
  }
}

}  // namespace

cudaError_t launch_quantize_q8(const void* src, void* dst, int64_t rows, int hkv,
                               const float* scale, int scale_count, cudaStream_t s) {
  const int chan = hkv * kHeadDim;
  const int64_t n8 = rows * chan / 8;
  const int64_t want = (n8 + 255) / 256;
  const int blocks = int(want < 148 * 16 ? want : 148 * 16);
  quantize_q8_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint4*>(src),
                                            static_cast<uint2*>(dst), n8, chan, scale,
                                            scale_count > 1 ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace p2p
