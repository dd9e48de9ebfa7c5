// argmax.cu -- ARGMAX (src/scripts/lfm-engine/kernels.js:362-399) for sm_100a: the greedy token
// of a decode step and the device-side advance of the meta buffer, so consecutive decode steps
// need no host write of the position (engine.js:239-240, 265-266 dispatch it after the LM head).
//
// One CTA of 1024 threads.  Thread t scans 16-byte chunks t, t + 1024, ... of the f16 logits
// (element by element when the logits are not 16-byte aligned or V is not a multiple of 8),
// keeping the first strictly larger value seeded with -3e38 / index 0 as the shader does; warp
// shuffles and one shared-memory step then keep the larger value, ties to the smaller index.
// Every thread visits its indices in increasing order, so the result is the shader's for any
// input: the smallest index among the maxima of the values above -3e38 (NaN never wins), or 0.
#include "common.cuh"
#include "kernels.h"

namespace p2p {
namespace {

constexpr int kArgmaxThreads = 1024;

__device__ __forceinline__ void keep_better(float& bv, uint32_t& bi, float ov, uint32_t oi) {
  if (ov > bv || (ov == bv && oi < bi)) {
    bv = ov;
    bi = oi;
  }
}

__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_step_kernel(const __half* logits, uint32_t v, int vec, uint32_t* tok,
                       uint32_t* out_tok, int64_t out_cap, uint32_t* mt, int32_t* err) {
  __shared__ float wv[kArgmaxThreads / 32];
  __shared__ uint32_t wi[kArgmaxThreads / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float best = -3.0e38f;
  uint32_t bidx = 0u;
  if (vec) {
    const uint4* p = reinterpret_cast<const uint4*>(logits);
    for (uint32_t c = t; c < v / 8u; c += kArgmaxThreads) {
      const uint4 u = p[c];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[k]);
        const float a = __low2float(h), b = __high2float(h);
        if (a > best) {
          best = a;
          bidx = c * 8u + 2u * k;
        }
        if (b > best) {
          best = b;
          bidx = c * 8u + 2u * k + 1u;
        }
      }
    }
  } else {
    for (uint32_t i = t; i < v; i += kArgmaxThreads) {
      const float a = __half2float(logits[i]);
      if (a > best) {
        best = a;
        bidx = i;
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
    keep_better(best, bidx, __shfl_down_sync(0xffffffffu, best, off),
                __shfl_down_sync(0xffffffffu, bidx, off));
  if (lane == 0) {
    wv[warp] = best;
    wi[warp] = bidx;
  }
  __syncthreads();
  if (warp == 0) {
    best = wv[lane];
    bidx = wi[lane];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      keep_better(best, bidx, __shfl_down_sync(0xffffffffu, best, off),
                  __shfl_down_sync(0xffffffffu, bidx, off));
    if (lane == 0) {  // kernels.js:393-398
      const uint32_t step = mt[2];
      tok[0] = bidx;
      if (int64_t(step) < out_cap) out_tok[step] = bidx;
      else atomicOr(err, kErrOutTokFull);  // the caller's token buffer is full: not stored
      mt[2] = step + 1u;
      mt[0] = mt[0] + 1u;
    }
  }
}

}  // namespace

cudaError_t launch_argmax_step(const void* logits, int32_t vocab, uint32_t* tok,
                               uint32_t* out_tok, int64_t out_cap, uint32_t* meta, int32_t* err,
                               cudaStream_t s) {
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0 && vocab % 8 == 0;
  argmax_step_kernel<<<1, kArgmaxThreads, 0, s>>>(static_cast<const __half*>(logits),
                                                   uint32_t(vocab), vec ? 1 : 0, tok, out_tok,
                                                   out_cap, meta, err);
  return cudaGetLastError();
}

}  // namespace p2p
