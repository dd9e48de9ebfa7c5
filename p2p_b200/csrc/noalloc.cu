// noalloc.cu -- ragged batched decode that allocates no device memory.
//
// p2p_attn_decode_ragged splits long sequences over several CTAs and keeps their partial
// results in a workspace the context allocates (and grows) with cudaMalloc.  Some callers
// cannot allow that on their request path: serving processes that hand nearly all free HBM
// to their own pool (a pre-reserved KV-cache arena) at start-up, so a library cudaMalloc later
// fails or fragments their budget, and hosts whose memory is owned by another component that
// forbids allocations after initialisation.  This entry point runs the same kernel with its
// scratch in a fixed file-scope __device__ array instead; the caller still passes every
// input and output buffer.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

// Only the declared C ABI is exported (the library is built with -fvisibility=hidden).
#pragma GCC visibility push(default)
#include "../../include/p2p_attn.h"
#pragma GCC visibility pop
#include "host_internal.h"
#include "kernels.h"

namespace {

// The whole scratch: split partials followed by the per-(sequence, head) counters.
constexpr size_t kScratchBytes = size_t(P2P_NOALLOC_SCRATCH_BYTES);
constexpr size_t kCounterAlign = 256;

// Every GPU that loads this library holds this array (32 MiB) until the process exits.  In
// host code `g_decode_scratch` is only a host-side stand-in for the symbol, never a device
// address: the address is fetched per device with cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_decode_scratch on `dev`, looked up once per device with that device
// current.  The first lookup on a device loads the module that holds the array, which is when
// the array is placed in that GPU's memory; p2p_ctx_create makes that lookup.
cudaError_t scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != dev) {
      cudaError_t e = cudaSetDevice(dev);
      if (e != cudaSuccess) return e;
    }
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace

namespace p2p {
cudaError_t noalloc_prepare(int device) {
  void* p = nullptr;
  return scratch_address(device, &p);
}
}  // namespace p2p

extern "C" p2p_status p2p_attn_decode_ragged_noalloc(
    p2p_ctx* ctx, const p2p_attn_params* prm, const void* qkv, int64_t ld_qkv,
    const void* norm_w, const void* rope, void* k_cache, void* v_cache, int64_t kv_rows,
    const int32_t* offsets, const int32_t* past, int32_t nseq, int32_t max_past,
    int32_t fused_prep, void* out, int64_t ld_o, void* stream) {
  p2p_status st = p2p::check_ragged(ctx, prm, qkv, ld_qkv, rope, k_cache, v_cache, kv_rows,
                                    offsets, past, nseq, max_past, fused_prep, out, ld_o,
                                    "decode_ragged_noalloc");
  if (st != P2P_OK || nseq == 0) return st;

  const int hkv = prm->num_kv_heads;
  const int group = prm->num_heads / hkv;
  // the same split choice as p2p_attn_decode_ragged, P2P_DECODE_SPLITS included
  int min_split = 16;
  int splits = p2p::decode_max_splits(int64_t(max_past) + 1, hkv, nseq, p2p::ctx_num_sms(ctx),
                                      &min_split);
  if (p2p::forced_decode_splits() > 0) {
    splits = p2p::forced_decode_splits();
    min_split = 16;
  }
  const size_t pbytes = p2p::decode_partials_bytes(splits, hkv, nseq, group);
  const size_t coff = (pbytes + kCounterAlign - 1) / kCounterAlign * kCounterAlign;
  const size_t cbytes = p2p::decode_counters_bytes(hkv, nseq);
  if (coff + cbytes > kScratchBytes) {
    char msg[256];
    std::snprintf(msg, sizeof msg,
                  "decode_ragged_noalloc: %d sequences x %d kv heads x %d splits need %zu bytes "
                  "of scratch; the fixed scratch holds %zu (P2P_NOALLOC_SCRATCH_BYTES)",
                  nseq, hkv, splits, coff + cbytes, kScratchBytes);
    return p2p::ctx_fail(ctx, P2P_ERR_INVALID_ARG, msg);
  }
  void* base = nullptr;
  cudaError_t e = scratch_address(p2p::ctx_device(ctx), &base);
  if (e != cudaSuccess) return p2p::ctx_fail(ctx, P2P_ERR_CUDA, cudaGetErrorString(e));

  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != p2p::ctx_device(ctx)) cudaSetDevice(p2p::ctx_device(ctx));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* scratch = static_cast<unsigned char*>(base);
  // The counters must start at zero; the array keeps whatever the previous call left.
  e = cudaMemsetAsync(scratch + coff, 0, cbytes, s);
  if (e == cudaSuccess) {
    p2p::DecodeArgs a{};
    p2p::fill_ragged(a, qkv, ld_qkv, norm_w, rope, k_cache, v_cache, kv_rows, offsets, past,
                     max_past, out, ld_o);
    a.hq = prm->num_heads;
    a.hkv = hkv;
    a.scale_log2 = p2p::eff_scale_log2(prm);
    a.eps = p2p::eff_eps_of(prm);
    a.err = p2p::ctx_dev_err(ctx);
    a.wait_deficit = p2p::debug_wait_deficit();
    a.min_split = min_split;
    a.partials = reinterpret_cast<float*>(scratch);
    a.counters = reinterpret_cast<int32_t*>(scratch + coff);
    e = p2p::launch_decode(a, p2p::kRagged, fused_prep != 0, prm->dtype, splits, nseq, s);
  }
  if (prev >= 0 && prev != p2p::ctx_device(ctx)) cudaSetDevice(prev);
  if (e != cudaSuccess) return p2p::ctx_fail(ctx, P2P_ERR_CUDA, cudaGetErrorString(e));
  return P2P_OK;
}
