// api.cu -- the extern "C" boundary of libp2pattn.so (declared in include/p2p_attn.h).
//
// Host-side responsibilities the reference engine keeps in JavaScript:
//   - argument validation and error reporting (engine.js:83, :379-380 throw; here statuses)
//   - the RoPE table (engine.js:60-71) and the meta buffer (engine.js:144, :388, :408, :422)
//   - per-layer K/V cache buffers and their growth (engine.js:152-165, :274-304)
//   - choosing the launch for each shader dispatch (engine.js:245-259)
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <tuple>
#include <vector>

// The library is built with -fvisibility=hidden; only the declared C ABI is exported.
#pragma GCC visibility push(default)
#include "../../include/p2p_attn.h"
#pragma GCC visibility pop
#include "host_internal.h"
#include "kernels.h"

struct p2p_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  uint32_t* meta = nullptr;
  int32_t* dev_err = nullptr;  // kernels set bits here (kErrPosBeyondCache); read by p2p_sync
  int32_t* host_err = nullptr;      // mapped page-locked word p2p_sync reads dev_err into
  int32_t* host_err_dev = nullptr;  // the same word's device address
  float* partials = nullptr;
  size_t partials_bytes = 0;
  int32_t* counters = nullptr;
  size_t counters_bytes = 0;
  void* w16 = nullptr;  // prompt-chunk projections: the dequantised f16 weights
  size_t w16_bytes = 0;
  std::map<std::tuple<int, int, double, int>, void*> rope;
  std::map<void*, size_t> shared;  // p2p_shared_alloc buffers and their sizes
  std::string err;
};

struct p2p_kv {
  p2p_ctx* ctx = nullptr;
  int n_layers = 0, hkv = 0, d = 0, dtype = 0;
  int64_t cap = 0;
  std::vector<void*> k, v;
};

namespace {

// Test hook: a device-allocation budget for this process (bytes; <0 = unlimited), used to
// exercise the OOM path without exhausting the GPU.
int64_t g_alloc_limit = -1;
int64_t g_alloc_used = 0;
std::mutex g_alloc_mu;

// Test hook: extra bytes every bounded device-side wait expects (0 = normal operation).
std::atomic<int32_t> g_wait_deficit{0};

struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

p2p_status fail(p2p_ctx* ctx, p2p_status s, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return s;
}

p2p_status cuda_fail(p2p_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, P2P_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

cudaError_t dev_alloc(void** p, size_t bytes) {
  {
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    if (g_alloc_limit >= 0 && g_alloc_used + int64_t(bytes) > g_alloc_limit) {
      *p = nullptr;
      return cudaErrorMemoryAllocation;
    }
  }
  cudaError_t e = cudaMalloc(p, bytes);
  if (e == cudaSuccess) {
    std::lock_guard<std::mutex> lk(g_alloc_mu);
    g_alloc_used += int64_t(bytes);
  }
  return e;
}

void dev_free(void* p, size_t bytes) {
  if (!p) return;
  cudaFree(p);
  std::lock_guard<std::mutex> lk(g_alloc_mu);
  g_alloc_used -= int64_t(bytes);
}

// NULL is the CUDA default stream (as for every CUDA library), not the context's stream:
// a caller that wants the context's own stream passes p2p_ctx_stream(ctx).
cudaStream_t pick_stream(p2p_ctx*, void* stream) { return static_cast<cudaStream_t>(stream); }

size_t elem_bytes(int dtype) { return dtype == P2P_F32 ? 4 : 2; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Shared validation of the uniform parameters.
p2p_status check_params(p2p_ctx* ctx, const p2p_attn_params* prm, bool allow_f32) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  if (!prm) return fail(ctx, P2P_ERR_INVALID_ARG, "params is NULL");
  if (prm->head_dim != 64)
    return fail(ctx, P2P_ERR_UNSUPPORTED, "head_dim %d: only 64 is implemented", prm->head_dim);
  if (prm->num_heads <= 0 || prm->num_kv_heads <= 0 || prm->num_heads % prm->num_kv_heads)
    return fail(ctx, P2P_ERR_INVALID_ARG, "num_heads %d / num_kv_heads %d", prm->num_heads,
                prm->num_kv_heads);
  const int g = prm->num_heads / prm->num_kv_heads;
  if (g != 1 && g != 2 && g != 4 && g != 8)
    return fail(ctx, P2P_ERR_UNSUPPORTED, "group size %d not in {1,2,4,8}", g);
  if (prm->dtype != P2P_F16 && !(allow_f32 && prm->dtype == P2P_F32))
    return fail(ctx, P2P_ERR_UNSUPPORTED, "dtype %d not supported by this entry point",
                prm->dtype);
  if (!(prm->scale >= 0.f) || !std::isfinite(prm->scale))
    return fail(ctx, P2P_ERR_INVALID_ARG, "scale must be finite and >= 0");
  return P2P_OK;
}

float eff_scale(const p2p_attn_params* prm) {
  return prm->scale > 0.f ? prm->scale : 1.0f / std::sqrt(float(prm->head_dim));
}
float eff_eps(const p2p_attn_params* prm) { return prm->eps > 0.f ? prm->eps : 1e-5f; }

// Grows one library-owned device buffer to at least `need` bytes; rare, so the device is
// synchronised first (no launch may still use the old buffer).
p2p_status ensure_buffer(p2p_ctx* ctx, void** ptr, size_t* have, size_t need, const char* what) {
  if (need <= *have) return P2P_OK;
  cudaDeviceSynchronize();
  dev_free(*ptr, *have);
  *ptr = nullptr;
  *have = 0;
  void* p = nullptr;
  if (dev_alloc(&p, need) != cudaSuccess)
    return fail(ctx, P2P_ERR_OOM, "%s of %zu bytes", what, need);
  *ptr = p;
  *have = need;
  return P2P_OK;
}

p2p_status ensure_workspace(p2p_ctx* ctx, size_t pbytes, size_t cbytes, cudaStream_t s) {
  if (pbytes > ctx->partials_bytes) {
    cudaDeviceSynchronize();  // rare growth: no launch may still use the old workspace
    dev_free(ctx->partials, ctx->partials_bytes);
    ctx->partials = nullptr;
    ctx->partials_bytes = 0;
    void* p = nullptr;
    if (dev_alloc(&p, pbytes) != cudaSuccess)
      return fail(ctx, P2P_ERR_OOM, "split-KV workspace of %zu bytes", pbytes);
    ctx->partials = static_cast<float*>(p);
    ctx->partials_bytes = pbytes;
  }
  if (cbytes > ctx->counters_bytes) {
    cudaDeviceSynchronize();
    dev_free(ctx->counters, ctx->counters_bytes);
    ctx->counters = nullptr;
    ctx->counters_bytes = 0;
    void* p = nullptr;
    if (dev_alloc(&p, cbytes) != cudaSuccess)
      return fail(ctx, P2P_ERR_OOM, "split-KV counters of %zu bytes", cbytes);
    cudaError_t e = cudaMemsetAsync(p, 0, cbytes, s);
    if (e != cudaSuccess) {
      dev_free(p, cbytes);
      return cuda_fail(ctx, e, "cudaMemsetAsync(counters)");
    }
    ctx->counters = static_cast<int32_t*>(p);
    ctx->counters_bytes = cbytes;
  }
  return P2P_OK;
}

// engine.js:28-50 semantics for the host-built table: double -> f32 (RNE) -> f16 (RNE).
uint16_t half_bits(float f) {
  const __half h = __float2half_rn(f);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

// Tuning knob: P2P_DECODE_SPLITS=<n> forces n key splits per (sequence, kv head).
int forced_splits() {
  static const int v = [] {
    const char* e = std::getenv("P2P_DECODE_SPLITS");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

// Tuning knob: P2P_PDL=<0|1|2> sets when a decode launch lets the next kernel of its stream
// start early (DecodeArgs::pdl); 0 turns programmatic dependent launch off.
int pdl_mode() {
  static const int v = [] {
    const char* e = std::getenv("P2P_PDL");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

// Tuning knob: P2P_DECODE_CLUSTER=0 makes decode steps use the workspace combine instead of
// the thread-block-cluster combine.
bool cluster_combine_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("P2P_DECODE_CLUSTER");
    return !(e && std::atoi(e) == 0);
  }();
  return v;
}

p2p_status run_decode(p2p_ctx* ctx, const p2p_attn_params* prm, p2p::DecodeArgs& a, int mode,
                      bool fused, int nz, int64_t max_len, cudaStream_t s) {
  const int hkv = prm->num_kv_heads;
  const int group = prm->num_heads / hkv;
  a.hq = prm->num_heads;
  a.hkv = hkv;
  a.scale_log2 = eff_scale(prm) * 1.4426950408889634f;
  a.eps = eff_eps(prm);
  a.err = ctx->dev_err;
  a.wait_deficit = g_wait_deficit.load();
  a.pdl = pdl_mode();
  int min_split = 16;
  int cluster = 0;
  int splits = 0;
  if (mode == p2p::kLayers && prm->dtype == P2P_F16 && cluster_combine_enabled()) {
    // Decode step over layers: the splits of one (layer, head chunk) form a cluster.
    cluster = forced_splits() > 0
                  ? std::min(forced_splits(), 16)
                  : p2p::decode_cluster_splits(max_len, hkv, group, nz, fused, ctx->num_sms);
    if (cluster > 1) splits = cluster;
    else cluster = 0;
  }
  if (cluster == 0) {
    splits = p2p::decode_max_splits(max_len, hkv, nz, ctx->num_sms, &min_split);
    if (forced_splits() > 0) {
      splits = forced_splits();
      min_split = 16;
    }
    if (mode == p2p::kPaged) {
      // a split's block-table entries must fit the kernel's shared copy
      const int64_t keys = (int64_t(p2p::kPagedTableCap - 3) << a.block_shift) - 16;
      const int64_t need = (max_len + keys - 1) / keys;
      if (splits < need) splits = int(need);
    }
    p2p_status st = ensure_workspace(ctx, p2p::decode_partials_bytes(splits, hkv, nz, group),
                                     p2p::decode_counters_bytes(hkv, nz), s);
    if (st != P2P_OK) return st;
    a.partials = ctx->partials;
    a.counters = ctx->counters;
  }
  a.min_split = min_split;
  cudaError_t e = p2p::launch_decode(a, mode, fused, prm->dtype, splits, nz, s, cluster);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "decode launch");
  return P2P_OK;
}

// The tcgen05 flash kernel on a causal prompt chunk: rows pos0 .. pos0+M-1 of q against
// cache keys 0 .. pos0+M-1; outs[0] is this GPU's output, outs[1..] other buffers of the same
// layout (other GPUs') that receive the same rows; head h lands at column (out_head0 + h)*D.
p2p_status run_causal_flash(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q,
                            int64_t ld_q, const void* k_cache, const void* v_cache,
                            int64_t kv_cap_tokens, void* const* outs, int n_outs, int64_t ld_o,
                            int out_head0, const uint32_t* meta_dev, int32_t pos0,
                            int32_t m_tokens, cudaStream_t s, void* mc_out = nullptr) {
  p2p::FlashArgs f{};
  f.mc_out = mc_out;
  f.q = q;
  f.k = k_cache;
  f.v = v_cache;
  f.out = outs[0];
  for (int t = 1; t < n_outs; ++t) f.extra_out[t - 1] = outs[t];
  f.n_extra_out = n_outs - 1;
  f.out_head0 = out_head0;
  f.ld_q = ld_q;
  f.ld_kv = int64_t(prm->num_kv_heads) * prm->head_dim;
  f.ld_o = ld_o;
  f.q_rows_total = m_tokens;
  f.kv_rows_total = kv_cap_tokens;
  f.batch_stride_q_rows = 0;
  f.batch_stride_kv_rows = 0;
  f.batch = 1;
  f.s_q = m_tokens;
  f.s_kv = 0;
  f.hq = prm->num_heads;
  f.hkv = prm->num_kv_heads;
  f.causal = 1;
  f.meta = meta_dev;
  f.pos0_host = pos0;
  f.scale_log2 = eff_scale(prm) * 1.4426950408889634f;
  f.err = ctx->dev_err;
  f.wait_deficit = g_wait_deficit.load();
  f.num_sms = ctx->num_sms;
  cudaError_t e = p2p::launch_flash(f, s);
  if (e == cudaErrorNotSupported) return fail(ctx, P2P_ERR_UNSUPPORTED, "prefill kernel");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "prefill launch");
  return P2P_OK;
}

}  // namespace

extern "C" {

int p2p_abi_version(void) { return P2P_ATTN_ABI_VERSION; }

const char* p2p_status_string(p2p_status s) {
  switch (s) {
    case P2P_OK: return "ok";
    case P2P_ERR_INVALID_ARG: return "invalid argument";
    case P2P_ERR_OOM: return "out of device memory";
    case P2P_ERR_KV_FULL: return "kv cache full";
    case P2P_ERR_CUDA: return "cuda error";
    case P2P_ERR_TIMEOUT: return "device wait timed out";
    case P2P_ERR_NCCL: return "nccl error";
    case P2P_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

p2p_status p2p_ctx_create(int device, p2p_ctx** out) {
  if (!out) return P2P_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    cudaGetLastError();
    return P2P_ERR_CUDA;
  }
  p2p_ctx* ctx = new (std::nothrow) p2p_ctx;
  if (!ctx) return P2P_ERR_OOM;
  ctx->device = device;
  DeviceGuard g(device);
  if (!g.ok) {
    delete ctx;
    return P2P_ERR_CUDA;
  }
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete ctx;
    return P2P_ERR_CUDA;
  }
  void* m = nullptr;
  if (dev_alloc(&m, 16) != cudaSuccess) {
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return P2P_ERR_OOM;
  }
  cudaMemset(m, 0, 16);
  ctx->meta = static_cast<uint32_t*>(m);
  void* e = nullptr;
  if (dev_alloc(&e, sizeof(int32_t)) != cudaSuccess) {
    dev_free(m, 16);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return P2P_ERR_OOM;
  }
  cudaMemset(e, 0, sizeof(int32_t));
  ctx->dev_err = static_cast<int32_t*>(e);
  // p2p_sync has a one-thread kernel move the error word into this mapped page-locked word on
  // the caller's stream; without it (allocation refused) p2p_sync falls back to a copy
  void* h = nullptr;
  void* hd = nullptr;
  if (cudaHostAlloc(&h, sizeof(int32_t), cudaHostAllocMapped) == cudaSuccess &&
      cudaHostGetDevicePointer(&hd, h, 0) == cudaSuccess) {
    ctx->host_err = static_cast<int32_t*>(h);
    ctx->host_err_dev = static_cast<int32_t*>(hd);
  } else {
    if (h) cudaFreeHost(h);
    cudaGetLastError();
  }
  // Place the no-alloc entry point's fixed scratch array on this device now, at start-up,
  // rather than at that entry point's first call (after which a host may have given the rest
  // of the device's memory to its own pool).
  if (p2p::noalloc_prepare(device) != cudaSuccess) {
    cudaGetLastError();
    p2p_ctx_destroy(ctx);
    return P2P_ERR_CUDA;
  }
  *out = ctx;
  return P2P_OK;
}

p2p_status p2p_ctx_destroy(p2p_ctx* ctx) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  for (auto& kv : ctx->rope) cudaFree(kv.second);
  for (auto& kv : ctx->shared) dev_free(kv.first, kv.second);
  dev_free(ctx->meta, 16);
  dev_free(ctx->dev_err, sizeof(int32_t));
  if (ctx->host_err) cudaFreeHost(ctx->host_err);
  dev_free(ctx->partials, ctx->partials_bytes);
  dev_free(ctx->counters, ctx->counters_bytes);
  dev_free(ctx->w16, ctx->w16_bytes);
  cudaStreamDestroy(ctx->stream);
  delete ctx;
  return P2P_OK;
}

const char* p2p_last_error(const p2p_ctx* ctx) { return ctx ? ctx->err.c_str() : "no context"; }

void* p2p_ctx_stream(p2p_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

namespace {
__global__ void take_error_word(int32_t* dev_err, int32_t* host_err) {
  *static_cast<volatile int32_t*>(host_err) = atomicExch(dev_err, 0);
}
}  // namespace

p2p_status p2p_sync(p2p_ctx* ctx, void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  int32_t flags = 0;
  cudaError_t e;
  if (ctx->host_err_dev) {
    // behind the stream's work, one thread swaps the error word to 0 and stores what it held
    // in mapped host memory: one stream synchronization, no device-wide one, no copy engine
    take_error_word<<<1, 1, 0, s>>>(ctx->dev_err, ctx->host_err_dev);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "reading the device error word");
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamSynchronize");
    flags = *static_cast<volatile int32_t*>(ctx->host_err);
  } else {
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamSynchronize");
    e = cudaMemcpy(&flags, ctx->dev_err, sizeof flags, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "reading the device error word");
  }
  if (flags) {
    if (!ctx->host_err_dev) {
      cudaMemsetAsync(ctx->dev_err, 0, sizeof flags, s);
      cudaStreamSynchronize(s);
    }
    if (flags & p2p::kErrPosBeyondCache)
      return fail(ctx, P2P_ERR_KV_FULL,
                  "a kernel was given a device-side position beyond its KV cache; that work "
                  "was skipped");
    if (flags & p2p::kErrTimeout)
      return fail(ctx, P2P_ERR_TIMEOUT,
                  "a kernel's bounded wait on another CTA ran out; its output was not written");
    if (flags & p2p::kErrLayout)
      return fail(ctx, P2P_ERR_CUDA,
                  "a kernel's dynamic shared memory did not start on the 1024-byte boundary "
                  "its tiles need; that work was skipped");
    if (flags & p2p::kErrOutTokFull)
      return fail(ctx, P2P_ERR_INVALID_ARG,
                  "argmax_step: the step index in the meta buffer reached out_tok's capacity; "
                  "that token was not stored (tok and the meta buffer were still updated)");
  }
  return P2P_OK;
}

// Test hook (not part of the reference contract): make bounded device waits run out.
p2p_status p2p_debug_set_wait_deficit(int32_t bytes) {
  if (bytes < 0 || bytes > (1 << 19)) return P2P_ERR_INVALID_ARG;
  g_wait_deficit.store(bytes);
  return P2P_OK;
}

// Test hook (not part of the reference contract): cap this process's device allocations.
p2p_status p2p_debug_set_alloc_limit(int64_t bytes) {
  std::lock_guard<std::mutex> lk(g_alloc_mu);
  g_alloc_limit = bytes;
  return P2P_OK;
}

p2p_status p2p_rope_table(p2p_ctx* ctx, int32_t max_ctx, int32_t head_dim, double theta,
                          int32_t dtype, const void** dev_table) {
  if (!ctx || !dev_table) return P2P_ERR_INVALID_ARG;
  if (max_ctx <= 0 || head_dim <= 0 || head_dim % 2 || !(theta > 0.0))
    return fail(ctx, P2P_ERR_INVALID_ARG, "rope table: max_ctx %d head_dim %d theta %g",
                max_ctx, head_dim, theta);
  if (dtype != P2P_F16 && dtype != P2P_F32)
    return fail(ctx, P2P_ERR_INVALID_ARG, "rope table dtype %d", dtype);
  auto key = std::make_tuple(max_ctx, head_dim, theta, dtype);
  auto it = ctx->rope.find(key);
  if (it != ctx->rope.end()) {
    *dev_table = it->second;
    return P2P_OK;
  }
  const int half = head_dim / 2;
  const size_t n = size_t(max_ctx) * head_dim;
  std::vector<uint16_t> h16;
  std::vector<float> h32;
  if (dtype == P2P_F16) h16.resize(n);
  else h32.resize(n);
  for (int p = 0; p < max_ctx; ++p)
    for (int i = 0; i < half; ++i) {  // engine.js:64-67
      const double ang = double(p) * std::pow(theta, double(-i) / double(half));
      const float c = float(std::cos(ang)), s = float(std::sin(ang));
      const size_t o = size_t(p) * head_dim;
      if (dtype == P2P_F16) {
        h16[o + i] = half_bits(c);
        h16[o + half + i] = half_bits(s);
      } else {
        h32[o + i] = c;
        h32[o + half + i] = s;
      }
    }
  DeviceGuard g(ctx->device);
  void* d = nullptr;
  const size_t bytes = n * elem_bytes(dtype);
  if (dev_alloc(&d, bytes) != cudaSuccess) return fail(ctx, P2P_ERR_OOM, "rope table");
  cudaError_t e = cudaMemcpy(d, dtype == P2P_F16 ? static_cast<const void*>(h16.data())
                                                 : static_cast<const void*>(h32.data()),
                             bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    dev_free(d, bytes);
    return cuda_fail(ctx, e, "rope upload");
  }
  ctx->rope[key] = d;
  *dev_table = d;
  return P2P_OK;
}

p2p_status p2p_meta(p2p_ctx* ctx, uint32_t** dev_meta) {
  if (!ctx || !dev_meta) return P2P_ERR_INVALID_ARG;
  *dev_meta = ctx->meta;
  return P2P_OK;
}

p2p_status p2p_meta_write(p2p_ctx* ctx, uint32_t pos0, uint32_t m_tokens, uint32_t step,
                          void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  // A small pageable source: cudaMemcpyAsync stages it before returning, so the local array
  // may go out of scope immediately.
  const uint32_t v[4] = {pos0, m_tokens, step, 0u};
  cudaError_t e =
      cudaMemcpyAsync(ctx->meta, v, sizeof v, cudaMemcpyHostToDevice, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(ctx, e, "meta write");
  return P2P_OK;
}

p2p_status p2p_argmax_step(p2p_ctx* ctx, const void* logits, int32_t vocab, uint32_t* tok,
                           uint32_t* out_tok, int64_t out_tok_cap, uint32_t* meta_dev,
                           void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  if (!logits || !tok || !out_tok || vocab <= 0 || out_tok_cap <= 0)
    return fail(ctx, P2P_ERR_INVALID_ARG, "argmax_step: NULL buffer, vocab %d or out_tok_cap %lld",
                vocab, (long long)out_tok_cap);
  DeviceGuard g(ctx->device);
  cudaError_t e = p2p::launch_argmax_step(logits, vocab, tok, out_tok, out_tok_cap,
                                          meta_dev ? meta_dev : ctx->meta, ctx->dev_err,
                                          pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(ctx, e, "argmax launch");
  return P2P_OK;
}

p2p_status p2p_kv_create(p2p_ctx* ctx, int32_t n_layers, int32_t num_kv_heads,
                         int32_t head_dim, int64_t cap_tokens, int32_t dtype, p2p_kv** out) {
  if (!ctx || !out) return P2P_ERR_INVALID_ARG;
  *out = nullptr;
  if (n_layers <= 0 || num_kv_heads <= 0 || head_dim != 64 || cap_tokens <= 0 ||
      (dtype != P2P_F16 && dtype != P2P_F32))
    return fail(ctx, P2P_ERR_INVALID_ARG, "kv_create: layers %d kv_heads %d head_dim %d cap %lld",
                n_layers, num_kv_heads, head_dim, (long long)cap_tokens);
  DeviceGuard g(ctx->device);
  p2p_kv* kv = new (std::nothrow) p2p_kv;
  if (!kv) return P2P_ERR_OOM;
  kv->ctx = ctx;
  kv->n_layers = n_layers;
  kv->hkv = num_kv_heads;
  kv->d = head_dim;
  kv->dtype = dtype;
  kv->cap = cap_tokens;
  const size_t bytes = size_t(cap_tokens) * num_kv_heads * head_dim * elem_bytes(dtype);
  for (int l = 0; l < n_layers; ++l) {
    void* k = nullptr;
    void* v = nullptr;
    if (dev_alloc(&k, bytes) != cudaSuccess || dev_alloc(&v, bytes) != cudaSuccess) {
      dev_free(k, k ? bytes : 0);
      for (size_t i = 0; i < kv->k.size(); ++i) {
        dev_free(kv->k[i], bytes);
        dev_free(kv->v[i], bytes);
      }
      delete kv;
      return fail(ctx, P2P_ERR_OOM, "kv cache of %zu bytes per buffer", bytes);
    }
    kv->k.push_back(k);
    kv->v.push_back(v);
  }
  *out = kv;
  return P2P_OK;
}

p2p_status p2p_kv_destroy(p2p_kv* kv) {
  if (!kv) return P2P_ERR_INVALID_ARG;
  DeviceGuard g(kv->ctx->device);
  cudaDeviceSynchronize();
  const size_t bytes = size_t(kv->cap) * kv->hkv * kv->d * elem_bytes(kv->dtype);
  for (int l = 0; l < kv->n_layers; ++l) {
    dev_free(kv->k[l], bytes);
    dev_free(kv->v[l], bytes);
  }
  delete kv;
  return P2P_OK;
}

p2p_status p2p_kv_ensure_capacity(p2p_kv* kv, int64_t need_tokens, int64_t grow_tokens,
                                  int64_t max_tokens, void* stream) {
  if (!kv) return P2P_ERR_INVALID_ARG;
  p2p_ctx* ctx = kv->ctx;
  if (need_tokens <= kv->cap) return P2P_OK;                  // engine.js:275
  if (need_tokens > max_tokens)                               // engine.js:276
    return fail(ctx, P2P_ERR_KV_FULL, "need %lld tokens > max %lld", (long long)need_tokens,
                (long long)max_tokens);
  if (grow_tokens <= 0) grow_tokens = 1;
  int64_t nc = kv->cap;
  while (nc < need_tokens) nc += grow_tokens;                 // engine.js:277-279
  if (nc > max_tokens) nc = max_tokens;
  DeviceGuard g(ctx->device);
  const size_t eb = size_t(kv->hkv) * kv->d * elem_bytes(kv->dtype);
  const size_t nbytes = size_t(nc) * eb, obytes = size_t(kv->cap) * eb;
  std::vector<void*> nk, nv;
  for (int l = 0; l < kv->n_layers; ++l) {                    // engine.js:280-286
    void* k = nullptr;
    void* v = nullptr;
    const bool ok = dev_alloc(&k, nbytes) == cudaSuccess && dev_alloc(&v, nbytes) == cudaSuccess;
    if (k) nk.push_back(k);
    if (v) nv.push_back(v);
    if (!ok) {
      for (void* p : nk) dev_free(p, nbytes);
      for (void* p : nv) dev_free(p, nbytes);
      return fail(ctx, P2P_ERR_OOM, "kv growth to %lld tokens", (long long)nc);
    }
  }
  cudaStream_t s = pick_stream(ctx, stream);
  for (int l = 0; l < kv->n_layers; ++l) {                    // engine.js:287-293
    cudaMemcpyAsync(nk[l], kv->k[l], obytes, cudaMemcpyDeviceToDevice, s);
    cudaMemcpyAsync(nv[l], kv->v[l], obytes, cudaMemcpyDeviceToDevice, s);
  }
  cudaError_t e = cudaStreamSynchronize(s);                   // engine.js:301
  for (int l = 0; l < kv->n_layers; ++l) {                    // engine.js:302
    dev_free(kv->k[l], obytes);
    dev_free(kv->v[l], obytes);
  }
  kv->k = nk;
  kv->v = nv;
  kv->cap = nc;
  if (e != cudaSuccess) return cuda_fail(ctx, e, "kv growth copy");
  return P2P_OK;
}

int64_t p2p_kv_capacity(const p2p_kv* kv) { return kv ? kv->cap : 0; }
void* p2p_kv_k(const p2p_kv* kv, int32_t layer) {
  return (kv && layer >= 0 && layer < kv->n_layers) ? kv->k[layer] : nullptr;
}
void* p2p_kv_v(const p2p_kv* kv, int32_t layer) {
  return (kv && layer >= 0 && layer < kv->n_layers) ? kv->v[layer] : nullptr;
}

p2p_status p2p_qk_prep(p2p_ctx* ctx, const p2p_attn_params* prm, const void* qkv,
                       int64_t ld_qkv, const void* norm_w, const void* rope, void* q_out,
                       int64_t ld_q, void* k_cache, void* v_cache, int64_t kv_cap_tokens,
                       const uint32_t* meta_dev, int32_t pos0, int32_t m_tokens, void* stream) {
  p2p_status st = check_params(ctx, prm, true);
  if (st != P2P_OK) return st;
  const int64_t row = int64_t(prm->num_heads + 2 * prm->num_kv_heads) * prm->head_dim;
  if (!qkv || !rope || !q_out || !k_cache || !v_cache)
    return fail(ctx, P2P_ERR_INVALID_ARG, "qk_prep: NULL buffer");
  if (m_tokens < 0 || m_tokens > 65535 || ld_qkv < row ||
      ld_q < int64_t(prm->num_heads) * prm->head_dim || (!meta_dev && pos0 < 0) ||
      kv_cap_tokens <= 0)
    return fail(ctx, P2P_ERR_INVALID_ARG, "qk_prep: M %d ld_qkv %lld ld_q %lld pos0 %d cap %lld",
                m_tokens, (long long)ld_qkv, (long long)ld_q, pos0, (long long)kv_cap_tokens);
  if (!meta_dev && int64_t(pos0) + m_tokens > kv_cap_tokens)
    return fail(ctx, P2P_ERR_KV_FULL, "qk_prep: pos0 %d + M %d > cache rows %lld", pos0,
                m_tokens, (long long)kv_cap_tokens);
  DeviceGuard g(ctx->device);
  p2p::QkPrepArgs a{qkv, ld_qkv, norm_w, rope, q_out, ld_q, k_cache, v_cache, kv_cap_tokens,
                    meta_dev, pos0, m_tokens, prm->num_heads, prm->num_kv_heads, eff_eps(prm),
                    ctx->dev_err};
  cudaError_t e = p2p::launch_qk_prep(a, prm->dtype, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(ctx, e, "qk_prep launch");
  return P2P_OK;
}

p2p_status p2p_attn(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q, int64_t ld_q,
                    const void* k_cache, const void* v_cache, int64_t kv_cap_tokens, void* out,
                    int64_t ld_o, const uint32_t* meta_dev, int32_t pos0, int32_t m_tokens,
                    void* stream) {
  p2p_status st = check_params(ctx, prm, m_tokens == 1);
  if (st != P2P_OK) return st;
  const int64_t qw = int64_t(prm->num_heads) * prm->head_dim;
  if (!q || !k_cache || !v_cache || !out) return fail(ctx, P2P_ERR_INVALID_ARG, "attn: NULL buffer");
  if (m_tokens < 0 || ld_q < qw || ld_o < qw || kv_cap_tokens <= 0 || (!meta_dev && pos0 < 0))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn: M %d ld_q %lld ld_o %lld cap %lld pos0 %d",
                m_tokens, (long long)ld_q, (long long)ld_o, (long long)kv_cap_tokens, pos0);
  if (!meta_dev && int64_t(pos0) + m_tokens > kv_cap_tokens)
    return fail(ctx, P2P_ERR_KV_FULL, "attn: pos0 %d + M %d > cache rows %lld", pos0, m_tokens,
                (long long)kv_cap_tokens);
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn: cache buffers must be 16-byte aligned");
  if (m_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  if (m_tokens == 1) {
    p2p::DecodeArgs a{};
    a.layers[0] = {q, nullptr, const_cast<void*>(k_cache), const_cast<void*>(v_cache), out};
    a.meta = meta_dev;
    a.pos_host = pos0;
    a.kv_cap = kv_cap_tokens;
    const int64_t max_len = meta_dev ? kv_cap_tokens : int64_t(pos0) + 1;
    return run_decode(ctx, prm, a, p2p::kLayers, false, 1, max_len, s);
  }
  if ((ld_q % 8) || (ld_o % 8) || !aligned16(q) || !aligned16(out))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn prefill: q/out must be 16-byte aligned rows");
  return run_causal_flash(ctx, prm, q, ld_q, k_cache, v_cache, kv_cap_tokens, &out, 1, ld_o, 0,
                          meta_dev, pos0, m_tokens, s);
}

static_assert(P2P_MAX_SCATTER_OUTS == p2p::kMaxFlashOuts, "one flash launch writes every output");

p2p_status p2p_attn_scatter(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q,
                            int64_t ld_q, const void* k_cache, const void* v_cache,
                            int64_t kv_cap_tokens, void* const* outs, int32_t n_outs,
                            int64_t ld_o, int32_t out_head0, const uint32_t* meta_dev,
                            int32_t pos0, int32_t m_tokens, void* stream) {
  p2p_status st = check_params(ctx, prm, false);
  if (st != P2P_OK) return st;
  const int64_t qw = int64_t(prm->num_heads) * prm->head_dim;
  if (!q || !k_cache || !v_cache || !outs || n_outs < 1 || n_outs > P2P_MAX_SCATTER_OUTS)
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn_scatter: NULL buffer or %d outputs (1..%d)",
                n_outs, P2P_MAX_SCATTER_OUTS);
  for (int t = 0; t < n_outs; ++t)
    if (!outs[t] || !aligned16(outs[t]))
      return fail(ctx, P2P_ERR_INVALID_ARG, "attn_scatter: output %d is NULL or misaligned", t);
  if (m_tokens < 0 || ld_q < qw || out_head0 < 0 || ld_o < (int64_t(out_head0) * prm->head_dim + qw) ||
      kv_cap_tokens <= 0 || (!meta_dev && pos0 < 0) || (ld_q % 8) || (ld_o % 8) || !aligned16(q))
    return fail(ctx, P2P_ERR_INVALID_ARG,
                "attn_scatter: M %d ld_q %lld ld_o %lld out_head0 %d cap %lld pos0 %d", m_tokens,
                (long long)ld_q, (long long)ld_o, out_head0, (long long)kv_cap_tokens, pos0);
  if (!meta_dev && int64_t(pos0) + m_tokens > kv_cap_tokens)
    return fail(ctx, P2P_ERR_KV_FULL, "attn_scatter: pos0 %d + M %d > cache rows %lld", pos0,
                m_tokens, (long long)kv_cap_tokens);
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn_scatter: cache buffers must be 16-byte aligned");
  if (m_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  return run_causal_flash(ctx, prm, q, ld_q, k_cache, v_cache, kv_cap_tokens, outs, n_outs, ld_o,
                          out_head0, meta_dev, pos0, m_tokens, pick_stream(ctx, stream));
}

p2p_status p2p_attn_multicast(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q,
                              int64_t ld_q, const void* k_cache, const void* v_cache,
                              int64_t kv_cap_tokens, void* mc_out, int64_t ld_o,
                              int32_t out_head0, const uint32_t* meta_dev, int32_t pos0,
                              int32_t m_tokens, void* stream) {
  p2p_status st = check_params(ctx, prm, false);
  if (st != P2P_OK) return st;
  const int64_t qw = int64_t(prm->num_heads) * prm->head_dim;
  if (!q || !k_cache || !v_cache || !mc_out || !aligned16(mc_out))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn_multicast: NULL or misaligned buffer");
  if (m_tokens < 0 || ld_q < qw || out_head0 < 0 || ld_o < (int64_t(out_head0) * prm->head_dim + qw) ||
      kv_cap_tokens <= 0 || (!meta_dev && pos0 < 0) || (ld_q % 8) || (ld_o % 8) || !aligned16(q))
    return fail(ctx, P2P_ERR_INVALID_ARG,
                "attn_multicast: M %d ld_q %lld ld_o %lld out_head0 %d cap %lld pos0 %d", m_tokens,
                (long long)ld_q, (long long)ld_o, out_head0, (long long)kv_cap_tokens, pos0);
  if (!meta_dev && int64_t(pos0) + m_tokens > kv_cap_tokens)
    return fail(ctx, P2P_ERR_KV_FULL, "attn_multicast: pos0 %d + M %d > cache rows %lld", pos0,
                m_tokens, (long long)kv_cap_tokens);
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn_multicast: cache buffers must be 16-byte aligned");
  if (m_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  // the kernel stores through mc_out alone; it also fills the launcher's one output slot
  return run_causal_flash(ctx, prm, q, ld_q, k_cache, v_cache, kv_cap_tokens, &mc_out, 1, ld_o,
                          out_head0, meta_dev, pos0, m_tokens, pick_stream(ctx, stream), mc_out);
}

p2p_status p2p_shared_alloc(p2p_ctx* ctx, size_t bytes, void** ptr,
                            unsigned char handle[P2P_IPC_HANDLE_BYTES]) {
  if (!ctx || !ptr || !handle || bytes == 0) return P2P_ERR_INVALID_ARG;
  *ptr = nullptr;
  DeviceGuard g(ctx->device);
  void* p = nullptr;
  if (dev_alloc(&p, bytes) != cudaSuccess) return fail(ctx, P2P_ERR_OOM, "shared buffer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    dev_free(p, bytes);
    return cuda_fail(ctx, e, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(h) <= P2P_IPC_HANDLE_BYTES, "IPC handle size");
  std::memset(handle, 0, P2P_IPC_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof(h));
  ctx->shared[p] = bytes;
  *ptr = p;
  return P2P_OK;
}

p2p_status p2p_shared_free(p2p_ctx* ctx, void* ptr) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  const auto it = ctx->shared.find(ptr);
  if (it == ctx->shared.end()) return fail(ctx, P2P_ERR_INVALID_ARG, "shared_free: unknown buffer");
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  dev_free(it->first, it->second);
  ctx->shared.erase(it);
  return P2P_OK;
}

p2p_status p2p_shared_open(p2p_ctx* ctx, const unsigned char handle[P2P_IPC_HANDLE_BYTES],
                           void** ptr) {
  if (!ctx || !handle || !ptr) return P2P_ERR_INVALID_ARG;
  *ptr = nullptr;
  DeviceGuard g(ctx->device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaIpcOpenMemHandle");
  return P2P_OK;
}

p2p_status p2p_shared_close(p2p_ctx* ctx, void* ptr) {
  if (!ctx || !ptr) return P2P_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaIpcCloseMemHandle");
  return P2P_OK;
}

p2p_status p2p_decode_step(p2p_ctx* ctx, const p2p_attn_params* prm, int32_t n_layers,
                           const p2p_decode_layer* layers, const void* rope,
                           int64_t kv_cap_tokens, const uint32_t* meta_dev, int32_t pos,
                           void* stream) {
  p2p_status st = check_params(ctx, prm, true);
  if (st != P2P_OK) return st;
  if (n_layers <= 0 || n_layers > P2P_MAX_LAYERS || !layers || !rope)
    return fail(ctx, P2P_ERR_INVALID_ARG, "decode_step: n_layers %d (max %d)", n_layers,
                P2P_MAX_LAYERS);
  if (kv_cap_tokens <= 0 || (!meta_dev && (pos < 0 || int64_t(pos) >= kv_cap_tokens)))
    return fail(ctx, meta_dev ? P2P_ERR_INVALID_ARG : P2P_ERR_KV_FULL,
                "decode_step: pos %d cache rows %lld", pos, (long long)kv_cap_tokens);
  p2p::DecodeArgs a{};
  for (int l = 0; l < n_layers; ++l) {
    const p2p_decode_layer& L = layers[l];
    if (!L.qkv || !L.k_cache || !L.v_cache || !L.out || !aligned16(L.k_cache) ||
        !aligned16(L.v_cache))
      return fail(ctx, P2P_ERR_INVALID_ARG, "decode_step: layer %d has a NULL or misaligned buffer", l);
    a.layers[l] = {L.qkv, L.norm_w, L.k_cache, L.v_cache, L.out};
  }
  a.rope = rope;
  a.meta = meta_dev;
  a.pos_host = pos;
  a.kv_cap = kv_cap_tokens;
  DeviceGuard g(ctx->device);
  // qkv rows in page-locked host memory: let one CTA of each cluster read them (the others get
  // the rotated q through distributed shared memory) instead of every split crossing the link
  cudaPointerAttributes pa{};
  if (cudaPointerGetAttributes(&pa, layers[0].qkv) == cudaSuccess)
    a.q_bcast = pa.type == cudaMemoryTypeHost ? 1 : 0;
  else
    cudaGetLastError();
  const int64_t max_len = meta_dev ? kv_cap_tokens : int64_t(pos) + 1;
  return run_decode(ctx, prm, a, p2p::kLayers, true, n_layers, max_len,
                    pick_stream(ctx, stream));
}

p2p_status p2p_attn_decode_ragged(p2p_ctx* ctx, const p2p_attn_params* prm, const void* qkv,
                                  int64_t ld_qkv, const void* norm_w, const void* rope,
                                  void* k_cache, void* v_cache, int64_t kv_rows,
                                  const int32_t* offsets, const int32_t* past, int32_t nseq,
                                  int32_t max_past, int32_t fused_prep, void* out, int64_t ld_o,
                                  void* stream) {
  p2p_status st = p2p::check_ragged(ctx, prm, qkv, ld_qkv, rope, k_cache, v_cache, kv_rows,
                                    offsets, past, nseq, max_past, fused_prep, out, ld_o,
                                    "decode_ragged");
  if (st != P2P_OK || nseq == 0) return st;
  p2p::DecodeArgs a{};
  p2p::fill_ragged(a, qkv, ld_qkv, norm_w, rope, k_cache, v_cache, kv_rows, offsets, past,
                   max_past, out, ld_o);
  DeviceGuard g(ctx->device);
  return run_decode(ctx, prm, a, p2p::kRagged, fused_prep != 0, nseq, int64_t(max_past) + 1,
                    pick_stream(ctx, stream));
}

p2p_status p2p_attn_decode_kv(p2p_ctx* ctx, const p2p_attn_params* prm,
                              const p2p_kv_layout* lay, const void* qkv, int64_t ld_qkv,
                              const void* norm_w, const void* rope, void* k_cache,
                              void* v_cache, int64_t kv_rows, const int32_t* offsets,
                              const int32_t* past, int32_t nseq, int32_t max_past,
                              int32_t fused_prep, void* out, int64_t ld_o, void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  if (!lay) return fail(ctx, P2P_ERR_INVALID_ARG, "decode_kv: layout is NULL");
  const bool paged = lay->block_size != 0;
  // the contiguous form needs offsets; the paged one ignores them (checked as non-NULL below)
  const int32_t* offs = paged ? past : offsets;
  p2p_status st = p2p::check_ragged(ctx, prm, qkv, ld_qkv, rope, k_cache, v_cache, kv_rows, offs,
                                    past, nseq, max_past, fused_prep, out, ld_o, "decode_kv");
  if (st != P2P_OK) return st;
  if (prm->dtype != P2P_F16)
    return fail(ctx, P2P_ERR_UNSUPPORTED, "decode_kv: q/out must be f16");
  if (lay->format != P2P_KV_F16 && lay->format != P2P_KV_I8)
    return fail(ctx, P2P_ERR_INVALID_ARG, "decode_kv: format %d", lay->format);
  const int chan = prm->num_kv_heads * prm->head_dim;
  if (lay->format == P2P_KV_I8 &&
      (!lay->k_scale || !lay->v_scale || (lay->scale_count != 1 && lay->scale_count != chan)))
    return fail(ctx, P2P_ERR_INVALID_ARG,
                "decode_kv: int8 caches need k/v scales, 1 or %d of them (got %d)", chan,
                lay->scale_count);
  int shift = 0;
  if (paged) {
    const int bs = lay->block_size;
    if (bs < 16 || bs > 4096 || (bs & (bs - 1)) || !lay->block_table || lay->max_blocks <= 0)
      return fail(ctx, P2P_ERR_INVALID_ARG,
                  "decode_kv: block_size %d (a power of two in 16..4096), block table %p, "
                  "max_blocks %d", bs, (const void*)lay->block_table, lay->max_blocks);
    while ((1 << shift) < bs) ++shift;
    if (int64_t(max_past) >= (int64_t(lay->max_blocks) << shift))
      return fail(ctx, P2P_ERR_INVALID_ARG, "decode_kv: max_past %d beyond %d blocks of %d",
                  max_past, lay->max_blocks, bs);
  } else if (!offsets) {
    return fail(ctx, P2P_ERR_INVALID_ARG, "decode_kv: contiguous caches need offsets");
  }
  if (nseq == 0) return P2P_OK;
  p2p::DecodeArgs a{};
  p2p::fill_ragged(a, qkv, ld_qkv, norm_w, rope, k_cache, v_cache, kv_rows, offsets, past,
                   max_past, out, ld_o);
  a.block_table = lay->block_table;
  a.max_blocks = lay->max_blocks;
  a.block_shift = shift;
  a.kv_format = lay->format == P2P_KV_I8 ? p2p::kKvI8 : p2p::kKvF16;
  a.k_scale = lay->k_scale;
  a.v_scale = lay->v_scale;
  a.scale_per_channel = lay->scale_count > 1 ? 1 : 0;
  DeviceGuard g(ctx->device);
  return run_decode(ctx, prm, a, paged ? p2p::kPaged : p2p::kRagged, fused_prep != 0, nseq,
                    int64_t(max_past) + 1, pick_stream(ctx, stream));
}

namespace {
// Validation of one MatMulNBits matrix argument: rows, k, alignment of its three buffers.
p2p_status check_q4(p2p_ctx* ctx, const p2p_q4_matrix* w, int32_t n, int32_t k,
                    const char* what, int32_t max_k = p2p::kGemvMaxK) {
  if (!w || !w->qweight || !w->scales || !w->zero_points)
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: NULL matrix or buffer", what);
  if ((n >= 0 && w->n != n) || w->n <= 0 || w->k != k || k <= 0 || k % 32 || k > max_k)
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: n %d (want %d), k %d (want %d; a multiple of "
                "32, at most %d)", what, w->n, n, w->k, k, max_k);
  if ((reinterpret_cast<uintptr_t>(w->qweight) | reinterpret_cast<uintptr_t>(w->zero_points)) &
          3u ||
      reinterpret_cast<uintptr_t>(w->scales) & 1u)
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: qweight / zero_points must be 4-byte aligned, "
                "scales 2-byte", what);
  return P2P_OK;
}
p2p::Q4Matrix to_q4(const p2p_q4_matrix* w) {
  return {static_cast<const uint32_t*>(w->qweight), static_cast<const __half*>(w->scales),
          static_cast<const uint32_t*>(w->zero_points), w->n};
}
}  // namespace

p2p_status p2p_gemv_q4(p2p_ctx* ctx, const p2p_q4_matrix* w, const void* x, void* y,
                       int64_t y_off, void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  p2p_status st = check_q4(ctx, w, -1, w ? w->k : 0, "gemv_q4");
  if (st != P2P_OK) return st;
  if (!x || !y || !aligned16(x) || y_off < 0 || (reinterpret_cast<uintptr_t>(y) & 1u))
    return fail(ctx, P2P_ERR_INVALID_ARG, "gemv_q4: x must be 16-byte aligned, y non-NULL");
  DeviceGuard g(ctx->device);
  p2p::GemvArgs a{to_q4(w), w->k, x, y, y_off};
  cudaError_t e = p2p::launch_gemv_q4(a, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(ctx, e, "gemv_q4 launch");
  return P2P_OK;
}

p2p_status p2p_qkv_gemv_prep(p2p_ctx* ctx, const p2p_attn_params* prm, const void* x,
                             const p2p_q4_matrix* wq, const p2p_q4_matrix* wk,
                             const p2p_q4_matrix* wv, const void* norm_w, const void* rope,
                             void* q_out, void* k_cache, void* v_cache, int64_t kv_cap_tokens,
                             const uint32_t* meta_dev, int32_t pos, void* stream) {
  p2p_status st = check_params(ctx, prm, false);
  if (st != P2P_OK) return st;
  if (prm->dtype != P2P_F16)
    return fail(ctx, P2P_ERR_UNSUPPORTED, "qkv_gemv_prep: the projection path is f16");
  const int k = wq ? wq->k : 0;
  const int qn = prm->num_heads * prm->head_dim, kn = prm->num_kv_heads * prm->head_dim;
  if ((st = check_q4(ctx, wq, qn, k, "qkv_gemv_prep (wq)")) != P2P_OK) return st;
  if ((st = check_q4(ctx, wk, kn, k, "qkv_gemv_prep (wk)")) != P2P_OK) return st;
  if ((st = check_q4(ctx, wv, kn, k, "qkv_gemv_prep (wv)")) != P2P_OK) return st;
  if (!x || !aligned16(x) || !rope || !q_out || !k_cache || !v_cache || kv_cap_tokens <= 0 ||
      (!meta_dev && pos < 0))
    return fail(ctx, P2P_ERR_INVALID_ARG, "qkv_gemv_prep: NULL or misaligned buffer, cap or pos");
  if (!meta_dev && int64_t(pos) >= kv_cap_tokens)
    return fail(ctx, P2P_ERR_KV_FULL, "qkv_gemv_prep: pos %d >= cache rows %lld", pos,
                (long long)kv_cap_tokens);
  DeviceGuard g(ctx->device);
  p2p::QkvPrepArgs a{to_q4(wq), to_q4(wk), to_q4(wv), k, x, norm_w, rope, q_out, k_cache,
                     v_cache, kv_cap_tokens, meta_dev, pos, prm->num_heads, prm->num_kv_heads,
                     eff_eps(prm), ctx->dev_err};
  cudaError_t e = p2p::launch_qkv_prep(a, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(ctx, e, "qkv_gemv_prep launch");
  return P2P_OK;
}

// P2P_GEMM_BN=256|192|128 fixes the GEMM's output tile width and P2P_GEMM_PAIR=0|1 its form
// (one CTA or a 2-CTA pair per tile; tests compare them on one shape); unset or anything
// else: chosen per shape.
static int gemm_bn_override() {
  const char* v = std::getenv("P2P_GEMM_BN");
  if (!v) return 0;
  const int bn = std::atoi(v);
  return (bn == 256 || bn == 192 || bn == 128) ? bn : 0;
}
static int gemm_pair_override() {
  const char* v = std::getenv("P2P_GEMM_PAIR");
  if (!v || (std::strcmp(v, "0") && std::strcmp(v, "1"))) return -1;
  return std::atoi(v);
}

// ---- prompt-chunk GEMM (kernels.js:70-145) -------------------------------------------------
// Shared by the 4-bit entry points (dequantise into the context's workspace first) and the
// f16-weight ones (weights made once by p2p_q4_to_f16).
static p2p_status gemm_check(p2p_ctx* ctx, int32_t n, int32_t k, const void* x, int64_t ld_x,
                             int32_t m_tokens, const void* y, int64_t ld_y, int64_t y_off,
                             const char* what) {
  if (!x || !y || m_tokens < 0 || ld_x < k || y_off < 0 || ld_y < y_off + n)
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: M %d ld_x %lld ld_y %lld y_off %lld", what,
                m_tokens, (long long)ld_x, (long long)ld_y, (long long)y_off);
  if (n % 64 || !aligned16(x) || (ld_x % 8) || !aligned16(y) || (ld_y % 8) || (y_off % 8))
    return fail(ctx, P2P_ERR_INVALID_ARG,
                "%s: n a multiple of 64, 16-byte aligned rows of x and y, y_off %% 8 == 0", what);
  return P2P_OK;
}

static p2p_status gemm_run(p2p_ctx* ctx, const void* w16, int32_t n, int32_t k, const void* x,
                           int64_t ld_x, int32_t m_tokens, void* y, int64_t ld_y, int64_t y_off,
                           cudaStream_t s, const char* what) {
  p2p::GemmArgs a{};
  a.x = x;
  a.ld_x = ld_x;
  a.w16 = w16;
  a.m = m_tokens;
  a.n = n;
  a.k = k;
  a.y = y;
  a.ld_y = ld_y;
  a.y_off = y_off;
  a.err = ctx->dev_err;
  a.bn = gemm_bn_override();
  a.pair = gemm_pair_override();
  const cudaError_t e = p2p::launch_gemm(a, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  return P2P_OK;
}

struct QkvPrepIo {
  const void* x;
  int64_t ld_x;
  const void* norm_w;
  const void* rope;
  void* q_out;
  int64_t ld_q;
  void* k_cache;
  void* v_cache;
  int64_t kv_cap;
  const uint32_t* meta;
  int32_t pos0, m;
};

static p2p_status qkv_check(p2p_ctx* ctx, const p2p_attn_params* prm, int32_t k,
                            const QkvPrepIo& io, const char* what) {
  p2p_status st = check_params(ctx, prm, false);
  if (st != P2P_OK) return st;
  if (prm->dtype != P2P_F16)
    return fail(ctx, P2P_ERR_UNSUPPORTED, "%s: the projection path is f16", what);
  const int qn = prm->num_heads * prm->head_dim;
  if (!io.x || !io.rope || !io.q_out || !io.k_cache || !io.v_cache || io.m < 0 ||
      io.ld_x < k || io.ld_q < qn || io.kv_cap <= 0 || (!io.meta && io.pos0 < 0))
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: M %d ld_x %lld ld_q %lld pos0 %d", what, io.m,
                (long long)io.ld_x, (long long)io.ld_q, io.pos0);
  if (!aligned16(io.x) || (io.ld_x % 8) || !aligned16(io.q_out) || (io.ld_q % 8) ||
      !aligned16(io.rope) || !aligned16(io.k_cache) || !aligned16(io.v_cache))
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: 16-byte aligned rows needed", what);
  if (!io.meta && int64_t(io.pos0) + io.m > io.kv_cap)
    return fail(ctx, P2P_ERR_KV_FULL, "%s: pos0 %d + M %d > cache rows %lld", what, io.pos0,
                io.m, (long long)io.kv_cap);
  return P2P_OK;
}

static p2p_status qkv_run(p2p_ctx* ctx, const p2p_attn_params* prm, const void* w16, int32_t k,
                          const QkvPrepIo& io, cudaStream_t s, const char* what) {
  p2p::GemmArgs a{};
  a.x = io.x;
  a.ld_x = io.ld_x;
  a.w16 = w16;
  a.m = io.m;
  a.n = (prm->num_heads + 2 * prm->num_kv_heads) * prm->head_dim;
  a.k = k;
  a.prep = 1;
  a.hq = prm->num_heads;
  a.hkv = prm->num_kv_heads;
  a.norm_w = io.norm_w;
  a.rope = io.rope;
  a.eps = eff_eps(prm);
  a.q_out = io.q_out;
  a.ld_q = io.ld_q;
  a.k_cache = io.k_cache;
  a.v_cache = io.v_cache;
  a.kv_cap = io.kv_cap;
  a.meta = io.meta;
  a.pos0 = io.pos0;
  a.err = ctx->dev_err;
  a.bn = gemm_bn_override();
  a.pair = gemm_pair_override();
  const cudaError_t e = p2p::launch_gemm(a, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  return P2P_OK;
}

p2p_status p2p_gemm_q4(p2p_ctx* ctx, const p2p_q4_matrix* w, const void* x, int64_t ld_x,
                       int32_t m_tokens, void* y, int64_t ld_y, int64_t y_off, void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  p2p_status st = check_q4(ctx, w, -1, w ? w->k : 0, "gemm_q4", INT32_MAX);
  if (st != P2P_OK) return st;
  if ((st = gemm_check(ctx, w->n, w->k, x, ld_x, m_tokens, y, ld_y, y_off, "gemm_q4")) !=
      P2P_OK)
    return st;
  if (m_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  st = ensure_buffer(ctx, &ctx->w16, &ctx->w16_bytes, size_t(w->n) * w->k * 2,
                     "dequantised weights");
  if (st != P2P_OK) return st;
  const p2p::Q4Matrix wm = to_q4(w);
  cudaError_t e = p2p::launch_dequant_q4(&wm, 1, w->k, ctx->w16, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "gemm_q4 dequant launch");
  return gemm_run(ctx, ctx->w16, w->n, w->k, x, ld_x, m_tokens, y, ld_y, y_off, s,
                  "gemm_q4 launch");
}

p2p_status p2p_qkv_gemm_prep(p2p_ctx* ctx, const p2p_attn_params* prm, const void* x,
                             int64_t ld_x, const p2p_q4_matrix* wq, const p2p_q4_matrix* wk,
                             const p2p_q4_matrix* wv, const void* norm_w, const void* rope,
                             void* q_out, int64_t ld_q, void* k_cache, void* v_cache,
                             int64_t kv_cap_tokens, const uint32_t* meta_dev, int32_t pos0,
                             int32_t m_tokens, void* stream) {
  const QkvPrepIo io{x,       ld_x,    norm_w,        rope,     q_out, ld_q,
                     k_cache, v_cache, kv_cap_tokens, meta_dev, pos0,  m_tokens};
  const int k = wq ? wq->k : 0;
  p2p_status st = qkv_check(ctx, prm, k, io, "qkv_gemm_prep");
  if (st != P2P_OK) return st;
  const int qn = prm->num_heads * prm->head_dim, kn = prm->num_kv_heads * prm->head_dim;
  if ((st = check_q4(ctx, wq, qn, k, "qkv_gemm_prep (wq)", INT32_MAX)) != P2P_OK) return st;
  if ((st = check_q4(ctx, wk, kn, k, "qkv_gemm_prep (wk)", INT32_MAX)) != P2P_OK) return st;
  if ((st = check_q4(ctx, wv, kn, k, "qkv_gemm_prep (wv)", INT32_MAX)) != P2P_OK) return st;
  if (m_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = pick_stream(ctx, stream);
  st = ensure_buffer(ctx, &ctx->w16, &ctx->w16_bytes, size_t(qn + 2 * kn) * k * 2,
                     "dequantised weights");
  if (st != P2P_OK) return st;
  // one [q rows | k rows | v rows][k] operand (one launch): the projection's columns are the
  // qkv row's
  const p2p::Q4Matrix ws[3] = {to_q4(wq), to_q4(wk), to_q4(wv)};
  cudaError_t e = p2p::launch_dequant_q4(ws, 3, k, ctx->w16, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "qkv_gemm_prep dequant launch");
  return qkv_run(ctx, prm, ctx->w16, k, io, s, "qkv_gemm_prep launch");
}

p2p_status p2p_q4_to_f16(p2p_ctx* ctx, const p2p_q4_matrix* w, void* dst, void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  p2p_status st = check_q4(ctx, w, -1, w ? w->k : 0, "q4_to_f16", INT32_MAX);
  if (st != P2P_OK) return st;
  if (!dst || !aligned16(dst))
    return fail(ctx, P2P_ERR_INVALID_ARG, "q4_to_f16: dst must be a 16-byte aligned buffer");
  DeviceGuard g(ctx->device);
  const p2p::Q4Matrix wm = to_q4(w);
  const cudaError_t e = p2p::launch_dequant_q4(&wm, 1, w->k, dst, pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(ctx, e, "q4_to_f16 launch");
  return P2P_OK;
}

static p2p_status check_w16(p2p_ctx* ctx, const void* w16, int32_t n, int32_t k,
                            const char* what) {
  if (!w16 || !aligned16(w16) || n <= 0 || k <= 0 || (k % 8))
    return fail(ctx, P2P_ERR_INVALID_ARG,
                "%s: f16 weights [n][k], 16-byte aligned, k a multiple of 8 (n %d k %d)", what,
                n, k);
  return P2P_OK;
}

p2p_status p2p_gemm_f16w(p2p_ctx* ctx, const void* w16, int32_t n, int32_t k, const void* x,
                         int64_t ld_x, int32_t m_tokens, void* y, int64_t ld_y, int64_t y_off,
                         void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  p2p_status st = check_w16(ctx, w16, n, k, "gemm_f16w");
  if (st != P2P_OK) return st;
  if ((st = gemm_check(ctx, n, k, x, ld_x, m_tokens, y, ld_y, y_off, "gemm_f16w")) != P2P_OK)
    return st;
  if (m_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  return gemm_run(ctx, w16, n, k, x, ld_x, m_tokens, y, ld_y, y_off, pick_stream(ctx, stream),
                  "gemm_f16w launch");
}

p2p_status p2p_qkv_gemm_prep_f16w(p2p_ctx* ctx, const p2p_attn_params* prm, const void* x,
                                  int64_t ld_x, const void* w16_qkv, int32_t k,
                                  const void* norm_w, const void* rope, void* q_out,
                                  int64_t ld_q, void* k_cache, void* v_cache,
                                  int64_t kv_cap_tokens, const uint32_t* meta_dev, int32_t pos0,
                                  int32_t m_tokens, void* stream) {
  const QkvPrepIo io{x,       ld_x,    norm_w,        rope,     q_out, ld_q,
                     k_cache, v_cache, kv_cap_tokens, meta_dev, pos0,  m_tokens};
  p2p_status st = qkv_check(ctx, prm, k, io, "qkv_gemm_prep_f16w");
  if (st != P2P_OK) return st;
  const int n = (prm->num_heads + 2 * prm->num_kv_heads) * prm->head_dim;
  if ((st = check_w16(ctx, w16_qkv, n, k, "qkv_gemm_prep_f16w")) != P2P_OK) return st;
  if (m_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  return qkv_run(ctx, prm, w16_qkv, k, io, pick_stream(ctx, stream), "qkv_gemm_prep_f16w launch");
}

p2p_status p2p_kv_quantize_q8(p2p_ctx* ctx, const void* src, void* dst, int64_t rows,
                              int32_t num_kv_heads, const float* scale, int32_t scale_count,
                              void* stream) {
  if (!ctx) return P2P_ERR_INVALID_ARG;
  if (!src || !dst || !scale || rows < 0 || num_kv_heads <= 0 ||
      (scale_count != 1 && scale_count != num_kv_heads * 64))
    return fail(ctx, P2P_ERR_INVALID_ARG, "kv_quantize_q8: rows %lld kv heads %d scales %d",
                (long long)rows, num_kv_heads, scale_count);
  if (!aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7u))
    return fail(ctx, P2P_ERR_INVALID_ARG, "kv_quantize_q8: src must be 16-byte, dst 8-byte aligned");
  if (rows == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  cudaError_t e = p2p::launch_quantize_q8(src, dst, rows, num_kv_heads, scale, scale_count,
                                          pick_stream(ctx, stream));
  if (e != cudaSuccess) return cuda_fail(ctx, e, "kv_quantize_q8 launch");
  return P2P_OK;
}

p2p_status p2p_attn_bidir(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q,
                          const void* k, const void* v, void* out, int64_t ld, int32_t batch,
                          int32_t s_tokens, void* stream) {
  p2p_status st = check_params(ctx, prm, false);
  if (st != P2P_OK) return st;
  if (!q || !k || !v || !out) return fail(ctx, P2P_ERR_INVALID_ARG, "attn_bidir: NULL buffer");
  const int64_t w = int64_t(prm->num_heads) * prm->head_dim;
  const int64_t kw = int64_t(prm->num_kv_heads) * prm->head_dim;
  if (batch < 0 || s_tokens < 0 || ld < (w > kw ? w : kw) || (ld % 8))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn_bidir: batch %d S %d ld %lld", batch, s_tokens,
                (long long)ld);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(ctx, P2P_ERR_INVALID_ARG, "attn_bidir: buffers must be 16-byte aligned");
  if (batch == 0 || s_tokens == 0) return P2P_OK;
  DeviceGuard g(ctx->device);
  p2p::FlashArgs f{};
  f.q = q;
  f.k = k;
  f.v = v;
  f.out = out;
  f.ld_q = f.ld_kv = f.ld_o = ld;
  f.q_rows_total = f.kv_rows_total = int64_t(batch) * s_tokens;
  f.batch_stride_q_rows = f.batch_stride_kv_rows = s_tokens;
  f.batch = batch;
  f.s_q = s_tokens;
  f.s_kv = s_tokens;
  f.hq = prm->num_heads;
  f.hkv = prm->num_kv_heads;
  f.causal = 0;
  f.meta = nullptr;
  f.pos0_host = 0;
  f.scale_log2 = eff_scale(prm) * 1.4426950408889634f;
  f.err = ctx->dev_err;
  f.wait_deficit = g_wait_deficit.load();
  f.num_sms = ctx->num_sms;
  cudaError_t e = p2p::launch_flash(f, pick_stream(ctx, stream));
  if (e == cudaErrorNotSupported) return fail(ctx, P2P_ERR_UNSUPPORTED, "bidir kernel");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "bidir launch");
  return P2P_OK;
}

}  // extern "C"

namespace p2p {
int ctx_device(const p2p_ctx* ctx) { return ctx->device; }
int ctx_num_sms(const p2p_ctx* ctx) { return ctx->num_sms; }
p2p_status ctx_fail(p2p_ctx* ctx, p2p_status s, const char* msg) { return fail(ctx, s, "%s", msg); }
p2p_status ctx_check_params(p2p_ctx* ctx, const p2p_attn_params* prm) {
  return check_params(ctx, prm, true);
}
float eff_scale_log2(const p2p_attn_params* prm) {
  return eff_scale(prm) * 1.4426950408889634f;
}
float eff_eps_of(const p2p_attn_params* prm) { return eff_eps(prm); }
int forced_decode_splits() { return forced_splits(); }
cudaError_t lib_alloc(void** p, size_t bytes) { return dev_alloc(p, bytes); }
void lib_free(void* p, size_t bytes) { dev_free(p, bytes); }
int32_t* ctx_dev_err(const p2p_ctx* ctx) { return ctx->dev_err; }
int32_t debug_wait_deficit() { return g_wait_deficit.load(); }

p2p_status check_ragged(p2p_ctx* ctx, const p2p_attn_params* prm, const void* qkv,
                        int64_t ld_qkv, const void* rope, const void* k_cache,
                        const void* v_cache, int64_t kv_rows, const int32_t* offsets,
                        const int32_t* past, int32_t nseq, int32_t max_past, int32_t fused_prep,
                        const void* out, int64_t ld_o, const char* who) {
  p2p_status st = check_params(ctx, prm, true);
  if (st != P2P_OK) return st;
  const int64_t qw = int64_t(prm->num_heads) * prm->head_dim;
  const int64_t row = qw + 2 * int64_t(prm->num_kv_heads) * prm->head_dim;
  if (!qkv || !k_cache || !v_cache || !offsets || !past || !out || (fused_prep && !rope))
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: NULL buffer", who);
  if (nseq < 0 || nseq > 65535 || max_past < 0 || kv_rows <= 0 || ld_o < qw ||
      ld_qkv < (fused_prep ? row : qw))
    return fail(ctx, P2P_ERR_INVALID_ARG,
                "%s: nseq %d max_past %d kv_rows %lld ld_qkv %lld ld_o %lld", who, nseq,
                max_past, (long long)kv_rows, (long long)ld_qkv, (long long)ld_o);
  if (!aligned16(k_cache) || !aligned16(v_cache))
    return fail(ctx, P2P_ERR_INVALID_ARG, "%s: cache buffers must be 16-byte aligned", who);
  if (fused_prep) {
    // a rope table this context built knows its rows: it must cover positions 0..max_past
    for (const auto& kv : ctx->rope)
      if (kv.second == rope && std::get<0>(kv.first) <= max_past)
        return fail(ctx, P2P_ERR_INVALID_ARG, "%s: rope table of %d rows, max_past %d", who,
                    std::get<0>(kv.first), max_past);
  }
  return P2P_OK;
}

void fill_ragged(DecodeArgs& a, const void* qkv, int64_t ld_qkv, const void* norm_w,
                 const void* rope, void* k_cache, void* v_cache, int64_t kv_rows,
                 const int32_t* offsets, const int32_t* past, int32_t max_past, void* out,
                 int64_t ld_o) {
  a.qkv = qkv;
  a.ld_qkv = ld_qkv;
  a.norm_w = norm_w;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.kv_cap = kv_rows;
  a.offsets = offsets;
  a.past = past;
  a.max_past = max_past;
  a.out = out;
  a.ld_o = ld_o;
  a.rope = rope;
}
}  // namespace p2p
