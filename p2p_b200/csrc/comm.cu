// comm.cu -- the library's own NCCL communicator and the head-sharded prefill that uses it.
//
// Long-context prefill splits by KV-head group over the GPUs of one node (one process per
// GPU): rank g owns kv heads [g*Hkv/G, (g+1)*Hkv/G) and their q heads, runs QK_PREP
// (kernels.js:216-266) and ATTN (kernels.js:268-319) on them, and the per-rank [M][Hq/G*D]
// slices are exchanged with one ncclAllGather over NVLink, then reassembled into the
// reference's [M][Hq*D] layout on every rank.  A host that calls the library through its C ABI
// (the engine's ATTN dispatch, engine.js:222) thus needs no collective library of its own.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, reusing a copy the process already
// loaded), so the library itself loads without it.  The communicator is non-blocking: every
// NCCL call is followed by a bounded host-side wait on ncclCommGetAsyncError, and
// p2p_comm_wait bounds the wait for a collective in flight on the GPU.  A wait that runs out
// aborts the communicator (ncclCommAbort ends NCCL's kernels) and returns P2P_ERR_TIMEOUT;
// an NCCL error returns P2P_ERR_NCCL.  An aborted communicator refuses further work.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>

#pragma GCC visibility push(default)
#include "../../include/p2p_attn.h"
#pragma GCC visibility pop
#include "host_internal.h"
#include "kernels.h"

static_assert(sizeof(ncclUniqueId) == P2P_COMM_ID_BYTES, "NCCL unique id size");

namespace {

// The NCCL entry points this file uses, resolved from the loaded library.
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) =
      nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GetVersion)(int*) = nullptr;
  bool ok = false;
  char why[256] = {0};
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = nullptr;
    if (const char* p = std::getenv("P2P_NCCL_LIB")) h = dlopen(p, RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's own copy
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      std::snprintf(api.why, sizeof api.why, "libnccl.so.2 could not be loaded: %s", dlerror());
      return;
    }
    bool all = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      if (!fn) {
        all = false;
        std::snprintf(api.why, sizeof api.why, "libnccl.so.2 lacks %s", name);
      }
    };
    get(api.GetUniqueId, "ncclGetUniqueId");
    get(api.CommInitRankConfig, "ncclCommInitRankConfig");
    get(api.CommGetAsyncError, "ncclCommGetAsyncError");
    get(api.CommAbort, "ncclCommAbort");
    get(api.CommFinalize, "ncclCommFinalize");
    get(api.CommDestroy, "ncclCommDestroy");
    get(api.AllGather, "ncclAllGather");
    get(api.AllReduce, "ncclAllReduce");
    get(api.GetErrorString, "ncclGetErrorString");
    get(api.GetVersion, "ncclGetVersion");
    api.ok = all;
  });
  return api;
}

using Clock = std::chrono::steady_clock;

// 16-byte pieces: out[m][g*W + c] = gather[g][m][c] for the G rank slices of width W halves.
__global__ void assemble_kernel(const uint4* __restrict__ gather, uint4* __restrict__ out,
                                int64_t m_tokens, int ranks, int w16, int64_t ld_o16) {
  const int64_t n = m_tokens * ranks * w16;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int c = int(i % w16);
    const int64_t t = i / w16;
    const int g = int(t % ranks);
    const int64_t m = t / ranks;
    out[m * ld_o16 + int64_t(g) * w16 + c] = gather[(int64_t(g) * m_tokens + m) * w16 + c];
  }
}

}  // namespace

struct p2p_comm {
  p2p_ctx* ctx = nullptr;
  int nranks = 0, rank = 0;
  int timeout_ms = 0;
  ncclComm_t comm = nullptr;
  bool aborted = false;
  // workspace of the sharded prefill, grown on demand: rotated q rows of this rank's heads and
  // the all-gather buffer [nranks][M][local width]; plus one float for p2p_comm_barrier
  void* q_buf = nullptr;
  size_t q_bytes = 0;
  void* gather = nullptr;
  size_t gather_bytes = 0;
  float* flag = nullptr;
};

namespace {

p2p_status comm_fail(p2p_comm* c, p2p_status s, const char* fmt, const char* detail) {
  char msg[400];
  std::snprintf(msg, sizeof msg, fmt, detail);
  return p2p::ctx_fail(c->ctx, s, msg);
}

// Abort after a failed or expired wait: NCCL's kernels in flight end, and the communicator is
// unusable from then on.
void abort_comm(p2p_comm* c) {
  if (c->comm && !c->aborted) nccl().CommAbort(c->comm);
  c->aborted = true;
  c->comm = nullptr;
}

// Bounded wait until the communicator's last non-blocking call has completed on the host.
p2p_status settle(p2p_comm* c, ncclResult_t r, const char* what) {
  const NcclApi& api = nccl();
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  while (r == ncclInProgress) {
    if (Clock::now() > deadline) {
      abort_comm(c);
      return comm_fail(c, P2P_ERR_TIMEOUT, "%s: no answer from the other ranks in time; the "
                                           "communicator was aborted", what);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    if (api.CommGetAsyncError(c->comm, &r) != ncclSuccess) r = ncclInternalError;
  }
  if (r != ncclSuccess) {
    const char* es = api.GetErrorString(r);
    abort_comm(c);
    char msg[300];
    std::snprintf(msg, sizeof msg, "%s: %s", what, es);
    return p2p::ctx_fail(c->ctx, P2P_ERR_NCCL, msg);
  }
  return P2P_OK;
}

p2p_status usable(p2p_comm* c) {
  if (!c || !c->ctx) return P2P_ERR_INVALID_ARG;
  if (c->aborted || !c->comm)
    return p2p::ctx_fail(c->ctx, P2P_ERR_NCCL, "communicator was aborted after an earlier "
                                               "failure; create a new one");
  return P2P_OK;
}

p2p_status grow(p2p_comm* c, void** p, size_t* have, size_t need, const char* what) {
  if (need <= *have) return P2P_OK;
  cudaDeviceSynchronize();  // rare growth: no launch may still use the old buffer
  p2p::lib_free(*p, *have);
  *p = nullptr;
  *have = 0;
  if (p2p::lib_alloc(p, need) != cudaSuccess)
    return comm_fail(c, P2P_ERR_OOM, "sharded prefill: %s workspace", what);
  *have = need;
  return P2P_OK;
}

}  // namespace

extern "C" {

p2p_status p2p_comm_unique_id(unsigned char id[P2P_COMM_ID_BYTES]) {
  if (!id) return P2P_ERR_INVALID_ARG;
  const NcclApi& api = nccl();
  if (!api.ok) return P2P_ERR_NCCL;
  ncclUniqueId u;
  if (api.GetUniqueId(&u) != ncclSuccess) return P2P_ERR_NCCL;
  std::memcpy(id, &u, sizeof u);
  return P2P_OK;
}

p2p_status p2p_comm_create(p2p_ctx* ctx, int32_t nranks, int32_t rank,
                           const unsigned char id[P2P_COMM_ID_BYTES], int32_t timeout_ms,
                           p2p_comm** out) {
  if (!ctx || !out || !id) return P2P_ERR_INVALID_ARG;
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks || timeout_ms <= 0)
    return p2p::ctx_fail(ctx, P2P_ERR_INVALID_ARG, "comm_create: bad nranks/rank/timeout");
  const NcclApi& api = nccl();
  if (!api.ok) return p2p::ctx_fail(ctx, P2P_ERR_NCCL, api.why);
  p2p_comm* c = new (std::nothrow) p2p_comm;
  if (!c) return P2P_ERR_OOM;
  c->ctx = ctx;
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_ms = timeout_ms;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != p2p::ctx_device(ctx) && cudaSetDevice(p2p::ctx_device(ctx)) != cudaSuccess) {
    delete c;
    return p2p::ctx_fail(ctx, P2P_ERR_CUDA, "comm_create: cannot select the context's device");
  }
  void* f = nullptr;
  if (p2p::lib_alloc(&f, sizeof(float)) != cudaSuccess) {
    if (prev >= 0) cudaSetDevice(prev);
    delete c;
    return p2p::ctx_fail(ctx, P2P_ERR_OOM, "comm_create: flag word");
  }
  c->flag = static_cast<float*>(f);
  cudaMemset(c->flag, 0, sizeof(float));
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof u);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // every call returns at once; settle() bounds the wait
  ncclResult_t r = api.CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
  p2p_status st;
  if (r != ncclSuccess && r != ncclInProgress) {
    c->comm = nullptr;
    st = p2p::ctx_fail(ctx, P2P_ERR_NCCL, api.GetErrorString(r));
  } else {
    st = settle(c, r, "comm_create (ncclCommInitRankConfig)");
  }
  if (prev >= 0 && prev != p2p::ctx_device(ctx)) cudaSetDevice(prev);
  if (st != P2P_OK) {
    p2p::lib_free(c->flag, sizeof(float));
    delete c;
    return st;
  }
  *out = c;
  return P2P_OK;
}

p2p_status p2p_comm_destroy(p2p_comm* c) {
  if (!c) return P2P_ERR_INVALID_ARG;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(p2p::ctx_device(c->ctx));
  p2p_status st = P2P_OK;
  if (c->comm && !c->aborted) {
    // finalize flushes the communicator's outstanding work (bounded); then release it
    ncclResult_t r = nccl().CommFinalize(c->comm);
    st = settle(c, r, "comm_destroy (ncclCommFinalize)");
    if (c->comm) nccl().CommDestroy(c->comm);
  }
  cudaDeviceSynchronize();
  p2p::lib_free(c->q_buf, c->q_bytes);
  p2p::lib_free(c->gather, c->gather_bytes);
  p2p::lib_free(c->flag, sizeof(float));
  if (prev >= 0) cudaSetDevice(prev);
  delete c;
  return st;
}

p2p_status p2p_comm_wait(p2p_comm* c, void* stream) {
  p2p_status st = usable(c);
  if (st != P2P_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
  for (;;) {
    cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return p2p::ctx_fail(c->ctx, P2P_ERR_CUDA, cudaGetErrorString(q));
    ncclResult_t r = ncclSuccess;
    nccl().CommGetAsyncError(c->comm, &r);
    if (r != ncclSuccess && r != ncclInProgress) {
      const char* es = nccl().GetErrorString(r);
      abort_comm(c);
      return comm_fail(c, P2P_ERR_NCCL, "comm_wait: %s", es);
    }
    if (Clock::now() > deadline) {
      // a peer never joined the collective: abort ends NCCL's kernels, so the stream drains
      abort_comm(c);
      const auto drain = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
      while (cudaStreamQuery(s) == cudaErrorNotReady && Clock::now() < drain)
        std::this_thread::sleep_for(std::chrono::microseconds(100));
      return p2p::ctx_fail(c->ctx, P2P_ERR_TIMEOUT,
                           "comm_wait: a collective did not complete in time (a peer left or "
                           "stalled); the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  return p2p_sync(c->ctx, stream);
}

p2p_status p2p_comm_barrier(p2p_comm* c, void* stream) {
  p2p_status st = usable(c);
  if (st != P2P_OK) return st;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(p2p::ctx_device(c->ctx));
  ncclResult_t r = nccl().AllReduce(c->flag, c->flag, 1, ncclFloat32, ncclSum, c->comm,
                                    static_cast<cudaStream_t>(stream));
  st = settle(c, r, "comm_barrier (ncclAllReduce)");
  if (prev >= 0) cudaSetDevice(prev);
  return st;
}

p2p_status p2p_attn_prefill_sharded(p2p_ctx* ctx, p2p_comm* c, const p2p_attn_params* prm,
                                    const void* qkv, int64_t ld_qkv, const void* norm_w,
                                    const void* rope, void* k_cache, void* v_cache,
                                    int64_t kv_cap_tokens, const uint32_t* meta_dev,
                                    int32_t pos0, int32_t m_tokens, void* out, int64_t ld_o,
                                    void* stream) {
  if (!ctx || !c || c->ctx != ctx) return P2P_ERR_INVALID_ARG;
  p2p_status st = p2p::ctx_check_params(ctx, prm);
  if (st != P2P_OK) return st;
  st = usable(c);
  if (st != P2P_OK) return st;
  if (prm->dtype != P2P_F16)
    return p2p::ctx_fail(ctx, P2P_ERR_UNSUPPORTED, "prefill_sharded: f16 only");
  const int G = c->nranks;
  if (prm->num_kv_heads % G)
    return p2p::ctx_fail(ctx, P2P_ERR_INVALID_ARG,
                         "prefill_sharded: the ranks must divide the kv heads");
  const int kvn = prm->num_kv_heads / G;
  const int qn = kvn * (prm->num_heads / prm->num_kv_heads);
  const int D = prm->head_dim;
  const int64_t wl = int64_t(qn) * D;                  // this rank's output width
  const int64_t row = int64_t(qn + 2 * kvn) * D;       // its qkv columns
  if (!qkv || !rope || !k_cache || !v_cache || !out)
    return p2p::ctx_fail(ctx, P2P_ERR_INVALID_ARG, "prefill_sharded: NULL buffer");
  if (m_tokens < 0 || m_tokens > 65535 || ld_qkv < row || kv_cap_tokens <= 0 ||
      ld_o < int64_t(prm->num_heads) * D || (ld_o % 8) || (!meta_dev && pos0 < 0) ||
      (reinterpret_cast<uintptr_t>(out) & 15u) ||
      ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u))
    return p2p::ctx_fail(ctx, P2P_ERR_INVALID_ARG,
                         "prefill_sharded: sizes, strides or alignment");
  if (!meta_dev && int64_t(pos0) + m_tokens > kv_cap_tokens)
    return p2p::ctx_fail(ctx, P2P_ERR_KV_FULL, "prefill_sharded: pos0 + M beyond the cache");
  if (m_tokens == 0) return P2P_OK;

  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(p2p::ctx_device(ctx));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t slice = size_t(m_tokens) * size_t(wl) * sizeof(__half);
  st = grow(c, &c->q_buf, &c->q_bytes, slice, "q rows");
  if (st == P2P_OK) st = grow(c, &c->gather, &c->gather_bytes, slice * G, "all-gather");
  cudaError_t e = cudaSuccess;
  if (st == P2P_OK) {  // QK_PREP on this rank's heads (its kv-cache slice is written here)
    p2p::QkPrepArgs a{qkv, ld_qkv, norm_w, rope, c->q_buf, wl, k_cache, v_cache,
                      kv_cap_tokens, meta_dev, pos0, m_tokens, qn, kvn,
                      p2p::eff_eps_of(prm), p2p::ctx_dev_err(ctx)};
    e = p2p::launch_qk_prep(a, P2P_F16, s);
  }
  unsigned char* mine = static_cast<unsigned char*>(c->gather) + slice * c->rank;
  if (st == P2P_OK && e == cudaSuccess) {  // ATTN on them, straight into this rank's slot
    p2p::FlashArgs f{};
    f.q = c->q_buf;
    f.k = k_cache;
    f.v = v_cache;
    f.out = mine;
    f.ld_q = wl;
    f.ld_kv = int64_t(kvn) * D;
    f.ld_o = wl;
    f.q_rows_total = m_tokens;
    f.kv_rows_total = kv_cap_tokens;
    f.batch = 1;
    f.s_q = m_tokens;
    f.hq = qn;
    f.hkv = kvn;
    f.causal = 1;
    f.meta = meta_dev;
    f.pos0_host = pos0;
    f.scale_log2 = p2p::eff_scale_log2(prm);
    f.err = p2p::ctx_dev_err(ctx);
    f.wait_deficit = p2p::debug_wait_deficit();
    f.num_sms = p2p::ctx_num_sms(ctx);
    e = p2p::launch_flash(f, s);
  }
  if (st == P2P_OK && e == cudaSuccess && G > 1) {  // one all-gather of the slices, in place
    ncclResult_t r = nccl().AllGather(mine, c->gather, slice / sizeof(__half), ncclFloat16,
                                      c->comm, s);
    st = settle(c, r, "prefill_sharded (ncclAllGather)");
  }
  if (st == P2P_OK && e == cudaSuccess) {  // [G][M][W] -> [M][G*W]
    const int w16 = int(wl * sizeof(__half) / 16);
    const int64_t n = int64_t(m_tokens) * G * w16;
    const int blocks = int((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    assemble_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint4*>(c->gather),
                                           static_cast<uint4*>(out), m_tokens, G, w16,
                                           ld_o * int64_t(sizeof(__half)) / 16);
    e = cudaGetLastError();
  }
  if (prev >= 0) cudaSetDevice(prev);
  if (st != P2P_OK) return st;
  if (e != cudaSuccess) return p2p::ctx_fail(ctx, P2P_ERR_CUDA, cudaGetErrorString(e));
  return P2P_OK;
}

}  // extern "C"
