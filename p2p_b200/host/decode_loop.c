/*
 * decode_loop.c -- a plain C host that drives the decode step through the C ABI alone, the
 * way a native engine binding (the N-API addon a JavaScript host would load) calls it: no
 * Python, no torch.  One attention step of the LFM2.5-1.2B decoder per token
 * (engine.js:411-437: writeBuffer of the new token's qkv rows, QK_PREP + ATTN for the six
 * attention layers, readback), with the six qkv rows and six output rows in page-locked host
 * memory that the kernel reads and writes across the host link itself, then one stream
 * synchronization per token.
 *
 *   p2p_decode_loop [--device N] [--steps K] [--warmup W] [--copies C] [--past P]
 *                   [--sched auto|spin|yield|block] [--graph 0|1] [--rows host|device]
 *
 * --sched sets how the host thread waits for the GPU (cudaSetDeviceFlags before the context
 * exists: spin keeps the core polling, the lowest latency for a serving thread that owns a
 * core); --graph 1 records each copy's step once as a CUDA graph and replays it per token
 * instead of launching through the C ABI each time (what a binding does once the shapes are
 * fixed; the kernel still reads and writes the host rows on every replay); --rows device keeps
 * the rows in device memory and moves them with one copy in (36 KB) and one copy out (24 KB)
 * per token on the same stream instead of the kernel crossing the host link itself.
 *
 * Prints one JSON line: microseconds per step (wall clock around K steps), the host bytes in
 * and out per step, and whether every output was finite.  The KV caches (C copies of the six
 * layers, rotated so consecutive steps do not hit in L2) are filled with seeded N(0,1)-shaped
 * values.
 */
#define _POSIX_C_SOURCE 199309L
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "p2p_attn.h"

#define HQ 32
#define HKV 8
#define D 64
#define LAYERS 6

static uint64_t rng_state = 0x9e3779b97f4a7c15ull;
static uint64_t splitmix(void) {
  uint64_t z = (rng_state += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
/* IEEE binary16 bits of a float, round to nearest even (values here stay in the normal range;
 * anything below 2^-14 in magnitude becomes a signed zero) */
static uint16_t float_to_half(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  const uint32_t sign = (b >> 16) & 0x8000u;
  const int32_t e = (int32_t)((b >> 23) & 0xff) - 127 + 15;
  const uint32_t m = b & 0x7fffffu;
  if (e <= 0) return (uint16_t)sign;
  if (e >= 31) return (uint16_t)(sign | 0x7bffu);
  uint32_t h = sign | ((uint32_t)e << 10) | (m >> 13);
  const uint32_t rest = m & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h += 1;
  return (uint16_t)h;
}
/* one N(0,1) sample (Box-Muller in double) */
static float normal(void) {
  const double u1 = ((splitmix() >> 11) + 1.0) / 9007199254740993.0;
  const double u2 = (splitmix() >> 11) / 9007199254740992.0;
  return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}
static uint16_t normal_half(void) { return float_to_half(normal()); }
static int finite_half(uint16_t h) { return (h & 0x7c00u) != 0x7c00u; }

static double now_s(void) {
  struct timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return t.tv_sec + 1e-9 * t.tv_nsec;
}

#define CHECK_P2P(call)                                                              \
  do {                                                                               \
    p2p_status st_ = (call);                                                         \
    if (st_ != P2P_OK) {                                                             \
      fprintf(stderr, "%s failed: %s (%s)\n", #call, p2p_status_string(st_),         \
              ctx ? p2p_last_error(ctx) : "");                                       \
      return 1;                                                                      \
    }                                                                                \
  } while (0)
#define CHECK_CUDA(call)                                                             \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    if (e_ != cudaSuccess) {                                                         \
      fprintf(stderr, "%s failed: %s\n", #call, cudaGetErrorString(e_));             \
      return 1;                                                                      \
    }                                                                                \
  } while (0)

int main(int argc, char** argv) {
  int device = 0, steps = 200, warmup = 20, copies = 12, past = 4096, use_graph = 0;
  const char* sched = "auto";
  const char* rows = "host";
  for (int i = 1; i + 1 < argc; i += 2) {
    if (!strcmp(argv[i], "--device")) device = atoi(argv[i + 1]);
    else if (!strcmp(argv[i], "--steps")) steps = atoi(argv[i + 1]);
    else if (!strcmp(argv[i], "--warmup")) warmup = atoi(argv[i + 1]);
    else if (!strcmp(argv[i], "--copies")) copies = atoi(argv[i + 1]);
    else if (!strcmp(argv[i], "--past")) past = atoi(argv[i + 1]);
    else if (!strcmp(argv[i], "--sched")) sched = argv[i + 1];
    else if (!strcmp(argv[i], "--graph")) use_graph = atoi(argv[i + 1]);
    else if (!strcmp(argv[i], "--rows")) rows = argv[i + 1];
  }
  unsigned flags = cudaDeviceScheduleAuto;
  if (!strcmp(sched, "spin")) flags = cudaDeviceScheduleSpin;
  else if (!strcmp(sched, "yield")) flags = cudaDeviceScheduleYield;
  else if (!strcmp(sched, "block")) flags = cudaDeviceScheduleBlockingSync;
  else if (strcmp(sched, "auto")) {
    fprintf(stderr, "bad --sched\n");
    return 2;
  }
  CHECK_CUDA(cudaSetDevice(device));
  CHECK_CUDA(cudaSetDeviceFlags(flags));
  if (steps < 1 || warmup < 0 || copies < 1 || past < 0) {
    fprintf(stderr, "bad arguments\n");
    return 2;
  }
  p2p_ctx* ctx = NULL;
  CHECK_P2P(p2p_ctx_create(device, &ctx));
  CHECK_CUDA(cudaSetDevice(device));
  const int64_t cap = past + 1;
  const p2p_attn_params prm = {HQ, HKV, D, 0.0f, 0.0f, P2P_F16};
  const void* rope = NULL;
  CHECK_P2P(p2p_rope_table(ctx, (int32_t)cap, D, 1e6, P2P_F16, &rope));
  uint32_t* meta = NULL;
  CHECK_P2P(p2p_meta(ctx, &meta));
  void* stream = p2p_ctx_stream(ctx);

  /* caches: `copies` sets of six layers, one seeded host buffer per layer uploaded to all */
  p2p_kv** kv = (p2p_kv**)calloc((size_t)copies, sizeof(p2p_kv*));
  const size_t row_elems = (size_t)HKV * D;
  const size_t buf_elems = (size_t)cap * row_elems;
  uint16_t* host = (uint16_t*)malloc(buf_elems * 2);
  for (int c = 0; c < copies; ++c) CHECK_P2P(p2p_kv_create(ctx, LAYERS, HKV, D, cap, P2P_F16, &kv[c]));
  for (int l = 0; l < LAYERS; ++l) {
    for (int t = 0; t < 2; ++t) {
      for (size_t i = 0; i < buf_elems; ++i) host[i] = normal_half();
      for (int c = 0; c < copies; ++c) {
        void* dst = t == 0 ? p2p_kv_k(kv[c], l) : p2p_kv_v(kv[c], l);
        CHECK_CUDA(cudaMemcpy(dst, host, buf_elems * 2, cudaMemcpyHostToDevice));
      }
    }
  }
  free(host);
  /* norm weights 1 + 0.1 N(0,1) in device memory; qkv / out rows in page-locked host memory */
  const size_t qkv_w = (size_t)(HQ + 2 * HKV) * D, out_w = (size_t)HQ * D;
  uint16_t nw_h[LAYERS][2 * D];
  for (int l = 0; l < LAYERS; ++l)
    for (int i = 0; i < 2 * D; ++i) nw_h[l][i] = float_to_half(1.0f + 0.1f * normal());
  void* nw_d = NULL;
  CHECK_CUDA(cudaMalloc(&nw_d, sizeof nw_h));
  CHECK_CUDA(cudaMemcpy(nw_d, nw_h, sizeof nw_h, cudaMemcpyHostToDevice));
  uint16_t* qkv_h = NULL;
  uint16_t* out_h = NULL;
  CHECK_CUDA(cudaHostAlloc((void**)&qkv_h, LAYERS * qkv_w * 2, cudaHostAllocDefault));
  CHECK_CUDA(cudaHostAlloc((void**)&out_h, LAYERS * out_w * 2, cudaHostAllocDefault));
  for (size_t i = 0; i < LAYERS * qkv_w; ++i) qkv_h[i] = normal_half();
  const int dev_rows = !strcmp(rows, "device");
  if (!dev_rows && strcmp(rows, "host")) {
    fprintf(stderr, "bad --rows\n");
    return 2;
  }
  uint16_t *qkv_d = NULL, *out_d = NULL;
  if (dev_rows) {
    CHECK_CUDA(cudaMalloc((void**)&qkv_d, LAYERS * qkv_w * 2));
    CHECK_CUDA(cudaMalloc((void**)&out_d, LAYERS * out_w * 2));
  }
  uint16_t* qkv_k = dev_rows ? qkv_d : qkv_h; /* the rows the kernel reads and writes */
  uint16_t* out_k = dev_rows ? out_d : out_h;

  p2p_decode_layer* layers = (p2p_decode_layer*)malloc(sizeof(p2p_decode_layer) * copies * LAYERS);
  for (int c = 0; c < copies; ++c)
    for (int l = 0; l < LAYERS; ++l) {
      p2p_decode_layer* L = &layers[c * LAYERS + l];
      L->qkv = qkv_k + l * qkv_w;
      L->norm_w = (const uint16_t*)nw_d + l * 2 * D;
      L->k_cache = p2p_kv_k(kv[c], l);
      L->v_cache = p2p_kv_v(kv[c], l);
      L->out = out_k + l * out_w;
    }
  CHECK_P2P(p2p_meta_write(ctx, (uint32_t)past, 1, 0, stream));
  CHECK_P2P(p2p_sync(ctx, stream));

#define STEP(c)                                                                            \
  do {                                                                                     \
    if (dev_rows)                                                                          \
      CHECK_CUDA(cudaMemcpyAsync(qkv_d, qkv_h, LAYERS * qkv_w * 2, cudaMemcpyHostToDevice, \
                                 (cudaStream_t)stream));                                   \
    CHECK_P2P(p2p_decode_step(ctx, &prm, LAYERS, &layers[(c) * LAYERS], rope, cap, meta, 0, \
                              stream));                                                    \
    if (dev_rows)                                                                          \
      CHECK_CUDA(cudaMemcpyAsync(out_h, out_d, LAYERS * out_w * 2, cudaMemcpyDeviceToHost, \
                                 (cudaStream_t)stream));                                   \
  } while (0)
  /* warm-up of the plain call (workspace, kernel attributes) before any capture */
  STEP(0);
  CHECK_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  cudaGraphExec_t* execs = NULL;
  if (use_graph) {
    execs = (cudaGraphExec_t*)calloc((size_t)copies, sizeof(cudaGraphExec_t));
    for (int c = 0; c < copies; ++c) {
      cudaGraph_t g;
      CHECK_CUDA(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal));
      STEP(c);
      CHECK_CUDA(cudaStreamEndCapture((cudaStream_t)stream, &g));
      CHECK_CUDA(cudaGraphInstantiate(&execs[c], g, 0));
      CHECK_CUDA(cudaGraphDestroy(g));
    }
  }

  double t0 = 0.0;
  for (int i = 0; i < warmup + steps; ++i) {
    if (i == warmup) t0 = now_s();
    /* the per-token call: the kernel reads qkv rows from and writes out rows to host memory */
    if (use_graph)
      CHECK_CUDA(cudaGraphLaunch(execs[i % copies], (cudaStream_t)stream));
    else
      STEP(i % copies);
    CHECK_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  }
  const double dt = (now_s() - t0) / steps;
  CHECK_P2P(p2p_sync(ctx, stream));
  int finite = 1;
  for (size_t i = 0; i < LAYERS * out_w; ++i) finite &= finite_half(out_h[i]);

  if (execs) {
    for (int c = 0; c < copies; ++c) cudaGraphExecDestroy(execs[c]);
    free(execs);
  }
  if (dev_rows) {
    cudaFree(qkv_d);
    cudaFree(out_d);
  }
  printf("{\"sched\": \"%s\", \"graph\": %d, \"rows\": \"%s\", ", sched, use_graph, rows);
  printf("\"us_per_step\": %.3f, \"h2d_bytes_per_step\": %zu, \"d2h_bytes_per_step\": %zu, "
         "\"steps\": %d, \"warmup\": %d, \"copies\": %d, \"past\": %d, \"outputs_finite\": %s}\n",
         dt * 1e6, (size_t)LAYERS * qkv_w * 2, (size_t)LAYERS * out_w * 2, steps, warmup,
         copies, past, finite ? "true" : "false");
  cudaFreeHost(qkv_h);
  cudaFreeHost(out_h);
  cudaFree(nw_d);
  for (int c = 0; c < copies; ++c) p2p_kv_destroy(kv[c]);
  free(kv);
  free(layers);
  p2p_ctx_destroy(ctx);
  return finite ? 0 : 3;
}
