// kernels.h -- host-side launchers of the sm_100a kernels (internal to libp2pattn.so).
#pragma once

#include <mutex>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace p2p {

// Kernel attributes (dynamic shared-memory size, carveout) belong to each device's context: a
// launcher sets them once per device, with that device current.  `setup(value)` runs on the
// first call for the current device; its status (and an int it may record, such as a count of
// resident clusters) is returned on every later call for that device.
constexpr int kMaxDevicesPerProcess = 64;
struct PerDeviceOnce {
  std::mutex mu;
  bool done[kMaxDevicesPerProcess] = {};
  cudaError_t err[kMaxDevicesPerProcess] = {};
  int value[kMaxDevicesPerProcess] = {};
};
template <class F>
cudaError_t per_device_once(PerDeviceOnce& st, F&& setup, int* value = nullptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevicesPerProcess) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(st.mu);
  if (!st.done[dev]) {
    st.err[dev] = setup(st.value[dev]);
    st.done[dev] = true;
  }
  if (value) *value = st.value[dev];
  return st.err[dev];
}

// ---- qk_prep.cu -----------------------------------------------------------------------------
struct QkPrepArgs {
  const void* qkv;
  int64_t ld_qkv;
  const void* norm_w;  // nullable
  const void* rope;
  void* q_out;
  int64_t ld_q;
  void* k_cache;
  void* v_cache;
  int64_t kv_cap;        // rows the cache buffers hold; rows >= kv_cap are never touched
  const uint32_t* meta;  // nullable -> pos0
  int32_t pos0;
  int32_t m_tokens;
  int32_t hq, hkv;
  float eps;
  int32_t* err;          // device error word: bit 0 = position beyond the cache
};
cudaError_t launch_qk_prep(const QkPrepArgs& a, int dtype, cudaStream_t s);
cudaError_t launch_argmax_step(const void* logits, int32_t vocab, uint32_t* tok,
                               uint32_t* out_tok, int64_t out_cap, uint32_t* meta, int32_t* err,
                               cudaStream_t s);

// ---- decode.cu ------------------------------------------------------------------------------
constexpr int kMaxLayers = 16;

struct DecodeLayer {
  const void* qkv;  // fused: qkv row [Hq*D + 2*Hkv*D]; unfused: rotated q row [Hq*D]
  const void* norm_w;
  void* k_cache;
  void* v_cache;
  void* out;
};

// One work "sequence" per blockIdx.z.  Mode kLayers: z indexes layers[], every sequence has
// the same past (meta[0] or pos_host).  Mode kRagged: z indexes sequences of one cache pair;
// rows start at offsets[z], past = past_dev[z], q/out rows z*ld.
// KV-cache storage of the ragged / paged decode: f16 rows, or int8 rows dequantised as
// f32(q) * scale with one f32 scale per tensor or per (kv head, dim) channel.
enum KvFormat { kKvF16 = 0, kKvI8 = 1 };

struct DecodeArgs {
  DecodeLayer layers[kMaxLayers];
  // ragged / paged modes
  const void* qkv;
  int64_t ld_qkv;
  const void* norm_w;
  void* k_cache;
  void* v_cache;
  const int32_t* offsets;
  const int32_t* past;
  int32_t max_past;      // a sequence with past > max_past is refused (the rope table's bound)
  // paged mode: k_cache / v_cache hold kv_cap pages of (1 << block_shift) token rows; key j of
  // sequence z lives in page block_table[z * max_blocks + (j >> block_shift)]
  const int32_t* block_table;
  int32_t max_blocks;
  int32_t block_shift;
  // int8 caches
  int32_t kv_format;       // KvFormat
  const float* k_scale;    // int8: 1 or hkv*64 scales (scale_per_channel)
  const float* v_scale;
  int32_t scale_per_channel;
  void* out;
  int64_t ld_o;
  // common
  const void* rope;
  const uint32_t* meta;  // nullable -> pos_host
  int32_t pos_host;
  int64_t kv_cap;        // rows per cache buffer: kLayers refuses a position >= kv_cap, kRagged
                         // a sequence with a negative entry or offsets[z] + past[z] >= kv_cap
  int32_t* err;          // device error word: bit 0 = position beyond the cache
  int32_t hq, hkv;
  float scale_log2;  // scale * log2(e)
  float eps;
  int32_t min_split;  // keys per split lower bound (multiple of 64)
  float* partials;    // [nz][hkv][max_splits][G][66]
  int32_t* counters;  // [nz][hkv], zero between launches
  int32_t wait_deficit;  // test hook: extra bytes the cluster combine waits for (0 normally)
  int32_t q_bcast;       // cluster form: rank 0 alone reads the qkv rows (host memory) and
                         // hands the rotated q to its peers
  int32_t pro_async;     // 1: the prologue's inputs (q/k/v heads, norm weights, rope row, key
                         // scales) are 16-byte aligned and device resident, and go to shared
                         // memory as the CTA's first cp.async group, ahead of its K/V tiles
  int32_t pdl;           // programmatic dependent launch: 0 off; 1 let the next kernel of the
                         // stream launch once every CTA has started, 2 once it has streamed
                         // its keys (the next kernel still waits for this one to complete
                         // before touching memory)
};

enum DecodeMode { kLayers = 0, kRagged = 1, kPaged = 2 };

// Block-table entries a paged split keeps in shared memory (a split covers at most
// (kPagedTableCap - 2) pages; the host sizes the grid so that it does).
constexpr int kPagedTableCap = 1024;

// grid = (max_splits, hkv, nz).  Workspace sizes in bytes for that grid.
size_t decode_partials_bytes(int max_splits, int hkv, int nz, int group);
size_t decode_counters_bytes(int hkv, int nz);
// cluster > 1: f16 kLayers only, max_splits == cluster (<= 8); the splits of one (layer,
// head chunk) form one thread-block cluster and combine through distributed shared memory,
// so partials/counters are not used.
cudaError_t launch_decode(const DecodeArgs& a, int mode, bool fused, int dtype, int max_splits,
                          int nz, cudaStream_t s, int cluster = 0);
// Cluster size for a decode step over nz layers (1 = use the workspace combine).
int decode_cluster_splits(int64_t max_len, int hkv, int group, int nz, bool fused, int num_sms);
// Choose the split count for a sequence of up to max_len keys.
int decode_max_splits(int64_t max_len, int hkv, int nz, int num_sms, int* min_split);

// ---- gemv_q4.cu -----------------------------------------------------------------------------
// A MatMulNBits matrix (bits 4, block 32, zero points): n rows of k values.
struct Q4Matrix {
  const uint32_t* qweight;      // [n][k/8], value 8w+i of a row is nibble i of word w
  const __half* scales;         // [n][k/32]
  const uint32_t* zero_points;  // bytes [n][ceil(k/32/2)] (low nibble: even block), as words
  int32_t n;
};
constexpr int kGemvMaxK = 4608;  // the GEMV shader's workgroup copy of x (kernels.js:31)
// Prompt-chunk projection on the tensor cores: y = x . W^T with W the dequantised f16 [n][k];
// plain (rows into y) or with QK_PREP on each 64-column head (prep != 0: columns [0, 64 hq)
// are q heads, then hkv k heads, then hkv v heads; q to q_out, k/v to cache rows pos0 + m).
struct GemmArgs {
  const void* x;  // f16 [m][ld_x]
  int64_t ld_x;
  const void* w16;  // f16 [n][k]
  int32_t m, n, k;  // n a multiple of 64
  void* y;          // plain: f16 rows [m][ld_y], outputs at column y_off
  int64_t ld_y, y_off;
  int32_t prep;
  int32_t hq, hkv;
  const void* norm_w;  // [q(64) | k(64)] or nullptr
  const void* rope;
  float eps;
  void* q_out;
  int64_t ld_q;
  void* k_cache;
  void* v_cache;
  int64_t kv_cap;
  const uint32_t* meta;  // nullable -> pos0
  int32_t pos0;
  int32_t* err;
  int32_t bn;    // output tile width 256 / 192 / 128; 0 = chosen by gemm_tiling()
  int32_t pair;  // 1: 2-CTA tiles (tcgen05 cta_group::2), 0: one CTA per tile, -1: chosen
};
struct GemmTiling {
  int bn;
  bool pair;
};
// The tiling with the shortest estimated makespan of m x n over `sms` persistent CTAs
// (force_bn 0 / force_pair -1: free).
GemmTiling gemm_tiling(int64_t m, int64_t n, int sms, int force_bn, int force_pair);
// f16 copies of `count` (1-3) 4-bit matrices with the same k, stacked along n in dst_f16.
cudaError_t launch_dequant_q4(const Q4Matrix* ws, int count, int32_t k, void* dst_f16,
                              cudaStream_t s);
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t s);
struct GemvArgs {
  Q4Matrix w;
  int32_t k;
  const void* x;  // f16 [k]
  void* y;        // f16, rows at y_off..y_off+n-1
  int64_t y_off;
};
struct QkvPrepArgs {
  Q4Matrix wq, wk, wv;  // Hq*64, Hkv*64, Hkv*64 rows of k values
  int32_t k;
  const void* x;        // f16 [k]: the normed hidden row of the token
  const void* norm_w;   // [q(64) | k(64)] or NULL
  const void* rope;     // [max_ctx][64]
  void* q_out;          // f16 [Hq*64]: rotated q
  void* k_cache;        // [cap][Hkv][64]: rotated k at row pos
  void* v_cache;        // [cap][Hkv][64]: v at row pos
  int64_t kv_cap;
  const uint32_t* meta;  // nullable -> pos_host
  int32_t pos_host;
  int32_t hq, hkv;
  float eps;
  int32_t* err;
};
cudaError_t launch_gemv_q4(const GemvArgs& a, cudaStream_t s);
cudaError_t launch_qkv_prep(const QkvPrepArgs& a, cudaStream_t s);

// ---- kv_quant.cu ----------------------------------------------------------------------------
// f16 cache rows [rows][hkv][64] -> int8, q = clamp(roundeven(x / scale), -128, 127) with one
// scale (scale_count 1) or one per (kv head, dim) channel (scale_count hkv*64).
cudaError_t launch_quantize_q8(const void* src, void* dst, int64_t rows, int hkv,
                               const float* scale, int scale_count, cudaStream_t s);

// ---- prefill_sm100.cu ----------------------------------------------------------------------
constexpr int kMaxFlashOuts = 8;  // output buffers one flash launch writes (one per rank)
struct FlashArgs {
  const void* q;  // [B][Sq][ld_q] rows, head h at column h*64
  const void* k;  // [B][Skv][ld_kv] rows, kv head at column kh*64
  const void* v;
  void* out;      // [B][Sq][ld_o]; head h of this call at column (out_head0 + h)*64
  void* extra_out[kMaxFlashOuts - 1];  // more buffers of out's layout that get the same rows
  int32_t n_extra_out;                 // (other GPUs' outputs, written over NVLink)
  int32_t out_head0;
  void* mc_out;  // non-null: NVLink multicast address of every GPU's output (out unused)
  int64_t ld_q, ld_kv, ld_o;
  int64_t q_rows_total, kv_rows_total;  // rows of the q / kv 2-D views (tensor-map extents)
  int64_t batch_stride_q_rows, batch_stride_kv_rows;  // rows between images
  int32_t batch;
  int32_t s_q;       // query rows per image (M)
  int32_t s_kv;      // key rows per image for non-causal; ignored when causal
  int32_t hq, hkv;
  int32_t causal;
  const uint32_t* meta;  // causal: pos0 = meta[0] (nullable -> pos0_host)
  int32_t pos0_host;
  float scale_log2;
  int32_t* err;          // device error word: bit 0 = position beyond the cache
  int32_t wait_deficit;  // test hook: extra bytes the Q-tile wait expects (0 normally)
  int32_t num_sms;       // non-causal: > 0 lets the last partial wave run as one-tile CTAs
};

// Device error word bits.
constexpr int kErrPosBeyondCache = 1;
constexpr int kErrTimeout = 2;  // a bounded device-side wait ran out; that work was not written
constexpr int kErrOutTokFull = 4;  // argmax_step: the step index reached out_tok's capacity
constexpr int kErrLayout = 8;  // a kernel found its shared memory misplaced; it wrote nothing
cudaError_t launch_flash(const FlashArgs& a, cudaStream_t s);

}  // namespace p2p
