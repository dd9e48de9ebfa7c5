/*
 * p2p_attn.h -- C ABI of the B200 (sm_100a) attention library for the LFM2.5-VL engine.
 *
 * The library replaces the three attention shaders of the reference engine and the buffer
 * plumbing around them:
 *   QK_PREP      src/scripts/lfm-engine/kernels.js:216-266   -> p2p_qk_prep
 *   ATTN         src/scripts/lfm-engine/kernels.js:268-319   -> p2p_attn (prefill and decode)
 *   QK_PREP+ATTN at M=1 for every attention layer of a step  -> p2p_decode_step
 *   ATTN over many independent sequences (ragged KV cache)   -> p2p_attn_decode_ragged
 *   VISION_ATTN  src/scripts/lfm-engine/vision-kernels.js:176-258 -> p2p_attn_bidir
 *   ropeTable    src/scripts/lfm-engine/engine.js:60-71      -> p2p_rope_table
 *   meta buffer  src/scripts/lfm-engine/engine.js:144,388,422 -> p2p_meta / p2p_meta_write
 *   ARGMAX       src/scripts/lfm-engine/kernels.js:362-399   -> p2p_argmax_step (the greedy
 *                token and the device-side advance of the meta buffer's position and step)
 *   KV cache     src/scripts/lfm-engine/engine.js:152-165 (alloc), :274-304 (growth)
 *                                                            -> p2p_kv_*
 *
 * Layouts are the reference's (row-major, f16 unless dtype says otherwise):
 *   qkv row      [Hq*D | Hkv*D | Hkv*D]      (kernels.js:219, engine.js:202-204)
 *   q / out      [M][ld] with head h at column h*D           (kernels.js:263, :317)
 *   K/V cache    [cap][Hkv][D] token-major, one K and one V buffer per layer (kernels.js:219)
 *   norm weights [q_norm(D) | k_norm(D)]     (engine.js:205-212)
 *   rope         [max_ctx][D] = [cos(D/2) | sin(D/2)] per position (engine.js:60-71)
 *   meta         uint32[4] = [pos0, M, step, 0] in device memory (engine.js:144, :388)
 *   vision q/k/v [B][S][ld] with head h at column h*D         (vision-kernels.js:198)
 *
 * Conventions: every call is asynchronous on the given CUDA stream (a cudaStream_t passed as
 * void*; NULL is the CUDA default stream, p2p_ctx_stream() the context's own stream).  A context is not thread-safe; use one per host thread.
 * Calls return a p2p_status and never abort; p2p_last_error() describes the last failure.
 * head_dim must be 64 (the reference's only head size); num_heads % num_kv_heads == 0 and
 * num_heads / num_kv_heads in {1, 2, 4, 8}.
 */
#ifndef P2P_ATTN_H
#define P2P_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define P2P_ATTN_ABI_VERSION 2

typedef enum p2p_status {
  P2P_OK = 0,
  P2P_ERR_INVALID_ARG = 1, /* bad shape, null pointer, misaligned buffer, bad dtype */
  P2P_ERR_OOM = 2,         /* device allocation failed (engine.js:280-286 error scope) */
  P2P_ERR_KV_FULL = 3,     /* KV cache cannot hold the request (engine.js:418-421 'kv_full') */
  P2P_ERR_CUDA = 4,        /* a CUDA runtime call failed */
  P2P_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up */
  P2P_ERR_NCCL = 6,        /* a collective failed */
  P2P_ERR_UNSUPPORTED = 7  /* valid request this build does not implement (e.g. head_dim != 64) */
} p2p_status;

typedef enum p2p_dtype { P2P_F16 = 0, P2P_F32 = 1 } p2p_dtype;

/* Uniform parameters of one attention layer (the WGSL constants and overrides:
 * kernels.js:268 (16/8/64, 0.125), vision-kernels.js:182-185 (S, NUM_HEADS, HEAD_DIM, SCALE)). */
typedef struct p2p_attn_params {
  int32_t num_heads;    /* Hq  (reference decoder 16, LFM2.5-1.2B 32, vision 12) */
  int32_t num_kv_heads; /* Hkv (reference 8; vision: equal to num_heads) */
  int32_t head_dim;     /* D = 64 */
  float scale;          /* multiplies f32(q); 0 selects 1/sqrt(D) = 0.125 */
  float eps;            /* q/k RMSNorm epsilon (kernels.js:252: 1e-5); 0 selects 1e-5 */
  int32_t dtype;        /* p2p_dtype of q/k/v/out/cache/rope; P2P_F32 only for decode */
} p2p_attn_params;

typedef struct p2p_ctx p2p_ctx;
typedef struct p2p_kv p2p_kv;

int p2p_abi_version(void);
const char* p2p_status_string(p2p_status s);

/* Context: owns a CUDA stream, the split-KV workspace and the meta buffer on `device`. */
p2p_status p2p_ctx_create(int device, p2p_ctx** out);
p2p_status p2p_ctx_destroy(p2p_ctx* ctx);
const char* p2p_last_error(const p2p_ctx* ctx);
void* p2p_ctx_stream(p2p_ctx* ctx); /* the context's cudaStream_t */
/* Waits for `stream`, then reports device-side refusals since the last p2p_sync (a position
 * read from meta_dev beyond the cache returns P2P_ERR_KV_FULL; the kernel skipped that work). */
p2p_status p2p_sync(p2p_ctx* ctx, void* stream);

/* engine.js:60-71: builds (once per (max_ctx, D, theta, dtype)) the table
 * rope[p][i] = cos(p * theta^(-i/(D/2))), rope[p][D/2+i] = sin(...), evaluated in double and
 * rounded through f32 to the storage type; returns a device pointer owned by the context. */
p2p_status p2p_rope_table(p2p_ctx* ctx, int32_t max_ctx, int32_t head_dim, double theta,
                          int32_t dtype, const void** dev_table);

/* engine.js:144: the device meta buffer [pos0, M, step, 0]; p2p_meta_write is the
 * queue.writeBuffer of engine.js:388/408/422 (an async 16-byte copy on `stream`). */
p2p_status p2p_meta(p2p_ctx* ctx, uint32_t** dev_meta);
p2p_status p2p_meta_write(p2p_ctx* ctx, uint32_t pos0, uint32_t m_tokens, uint32_t step,
                          void* stream);

/* kernels.js:362-399 (ARGMAX, dispatched at engine.js:239-240, 265-266 with the bindings
 * logits, tok, mt, outTok): the greedy token over `vocab` f16 logits -- the smallest index
 * among the maxima of the values above -3e38 (NaN never wins), else 0 -- is stored in tok[0]
 * and out_tok[meta[2]], then meta[2] (step) and meta[0] (position) advance by one, all on the
 * device, so the next decode step reads its position from the meta buffer without a host
 * write.  meta_dev NULL uses the context's meta buffer.  When meta[2] >= out_tok_cap the
 * token is not stored in out_tok and p2p_sync reports P2P_ERR_INVALID_ARG. */
p2p_status p2p_argmax_step(p2p_ctx* ctx, const void* logits, int32_t vocab, uint32_t* tok,
                           uint32_t* out_tok, int64_t out_tok_cap, uint32_t* meta_dev,
                           void* stream);

/* engine.js:152-165: one K and one V buffer [cap][Hkv][D] per attention layer. */
p2p_status p2p_kv_create(p2p_ctx* ctx, int32_t n_layers, int32_t num_kv_heads,
                         int32_t head_dim, int64_t cap_tokens, int32_t dtype, p2p_kv** out);
p2p_status p2p_kv_destroy(p2p_kv* kv);
/* engine.js:274-304: if need > capacity, grow in steps of grow_tokens (at most max_tokens),
 * copying the old rows; returns P2P_ERR_KV_FULL when need > max_tokens and P2P_ERR_OOM when
 * the allocation fails (the old cache is then kept).  Pointers change on growth. */
p2p_status p2p_kv_ensure_capacity(p2p_kv* kv, int64_t need_tokens, int64_t grow_tokens,
                                  int64_t max_tokens, void* stream);
int64_t p2p_kv_capacity(const p2p_kv* kv);
void* p2p_kv_k(const p2p_kv* kv, int32_t layer);
void* p2p_kv_v(const p2p_kv* kv, int32_t layer);

/* kernels.js:216-266 (QK_PREP, dispatched (Hq+2Hkv, M) at engine.js:221): for token m at
 * pos = pos0 + m, per-head RMSNorm of q and k (eps, weights norm_w = [q(D) | k(D)], result
 * rounded to f16), rotate-half RoPE with the f16 table, rotated q to q_out, rotated k and raw
 * v to cache row pos.  norm_w NULL skips the norm.  pos0 is read from meta_dev[0] on the
 * device when meta_dev is not NULL (then the host pos0 argument is ignored).  kv_cap_tokens
 * is the number of rows the cache buffers hold: a host pos0 + M beyond it returns
 * P2P_ERR_KV_FULL; a device-side position beyond it is skipped and reported by p2p_sync. */
p2p_status p2p_qk_prep(p2p_ctx* ctx, const p2p_attn_params* prm, const void* qkv,
                       int64_t ld_qkv, const void* norm_w, const void* rope, void* q_out,
                       int64_t ld_q, void* k_cache, void* v_cache, int64_t kv_cap_tokens,
                       const uint32_t* meta_dev, int32_t pos0, int32_t m_tokens, void* stream);

/* kernels.js:268-319 (ATTN, dispatched (Hq, M) at engine.js:222): causal GQA of M rotated
 * query rows at positions pos0..pos0+M-1 over cache keys 0..pos, kv head h / (Hq/Hkv),
 * out = f16(softmax(scale * q.k) v).  M == 1 runs the split-KV decode kernel; M > 1 runs the
 * tcgen05 flash-attention kernel.  kv_cap_tokens is the number of rows the cache buffers
 * hold (bounds the work grid when pos0 comes from meta_dev). */
p2p_status p2p_attn(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q, int64_t ld_q,
                    const void* k_cache, const void* v_cache, int64_t kv_cap_tokens, void* out,
                    int64_t ld_o, const uint32_t* meta_dev, int32_t pos0, int32_t m_tokens,
                    void* stream);

/* Head-sharded causal prefill on several GPUs of one node (one process per GPU).  Each rank
 * runs ATTN (kernels.js:268-319) for its own kv-head group -- prm counts the local heads, q
 * and the caches hold only them -- and the kernel writes every output row straight into the
 * full [M][ld_o] output buffer of every rank: outs[0] is this rank's own, outs[1..n_outs)
 * other ranks' buffers opened with p2p_shared_open (the rows cross NVLink as the kernel's own
 * stores), local head h at column (out_head0 + h) * D of each.  This replaces ATTN followed by
 * an all-gather of the per-rank slices and their reassembly.  The call only orders this
 * rank's writes; before a rank reads its buffer (or any rank writes the buffers again) the
 * ranks must order themselves, e.g. with any collective on the stream after this call. */
#define P2P_MAX_SCATTER_OUTS 8
p2p_status p2p_attn_scatter(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q,
                            int64_t ld_q, const void* k_cache, const void* v_cache,
                            int64_t kv_cap_tokens, void* const* outs, int32_t n_outs,
                            int64_t ld_o, int32_t out_head0, const uint32_t* meta_dev,
                            int32_t pos0, int32_t m_tokens, void* stream);

/* As p2p_attn_scatter, but the output rows go out once, as NVLink multicast stores
 * (multimem.st) to mc_out, the multicast address of a buffer bound on every rank of the node
 * (e.g. a symmetric-memory allocation with multicast support): NVSwitch writes each row into
 * every rank's [M][ld_o] buffer, so a GPU sends its rows once instead of once per peer. */
p2p_status p2p_attn_multicast(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q,
                              int64_t ld_q, const void* k_cache, const void* v_cache,
                              int64_t kv_cap_tokens, void* mc_out, int64_t ld_o,
                              int32_t out_head0, const uint32_t* meta_dev, int32_t pos0,
                              int32_t m_tokens, void* stream);

/* Device buffers shared between the processes of one node (CUDA IPC): p2p_shared_alloc
 * allocates `bytes` on the context's device and returns an opaque handle that another
 * process passes to p2p_shared_open to map the same memory (its GPU then reads and writes it
 * over NVLink).  Close every mapping (p2p_shared_close) before the owner frees the buffer
 * (p2p_shared_free); both wait for the device first. */
#define P2P_IPC_HANDLE_BYTES 64
p2p_status p2p_shared_alloc(p2p_ctx* ctx, size_t bytes, void** ptr,
                            unsigned char handle[P2P_IPC_HANDLE_BYTES]);
p2p_status p2p_shared_free(p2p_ctx* ctx, void* ptr);
p2p_status p2p_shared_open(p2p_ctx* ctx, const unsigned char handle[P2P_IPC_HANDLE_BYTES],
                           void** ptr);
p2p_status p2p_shared_close(p2p_ctx* ctx, void* ptr);

/* The library's own communicator over the GPUs of one node (one process per GPU), used by
 * p2p_attn_prefill_sharded and to order the ranks after p2p_attn_scatter/_multicast.  NCCL is
 * loaded at run time (libnccl.so.2; P2P_NCCL_LIB names another file).  Rank 0 calls
 * p2p_comm_unique_id and hands the bytes to the other ranks over any side channel; every rank
 * then calls p2p_comm_create.  Every wait on the other ranks is bounded by timeout_ms on the
 * host: when it runs out the communicator is aborted (its collectives in flight end) and the
 * call returns P2P_ERR_TIMEOUT; an NCCL failure returns P2P_ERR_NCCL.  An aborted communicator
 * returns P2P_ERR_NCCL from every later call; destroy it and create a new one.  The reference
 * has no multi-GPU code: these serve the ATTN dispatch (engine.js:222) split over GPUs. */
#define P2P_COMM_ID_BYTES 128
typedef struct p2p_comm p2p_comm;
p2p_status p2p_comm_unique_id(unsigned char id[P2P_COMM_ID_BYTES]);
p2p_status p2p_comm_create(p2p_ctx* ctx, int32_t nranks, int32_t rank,
                           const unsigned char id[P2P_COMM_ID_BYTES], int32_t timeout_ms,
                           p2p_comm** out);
p2p_status p2p_comm_destroy(p2p_comm* comm);
/* Waits (bounded) until `stream` has drained, collectives included, then as p2p_sync. */
p2p_status p2p_comm_wait(p2p_comm* comm, void* stream);
/* A one-element all-reduce on `stream`: every rank's earlier work on its stream (e.g. the
 * NVLink stores of p2p_attn_scatter) is complete before any rank's later work starts. */
p2p_status p2p_comm_barrier(p2p_comm* comm, void* stream);

/* kernels.js:216-319 (QK_PREP + ATTN of a causal prompt chunk) split by kv-head group over the
 * communicator's ranks: rank g owns kv heads [g*Hkv/G, (g+1)*Hkv/G) and their q heads.  prm
 * counts the model's heads; qkv holds this rank's columns only, [M][ld_qkv] rows
 * [its q heads | its k heads | its v heads] (what a column-parallel QKV projection produces);
 * k_cache/v_cache are this rank's [cap][Hkv/G][D] slices, written at rows pos0..pos0+M-1.
 * The rank's attention rows are exchanged with one all-gather over NVLink and every rank's
 * out [M][ld_o] receives all heads (head h at column h*D).  Workspace lives in the
 * communicator and grows on the first call of a larger M (capture graphs after that call). */
p2p_status p2p_attn_prefill_sharded(p2p_ctx* ctx, p2p_comm* comm, const p2p_attn_params* prm,
                                    const void* qkv, int64_t ld_qkv, const void* norm_w,
                                    const void* rope, void* k_cache, void* v_cache,
                                    int64_t kv_cap_tokens, const uint32_t* meta_dev,
                                    int32_t pos0, int32_t m_tokens, void* out, int64_t ld_o,
                                    void* stream);

/* One decode step (QK_PREP then ATTN with M = 1, engine.js:425-429) for up to
 * P2P_MAX_LAYERS attention layers in ONE launch: for each layer the new token's qkv row is
 * normed/rotated, its k/v are appended at row pos, and its Hq output rows are written.
 * Layers are independent (each layer's q comes from its own qkv row).  The qkv and out rows
 * may be device memory or page-locked host memory (cudaHostAlloc / cudaHostRegister): the
 * kernel then reads the inputs and writes the outputs across the host link itself, with no
 * separate copy, and the host reads the outputs after synchronizing the stream.  The caches,
 * norm weights, rope table and meta buffer stay in device memory. */
#define P2P_MAX_LAYERS 16
typedef struct p2p_decode_layer {
  const void* qkv;    /* [Hq*D + 2*Hkv*D] row of the new token */
  const void* norm_w; /* [q(D) | k(D)] or NULL */
  void* k_cache;      /* [cap][Hkv][D] */
  void* v_cache;
  void* out;          /* [Hq*D] */
} p2p_decode_layer;
p2p_status p2p_decode_step(p2p_ctx* ctx, const p2p_attn_params* prm, int32_t n_layers,
                           const p2p_decode_layer* layers, const void* rope,
                           int64_t kv_cap_tokens, const uint32_t* meta_dev, int32_t pos,
                           void* stream);

/* Batched decode over nseq independent sequences sharing one cache buffer pair
 * [kv_rows][Hkv][D]: sequence i owns rows offsets[i] .. offsets[i]+past[i] and its new token
 * goes to row offsets[i]+past[i].  With fused_prep != 0, qkv rows [nseq][ld_qkv] are
 * normed/rotated and the new k/v appended (as p2p_decode_step); with fused_prep == 0, qkv
 * holds already-rotated q rows [nseq][ld_qkv] and the new k/v must already be in the cache.
 * offsets and past are device int32 arrays.  max_past is the largest past[i] allowed: it sizes
 * the grid, and the rope table must hold at least max_past + 1 rows.  The kernel checks every
 * sequence before touching it: one with a negative entry, past[i] > max_past or
 * offsets[i] + past[i] >= kv_rows is skipped (its output rows are not written) and the next
 * p2p_sync returns P2P_ERR_KV_FULL; the other sequences are computed normally. */
p2p_status p2p_attn_decode_ragged(p2p_ctx* ctx, const p2p_attn_params* prm, const void* qkv,
                                  int64_t ld_qkv, const void* norm_w, const void* rope,
                                  void* k_cache, void* v_cache, int64_t kv_rows,
                                  const int32_t* offsets, const int32_t* past, int32_t nseq,
                                  int32_t max_past, int32_t fused_prep, void* out, int64_t ld_o,
                                  void* stream);

/* KV-cache formats beyond the engine's f16 token-major buffers, for the batched decode:
 *   - int8 rows (the int8 cache of the reference bundle's GroupQueryAttention kernels,
 *     public/kernels/megakernel.json: a value is stored as q = clamp(roundeven(x / scale),
 *     -128, 127) and read as f32(q) * scale, with one f32 scale per tensor or one per
 *     (kv head, dim) channel, index kh*D + d), which halves the bytes a decode step streams;
 *   - paged caches (the bundle's PagedAttention layout): k_cache / v_cache are pools of
 *     [kv_rows pages][block_size][Hkv][D] and key j of sequence i is row j % block_size of page
 *     block_table[i * max_blocks + j / block_size].
 * block_size 0 selects the contiguous form of p2p_attn_decode_ragged (offsets). */
typedef enum p2p_kv_format { P2P_KV_F16 = 0, P2P_KV_I8 = 1 } p2p_kv_format;
typedef struct p2p_kv_layout {
  int32_t format;              /* p2p_kv_format */
  const float* k_scale;        /* int8: scale_count f32 scales in device memory */
  const float* v_scale;
  int32_t scale_count;         /* 1 (per tensor) or Hkv*D (per channel) */
  int32_t block_size;          /* 0: contiguous rows at offsets[i]; else tokens per page, a
                                  power of two in 16..4096 */
  const int32_t* block_table;  /* paged: device int32 [nseq][max_blocks] page indices */
  int32_t max_blocks;
} p2p_kv_layout;

/* p2p_attn_decode_ragged over any of these formats: kv_rows counts the cache's rows
 * (contiguous) or pages (paged); offsets is used by the contiguous form only.  With fused_prep
 * the new token's k/v are appended in the cache's format (int8: quantised as above).  The
 * kernel checks every sequence before touching it -- a negative entry, past[i] > max_past,
 * rows beyond kv_rows, more pages than max_blocks or a block-table entry outside the pool --
 * and skips it; p2p_sync then returns P2P_ERR_KV_FULL. */
p2p_status p2p_attn_decode_kv(p2p_ctx* ctx, const p2p_attn_params* prm,
                              const p2p_kv_layout* layout, const void* qkv, int64_t ld_qkv,
                              const void* norm_w, const void* rope, void* k_cache,
                              void* v_cache, int64_t kv_rows, const int32_t* offsets,
                              const int32_t* past, int32_t nseq, int32_t max_past,
                              int32_t fused_prep, void* out, int64_t ld_o, void* stream);

/* Converts f16 cache rows [rows][Hkv][D] to the int8 format above (src 16-byte and dst 8-byte
 * aligned; the same restated rule the decode uses when it appends). */
p2p_status p2p_kv_quantize_q8(p2p_ctx* ctx, const void* src, void* dst, int64_t rows,
                              int32_t num_kv_heads, const float* scale, int32_t scale_count,
                              void* stream);

/* The 4-bit projections on either side of the attention path, for one token (decode).  A
 * matrix is ONNX MatMulNBits with bits 4, block 32 and zero points (kernels.js:4-9): qweight
 * u32 [n][k/8] (value 8w+i of a row is nibble i of word w), scales f16 [n][k/32], zero_points
 * bytes [n][ceil(k/32/2)] (low nibble = even block; 4-byte aligned, read as u32 words), value
 * (q - zp) * scale.  k must be a multiple of 32 and at most 4608.  Every output is computed
 * as the GEMV shader computes it (kernels.js:22-68), so the results are bit-identical to it. */
typedef struct p2p_q4_matrix {
  const void* qweight;
  const void* scales;
  const void* zero_points;
  int32_t n;
  int32_t k;
} p2p_q4_matrix;

/* kernels.js:22-68 (GEMV): y[y_off + n] = f16(x . W[n]) for one f16 row x [k] -- the o_proj
 * that consumes the attention row (engine.js:224), or any other projection of the engine. */
p2p_status p2p_gemv_q4(p2p_ctx* ctx, const p2p_q4_matrix* w, const void* x, void* y,
                       int64_t y_off, void* stream);

/* The q/k/v projections of one token (three GEMV dispatches, engine.js:202-204) with QK_PREP
 * (kernels.js:216-266) in their epilogue: from the normed hidden row x [k], wq/wk/wv with
 * Hq*64 / Hkv*64 / Hkv*64 rows produce the qkv row in f16 (never written to memory), whose
 * heads are normed and rotated as QK_PREP does -- rotated q to q_out [Hq*64], rotated k and raw
 * v to cache row pos (meta_dev[0] when meta_dev is not NULL).  Bit-identical to the GEMVs
 * followed by QK_PREP.  A host position at or beyond kv_cap_tokens returns P2P_ERR_KV_FULL; a
 * device one is refused by the kernel (nothing written) and reported by p2p_sync. */
p2p_status p2p_qkv_gemv_prep(p2p_ctx* ctx, const p2p_attn_params* prm, const void* x,
                             const p2p_q4_matrix* wq, const p2p_q4_matrix* wk,
                             const p2p_q4_matrix* wv, const void* norm_w, const void* rope,
                             void* q_out, void* k_cache, void* v_cache, int64_t kv_cap_tokens,
                             const uint32_t* meta_dev, int32_t pos, void* stream);

/* kernels.js:70-145 (GEMM): the same projection for a prompt chunk of M > 1 tokens,
 * y[m * ld_y + y_off + n] = f16(x[m] . W[n]) for x [M][ld_x].  The weights are dequantised to
 * f16 (each value rounded once; the shader keeps f32) into a context workspace and multiplied
 * on the tensor cores with f32 accumulation, so results agree with the shader to f16 rounding,
 * not bit for bit.  No k limit; n a multiple of 64; x and y rows 16-byte aligned (ld_x, ld_y
 * and y_off multiples of 8).  The workspace is shared by the context's calls: calls on
 * different streams of one context must not overlap.  It grows (synchronising the device) on
 * the first call with a larger matrix: make that call before capturing a CUDA graph. */
p2p_status p2p_gemm_q4(p2p_ctx* ctx, const p2p_q4_matrix* w, const void* x, int64_t ld_x,
                       int32_t m_tokens, void* y, int64_t ld_y, int64_t y_off, void* stream);

/* The q/k/v projections of a prompt chunk (three GEMM dispatches, engine.js:202-204) with
 * QK_PREP (kernels.js:216-266) in the epilogue: from the normed hidden rows x [M][ld_x], the
 * f16 qkv row of every token is formed on the tensor cores (never written to memory) and its
 * heads are normed and rotated as QK_PREP does -- rotated q to q_out [M][ld_q], rotated k and
 * raw v to cache rows pos0 .. pos0+M-1 (pos0 = meta_dev[0] when meta_dev is not NULL).
 * Given the same f16 projection the QK_PREP part is bit-identical to the shader.  Positions as
 * in p2p_qk_prep; alignment as in p2p_gemm_q4. */
p2p_status p2p_qkv_gemm_prep(p2p_ctx* ctx, const p2p_attn_params* prm, const void* x,
                             int64_t ld_x, const p2p_q4_matrix* wq, const p2p_q4_matrix* wk,
                             const p2p_q4_matrix* wv, const void* norm_w, const void* rope,
                             void* q_out, int64_t ld_q, void* k_cache, void* v_cache,
                             int64_t kv_cap_tokens, const uint32_t* meta_dev, int32_t pos0,
                             int32_t m_tokens, void* stream);

/* Resident f16 weights.  The engine builds every 4-bit matrix once (engine.js:100, `proj`) and
 * the GEMM entry points above dequantise it again on every call.  A B200 holds the f16 copy of
 * all of a small model's projections many times over, so the copy can be made once, where the
 * engine uploads its weights, and reused by every prompt chunk:
 *   p2p_q4_to_f16       dst [n][k] f16 = (q - zp) * scale, rounded once (the same values the
 *                       4-bit GEMM entry points compute per call); dst 16-byte aligned.
 *   p2p_gemm_f16w       p2p_gemm_q4 on such a copy (w16 [n][k], k a multiple of 8);
 *   p2p_qkv_gemm_prep_f16w  p2p_qkv_gemm_prep on the q, k and v copies stacked along n:
 *                       w16_qkv [q rows | k rows | v rows][k].
 * Given the same copy, the outputs equal the 4-bit entry points' bit for bit.  These two use no
 * context workspace, so calls on different streams may overlap. */
p2p_status p2p_q4_to_f16(p2p_ctx* ctx, const p2p_q4_matrix* w, void* dst, void* stream);
p2p_status p2p_gemm_f16w(p2p_ctx* ctx, const void* w16, int32_t n, int32_t k, const void* x,
                         int64_t ld_x, int32_t m_tokens, void* y, int64_t ld_y, int64_t y_off,
                         void* stream);
p2p_status p2p_qkv_gemm_prep_f16w(p2p_ctx* ctx, const p2p_attn_params* prm, const void* x,
                                  int64_t ld_x, const void* w16_qkv, int32_t k,
                                  const void* norm_w, const void* rope, void* q_out,
                                  int64_t ld_q, void* k_cache, void* v_cache,
                                  int64_t kv_cap_tokens, const uint32_t* meta_dev, int32_t pos0,
                                  int32_t m_tokens, void* stream);

/* vision-kernels.js:176-258 (VISION_ATTN, dispatched (NUM_HEADS, S) at vision.js:271-276),
 * batched: out[b] = softmax(scale * q[b] k[b]^T) v[b] per head, no mask, tcgen05 kernel.
 * q/k/v/out are [batch][s_tokens][ld] with head h at column h*D. */
p2p_status p2p_attn_bidir(p2p_ctx* ctx, const p2p_attn_params* prm, const void* q,
                          const void* k, const void* v, void* out, int64_t ld, int32_t batch,
                          int32_t s_tokens, void* stream);

/* No counterpart in the reference.  The same operation as p2p_attn_decode_ragged (same
 * arguments, same kernel) for callers that cannot allocate device memory while serving:
 * processes that hand nearly all free HBM to their own pool at start-up, and hosts whose device
 * memory belongs to another component.  It never calls cudaMalloc/cudaFree: the split-KV
 * scratch lives in a fixed array of P2P_NOALLOC_SCRATCH_BYTES inside the library, which every
 * GPU that loads the library holds until the process exits.  A request whose scratch
 * (nseq x kv heads x splits x up to 4 heads x 66 floats, plus counters) exceeds it returns
 * P2P_ERR_INVALID_ARG with the sizes in p2p_last_error().  p2p_ctx_create looks up the
 * array's device address on its device (loading the module that holds it, which is when the
 * array takes its place in device memory), so the array is in place before the host reserves
 * its pool if the context is created first; the calls themselves then allocate nothing.
 * Sequences are checked as for p2p_attn_decode_ragged (kv_rows, max_past).  All calls share
 * the array: calls that overlap on the GPU (other streams, other contexts on the same device)
 * race and must be ordered by the caller. */
#define P2P_NOALLOC_SCRATCH_BYTES (32u << 20)
p2p_status p2p_attn_decode_ragged_noalloc(p2p_ctx* ctx, const p2p_attn_params* prm,
                                          const void* qkv, int64_t ld_qkv, const void* norm_w,
                                          const void* rope, void* k_cache, void* v_cache,
                                          int64_t kv_rows, const int32_t* offsets,
                                          const int32_t* past,
                                          int32_t nseq, int32_t max_past, int32_t fused_prep,
                                          void* out, int64_t ld_o, void* stream);

/* Test hook, no counterpart in the reference: cap this process's device allocations made by
 * the library at `bytes` (< 0 removes the cap), so the P2P_ERR_OOM paths can be exercised
 * without exhausting a shared GPU. */
p2p_status p2p_debug_set_alloc_limit(int64_t bytes);

/* Test hook, no counterpart in the reference: kernels launched afterwards that wait on other
 * CTAs or on copies (the flash prefill's Q tile, the decode step's cluster combine) expect
 * `bytes` more on that wait than will ever arrive, so the wait runs out after its 1 s limit,
 * the kernel writes no output for that work and the next p2p_sync returns P2P_ERR_TIMEOUT.
 * 0 restores normal operation.  Exercises the bounded-wait path without any fault. */
p2p_status p2p_debug_set_wait_deficit(int32_t bytes);

/* Measurement reference, no counterpart in the reference: one launch that reads `bytes`
 * (a multiple of 16) from the 16-byte aligned device buffer src once, with the plainest
 * full-bandwidth access pattern (16-byte loads, eight in flight per thread, two 512-thread
 * CTAs per SM), and XORs every 32-bit word into *xor_out (device memory; the caller zeroes
 * it).  Timed like a decode step, it is the speed of light of streaming those bytes in one
 * launch. */
p2p_status p2p_debug_stream_read(p2p_ctx* ctx, const void* src, int64_t bytes,
                                 uint32_t* xor_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
