/*
 * p2p_oracle.h -- CPU restatement of the reference attention path (TEST INFRASTRUCTURE).
 *
 * This library is the parity checker and the timed CPU baseline.  It is never linked into,
 * loaded by, or called from the product library (p2p_b200/libp2pattn.so); only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs use it.
 *
 * It restates, in the same loop order, chunk sizes and f16 rounding points:
 *   - toHalfBits         src/scripts/lfm-engine/engine.js:28-50
 *   - ropeTable          src/scripts/lfm-engine/engine.js:60-71
 *   - QK_PREP            src/scripts/lfm-engine/kernels.js:216-266
 *   - ATTN               src/scripts/lfm-engine/kernels.js:268-319
 *   - VISION_ATTN        src/scripts/lfm-engine/vision-kernels.js:176-258
 *   - ARGMAX             src/scripts/lfm-engine/kernels.js:362-399 (greedy token + the
 *                        device-side advance of the meta buffer's position and step)
 * generalised from the reference's hard-coded 16 q heads / 8 kv heads / head_dim 64 /
 * row strides 2048, 1024, 768 to runtime (Hq, Hkv, D, strides).  For Hq=16, Hkv=8, D=64 it
 * performs the reference's operations in the reference's order.
 *
 * Parity pin: the reference is WGSL inside JavaScript and cannot execute here (no WebGPU,
 * no Node).  oracle/wgsl2cpp.py mechanically translates the reference's own shader text
 * into C++ (written to oracle/_ref/, never committed) and tests/test_oracle_pin.py checks
 * this restatement bit-for-bit against that translation on seeded inputs; toHalfBits is
 * checked exhaustively against IEEE round-to-nearest-even.  Where oracle/_ref cannot be
 * built (no reference sources present), parity against the reference is unpinned and
 * rests on the committed golden fixtures produced by that translation.
 *
 * Storage: "h" functions take IEEE binary16 bit patterns (uint16_t); "f" functions take
 * float storage and drop every f16 rounding point (the fp32 decode case).
 * All arithmetic is IEEE single precision without FMA contraction (-ffp-contract=off).
 */
#ifndef P2P_ORACLE_H
#define P2P_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* engine.js:28-50: f32 -> f16 bits, round to nearest even, subnormals kept. */
uint16_t p2p_or_f32_to_f16(float v);
float p2p_or_f16_to_f32(uint16_t h);
void p2p_or_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n);
void p2p_or_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n);

/* engine.js:60-71: out[p][0:D/2] = f16(cos(p * theta^(-i/(D/2)))), out[p][D/2:D] = sin.
 * The angle and the trig are evaluated in double; the result goes double -> f32 -> f16
 * exactly as toHalfBits does (Float32Array store, then RNE to half). */
void p2p_or_rope_table(int max_ctx, int d, double theta, uint16_t* out);
/* The same table kept in f32 (used by the fp32-storage decode case). */
void p2p_or_rope_table_f32(int max_ctx, int d, double theta, float* out);

/* kernels.js:216-266.  qkv rows [M][ld_qkv]: q heads at column 0, k heads at Hq*D, v heads at
 * (Hq+Hkv)*D.  nw = [q_norm(D) | k_norm(D)] or NULL (no q/k RMSNorm).  Rotated q goes to
 * q_out[M][ld_q]; rotated k and raw v go to kc/vc rows pos0..pos0+M-1 of layout
 * [cap][Hkv][D].  eps is the RMSNorm epsilon (reference: 1e-5). */
void p2p_or_qk_prep_h(int hq, int hkv, int d, float eps, const uint16_t* qkv, int64_t ld_qkv,
                      const uint16_t* nw, const uint16_t* rope, uint16_t* q_out, int64_t ld_q,
                      uint16_t* kc, uint16_t* vc, int pos0, int m_tokens);
void p2p_or_qk_prep_f(int hq, int hkv, int d, float eps, const float* qkv, int64_t ld_qkv,
                      const float* nw, const float* rope, float* q_out, int64_t ld_q, float* kc,
                      float* vc, int pos0, int m_tokens);

/* kernels.js:268-319.  Token m (position pos0+m) of head h attends cache keys 0..pos0+m of kv
 * head h/(Hq/Hkv), 128-key chunks, running max seeded at -3e38, out = f16(acc/l).
 * scale multiplies f32(q) (reference: 0.125). */
void p2p_or_attn_h(int hq, int hkv, int d, float scale, const uint16_t* q, int64_t ld_q,
                   const uint16_t* kc, const uint16_t* vc, uint16_t* out, int64_t ld_o,
                   int pos0, int m_tokens);
void p2p_or_attn_f(int hq, int hkv, int d, float scale, const float* q, int64_t ld_q,
                   const float* kc, const float* vc, float* out, int64_t ld_o, int pos0,
                   int m_tokens);

/* Ragged batched decode: sequence i has its cache at token row offsets[i] of kc/vc
 * ([rows][Hkv][D]), attends keys 0..past[i] (its past plus the new token already stored at
 * row offsets[i]+past[i]); q/out rows [nseq][ld].  Each sequence is exactly
 * p2p_or_attn_h with pos0 = past[i], M = 1 on its own cache slice. */
void p2p_or_attn_ragged_h(int hq, int hkv, int d, float scale, const uint16_t* q, int64_t ld_q,
                          const uint16_t* kc, const uint16_t* vc, const int64_t* offsets,
                          const int32_t* past, int nseq, uint16_t* out, int64_t ld_o);

/* kernels.js:22-68 (GEMV, MatMulNBits 4-bit weights, block 32, zero points): the QKV and
 * o_proj projections around the attention path (engine.js:202-204, :224) for one token. */
void p2p_or_gemv_q4(int k, int n_rows, const uint16_t* x, const uint32_t* wq, const uint16_t* sc,
                    const uint32_t* zp, uint16_t* y, int64_t y_off);
void p2p_or_gemm_q4(int m_rows, int k, int n_rows, const uint16_t* x, const uint32_t* wq,
                    const uint16_t* sc, const uint32_t* zp, uint16_t* y, int64_t y_stride,
                    int64_t y_off);
/* The int8 KV cache (the reference bundle's GroupQueryAttention int8 cache: quantise
 * clamp(roundeven(x / scale), -128, 127), dequantise f32(q) * scale, scale per tensor or per
 * (kv head, dim) channel): conversion of f16 rows, and ATTN (kernels.js:268-319) per sequence
 * over int8 cache slices, as p2p_or_attn_ragged_h. */
void p2p_or_quantize_q8(const uint16_t* src, int8_t* dst, int64_t rows, int hkv, int d,
                        const float* scale, int per_channel);
void p2p_or_attn_ragged_q8(int hq, int hkv, int d, float scale, const uint16_t* q, int64_t ld_q,
                           const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                           int per_channel, const int64_t* offsets, const int32_t* past,
                           int nseq, uint16_t* out, int64_t ld_o);
/* vision-kernels.js:176-258.  Bidirectional MHA over S tokens per image, 64-key chunks, first
 * chunk initialises the running max, out = f16(acc/sum).  q/k/v/out are [B][S][ld] with head
 * h at column h*D. */
void p2p_or_vision_attn_h(int nh, int d, float scale, int batch, int s_tokens,
                          const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          uint16_t* out, int64_t ld);

/* Float64 evaluation of softmax(q k^T * scale) v for one (head, token) row set, used to bound
 * the restatement's own rounding error.  Same layouts as p2p_or_attn_h; causal over the
 * cache; no f16 rounding of the output. */
void p2p_or_attn_exact(int hq, int hkv, int d, double scale, const uint16_t* q, int64_t ld_q,
                       const uint16_t* kc, const uint16_t* vc, double* out, int64_t ld_o,
                       int pos0, int m_tokens);

/* kernels.js:362-399: greedy argmax over v f16 logits (ties to the smaller index; values not
 * above -3e38 and NaN never win, index 0 if none does), stored in tok[0] and out_tok[mt[2]],
 * then mt[2] (step) and mt[0] (position) advance by one. */
void p2p_or_argmax_h(const uint16_t* logits, uint32_t v, uint32_t* tok, uint32_t* mt,
                     uint32_t* out_tok);

/* OpenMP threads the parallel loops may use (0 = library default). Returns the count used. */
int p2p_or_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
