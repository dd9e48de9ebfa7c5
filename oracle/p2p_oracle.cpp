// p2p_oracle.cpp -- CPU restatement of the reference attention path (TEST INFRASTRUCTURE ONLY).
//
// Checker and timed CPU baseline for the CUDA library; nothing in the product path links or
// loads it.  Each routine cites the reference lines it follows.  Build flags matter:
// -O2 -ffp-contract=off (no FMA contraction, so every multiply and add rounds like the
// shader's separate f32 operations).  OpenMP parallelises over the shader's workgroup grid
// (head, token), which does not change any per-row arithmetic.
#include "p2p_oracle.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// ---- f16 <-> f32 -----------------------------------------------------------------------
// engine.js:28-50 (toHalfBits): sign, rebias the exponent, round the dropped mantissa bits to
// nearest even; exponents below the normal range go through the subnormal shift; NaN keeps a
// quiet payload bit; overflow saturates to infinity.
inline uint16_t f32_to_f16(float v) {
  uint32_t x;
  std::memcpy(&x, &v, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t e = int32_t((x >> 23) & 0xffu) - 127 + 15;
  uint32_t m = x & 0x7fffffu;
  if (((x >> 23) & 0xffu) == 0xffu) return uint16_t(sign | 0x7c00u | (m ? 0x200u : 0u));
  if (e >= 31) return uint16_t(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return uint16_t(sign);
    m |= 0x800000u;
    const int shift = 14 - e;
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return uint16_t(sign | h);
  }
  uint32_t h = (uint32_t(e) << 10) | (m >> 13);
  const uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return uint16_t(sign | h);
}

// engine.js:331-345 (the h2f table): exact widening of binary16.
inline float f16_to_f32(uint16_t h) {
  const uint32_t s = uint32_t(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 31u;
  const uint32_t m = h & 1023u;
  if (e == 0) {
    const float mag = std::ldexp(float(m), -24);  // 2^-14 * m/1024, exact
    return (h & 0x8000u) ? -mag : mag;
  }
  uint32_t bits;
  if (e == 31) bits = s | 0x7f800000u | (m << 13);
  else bits = s | ((e + 112u) << 23) | (m << 13);
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// Storage policies: Half keeps the shader's f16 buffers and rounding points; Flt stores f32
// and turns every f16() rounding point into the identity.
struct Half {
  using T = uint16_t;
  static inline float ld(T x) { return f16_to_f32(x); }
  static inline T st(float x) { return f32_to_f16(x); }
  static inline float rnd(float x) { return f16_to_f32(f32_to_f16(x)); }
};
struct Flt {
  using T = float;
  static inline float ld(T x) { return x; }
  static inline T st(float x) { return x; }
  static inline float rnd(float x) { return x; }
};

// kernels.js:216-266.  One "workgroup" per (unit, token): units [0,Hq) are q heads, [Hq,Hq+Hkv)
// k heads, [Hq+Hkv, Hq+2Hkv) v heads (copy only).  The sum of squares uses the shader's shared
// memory tree (stride D/2, D/4, ..., 1) so the f32 rounding matches.
template <class P>
void qk_prep(int hq, int hkv, int d, float eps, const typename P::T* qkv, int64_t ld_qkv,
             const typename P::T* nw, const typename P::T* rope, typename P::T* q_out,
             int64_t ld_q, typename P::T* kc, typename P::T* vc, int pos0, int m_tokens) {
  const int units = hq + 2 * hkv;
  const int half = d / 2;
#pragma omp parallel for collapse(2) schedule(static)
  for (int m = 0; m < m_tokens; ++m) {
    for (int unit = 0; unit < units; ++unit) {
      const int64_t pos = int64_t(pos0) + m;
      const typename P::T* row = qkv + int64_t(m) * ld_qkv;
      if (unit >= hq + hkv) {  // kernels.js:237-241 -- v heads: raw copy into the cache
        const int kh = unit - hq - hkv;
        for (int e = 0; e < d; ++e)
          vc[(pos * hkv + kh) * d + e] = row[int64_t(hq + hkv) * d + int64_t(kh) * d + e];
        continue;
      }
      const bool isq = unit < hq;
      const int64_t off = isq ? int64_t(unit) * d : int64_t(hq) * d + int64_t(unit - hq) * d;
      std::vector<float> v(d), red(d), nv(d);
      for (int e = 0; e < d; ++e) {
        v[e] = P::ld(row[off + e]);
        red[e] = v[e] * v[e];
      }
      if (nw) {
        for (int s = d / 2; s > 0; s >>= 1)  // kernels.js:248-251
          for (int e = 0; e < s; ++e) red[e] += red[e + s];
        const float inv = 1.0f / std::sqrt(red[0] / float(d) + eps);  // kernels.js:252
        for (int e = 0; e < d; ++e) {
          const float w = P::ld(nw[isq ? e : d + e]);          // kernels.js:253-254
          nv[e] = P::rnd(v[e] * inv * w);                      // kernels.js:255
        }
      } else {
        for (int e = 0; e < d; ++e) nv[e] = v[e];  // no q/k norm: the f16 input is unchanged
      }
      for (int e = 0; e < d; ++e) {  // kernels.js:257-264 -- rotate-half RoPE
        const int i = e % half;
        const float cs = P::ld(rope[pos * d + i]);
        const float sn = P::ld(rope[pos * d + half + i]);
        float r;
        if (e < half) r = nv[e] * cs - nv[e + half] * sn;
        else r = nv[e] * cs + nv[e - half] * sn;
        if (isq) q_out[int64_t(m) * ld_q + int64_t(unit) * d + e] = P::st(r);
        else kc[(pos * hkv + (unit - hq)) * d + e] = P::st(r);
      }
    }
  }
}

// kernels.js:268-319 for one (head, token): 128-key chunks; within a chunk every lane computes
// its score, the chunk max includes the -3e38 fillers, running sum and accumulator are
// rescaled by exp(old_max - new_max) and then the chunk's keys are added in order.
template <class P>
void attn_row(int hkv, int d, int group, float scale, const typename P::T* qrow,
              const typename P::T* kc, const typename P::T* vc, int h, int64_t pos,
              typename P::T* orow) {
  constexpr int CH = 128;
  const int kh = h / group;
  float qs[256];
  float sc[CH];
  std::vector<float> acc(d, 0.0f);
  for (int e = 0; e < d; ++e) qs[e] = P::ld(qrow[int64_t(h) * d + e]) * scale;  // :283
  float rm = -3.0e38f;
  float rl = 0.0f;
  for (int64_t j0 = 0; j0 <= pos; j0 += CH) {  // :288
    for (int t = 0; t < CH; ++t) {             // :289-297
      const int64_t j = j0 + t;
      float s = -3.0e38f;
      if (j <= pos) {
        float dot = 0.0f;
        const typename P::T* kr = kc + (j * hkv + kh) * d;
        for (int e = 0; e < d; ++e) dot += qs[e] * P::ld(kr[e]);
        s = dot;
      }
      sc[t] = s;
    }
    float cm = -3.0e38f;
    for (int t = 0; t < CH; ++t) cm = std::fmax(cm, sc[t]);  // :299-300
    const float nm = std::fmax(rm, cm);                       // :301
    const float f = std::exp(rm - nm);                        // :302
    rl = rl * f;
    for (int e = 0; e < d; ++e) acc[e] = acc[e] * f;
    for (int t = 0; t < CH; ++t) {  // :305-312
      const int64_t j2 = j0 + t;
      if (j2 > pos) break;
      const float p = std::exp(sc[t] - nm);
      rl += p;
      const typename P::T* vr = vc + (j2 * hkv + kh) * d;
      for (int e = 0; e < d; ++e) acc[e] += p * P::ld(vr[e]);
    }
    rm = nm;
  }
  for (int e = 0; e < d; ++e) orow[int64_t(h) * d + e] = P::st(acc[e] / rl);  // :317
}

template <class P>
void attn(int hq, int hkv, int d, float scale, const typename P::T* q, int64_t ld_q,
          const typename P::T* kc, const typename P::T* vc, typename P::T* out, int64_t ld_o,
          int pos0, int m_tokens) {
  const int group = hq / hkv;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int m = 0; m < m_tokens; ++m)
    for (int h = 0; h < hq; ++h)
      attn_row<P>(hkv, d, group, scale, q + int64_t(m) * ld_q, kc, vc, h, int64_t(pos0) + m,
                  out + int64_t(m) * ld_o);
}

}  // namespace

// The int8 KV cache of the reference bundle's GroupQueryAttention kernels
// (public/kernels/megakernel.json, com.microsoft.GroupQueryAttention): gqa-present.wgsl.jinja
// (bits == 8) appends q = i32(clamp(round(x / scale), QMIN = -128, QMAX = 127)) with WGSL's
// round() (to nearest even) and scale = k_scale[perChannel ? hk*HEAD_DIM + d : 0];
// attn-flash-decode-splitk.wgsl.jinja reads f32(q) * scale (load_key4 / load_value4).
inline int8_t quantize_q8(float x, float scale) {
  float q = std::nearbyint(x / scale);  // default rounding mode: to nearest even
  q = std::fmin(std::fmax(q, -128.0f), 127.0f);
  return static_cast<int8_t>(q);
}

// ATTN (kernels.js:268-319, the loop of attn_row) over an int8 cache: every key and value
// element is dequantised to f32(q) * scale where the f16 shader converts f32(k).
void attn_row_q8(int hkv, int d, int group, float scale, const uint16_t* qrow,
                 const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                 int per_channel, int h, int64_t pos, uint16_t* orow) {
  constexpr int CH = 128;
  const int kh = h / group;
  float qs[256];
  float sc[CH];
  std::vector<float> acc(d, 0.0f);
  auto kscale = [&](int e) { return per_channel ? ks[kh * d + e] : ks[0]; };
  auto vscale = [&](int e) { return per_channel ? vs[kh * d + e] : vs[0]; };
  for (int e = 0; e < d; ++e) qs[e] = f16_to_f32(qrow[int64_t(h) * d + e]) * scale;
  float rm = -3.0e38f;
  float rl = 0.0f;
  for (int64_t j0 = 0; j0 <= pos; j0 += CH) {
    for (int t = 0; t < CH; ++t) {
      const int64_t j = j0 + t;
      float s = -3.0e38f;
      if (j <= pos) {
        float dot = 0.0f;
        const int8_t* kr = kc + (j * hkv + kh) * d;
        for (int e = 0; e < d; ++e) dot += qs[e] * (float(kr[e]) * kscale(e));
        s = dot;
      }
      sc[t] = s;
    }
    float cm = -3.0e38f;
    for (int t = 0; t < CH; ++t) cm = std::fmax(cm, sc[t]);
    const float nm = std::fmax(rm, cm);
    const float f = std::exp(rm - nm);
    rl = rl * f;
    for (int e = 0; e < d; ++e) acc[e] = acc[e] * f;
    for (int t = 0; t < CH; ++t) {
      const int64_t j2 = j0 + t;
      if (j2 > pos) break;
      const float p = std::exp(sc[t] - nm);
      rl += p;
      const int8_t* vr = vc + (j2 * hkv + kh) * d;
      for (int e = 0; e < d; ++e) acc[e] += p * (float(vr[e]) * vscale(e));
    }
    rm = nm;
  }
  for (int e = 0; e < d; ++e) orow[int64_t(h) * d + e] = f32_to_f16(acc[e] / rl);
}

extern "C" {

uint16_t p2p_or_f32_to_f16(float v) { return f32_to_f16(v); }
float p2p_or_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

void p2p_or_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) dst[i] = f32_to_f16(src[i]);
}
void p2p_or_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) dst[i] = f16_to_f32(src[i]);
}

// engine.js:60-71.
void p2p_or_rope_table(int max_ctx, int d, double theta, uint16_t* out) {
  const int half = d / 2;
#pragma omp parallel for schedule(static)
  for (int p = 0; p < max_ctx; ++p) {
    for (int i = 0; i < half; ++i) {
      const double ang = double(p) * std::pow(theta, double(-i) / double(half));
      out[int64_t(p) * d + i] = f32_to_f16(float(std::cos(ang)));
      out[int64_t(p) * d + half + i] = f32_to_f16(float(std::sin(ang)));
    }
  }
}

void p2p_or_rope_table_f32(int max_ctx, int d, double theta, float* out) {
  const int half = d / 2;
#pragma omp parallel for schedule(static)
  for (int p = 0; p < max_ctx; ++p) {
    for (int i = 0; i < half; ++i) {
      const double ang = double(p) * std::pow(theta, double(-i) / double(half));
      out[int64_t(p) * d + i] = float(std::cos(ang));
      out[int64_t(p) * d + half + i] = float(std::sin(ang));
    }
  }
}

void p2p_or_qk_prep_h(int hq, int hkv, int d, float eps, const uint16_t* qkv, int64_t ld_qkv,
                      const uint16_t* nw, const uint16_t* rope, uint16_t* q_out, int64_t ld_q,
                      uint16_t* kc, uint16_t* vc, int pos0, int m_tokens) {
  qk_prep<Half>(hq, hkv, d, eps, qkv, ld_qkv, nw, rope, q_out, ld_q, kc, vc, pos0, m_tokens);
}
void p2p_or_qk_prep_f(int hq, int hkv, int d, float eps, const float* qkv, int64_t ld_qkv,
                      const float* nw, const float* rope, float* q_out, int64_t ld_q, float* kc,
                      float* vc, int pos0, int m_tokens) {
  qk_prep<Flt>(hq, hkv, d, eps, qkv, ld_qkv, nw, rope, q_out, ld_q, kc, vc, pos0, m_tokens);
}

void p2p_or_attn_h(int hq, int hkv, int d, float scale, const uint16_t* q, int64_t ld_q,
                   const uint16_t* kc, const uint16_t* vc, uint16_t* out, int64_t ld_o,
                   int pos0, int m_tokens) {
  attn<Half>(hq, hkv, d, scale, q, ld_q, kc, vc, out, ld_o, pos0, m_tokens);
}
void p2p_or_attn_f(int hq, int hkv, int d, float scale, const float* q, int64_t ld_q,
                   const float* kc, const float* vc, float* out, int64_t ld_o, int pos0,
                   int m_tokens) {
  attn<Flt>(hq, hkv, d, scale, q, ld_q, kc, vc, out, ld_o, pos0, m_tokens);
}

// kernels.js:22-68 (GEMV, ONNX MatMulNBits bits=4 block_size=32 with zero points,
// kernels.js:4-9): y[y_off + n] = f16(sum_k x[k] * W[n][k]).  Row n is one workgroup
// subgroup of 32 lanes: lane l walks words w = l, l+32, ... of the row (8 nibbles each,
// element 8w+i is nibble i), a = sum_i f32(x[8w+i]) * (q_i - zp) in order, acc += a * scale,
// then the shader's shared-memory tree over the 32 lanes (red[l] += red[l+s], s = 16..1).
void p2p_or_gemv_q4(int k, int n_rows, const uint16_t* x, const uint32_t* wq, const uint16_t* sc,
                    const uint32_t* zp, uint16_t* y, int64_t y_off) {
  const int nb = k / 32, zr = (nb + 1) / 2, wpr = k / 8;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < n_rows; ++n) {
    float red[32];
    for (int lane = 0; lane < 32; ++lane) {
      float acc = 0.0f;
      for (int w = lane; w < wpr; w += 32) {  // kernels.js:46-59
        const uint32_t word = wq[int64_t(n) * wpr + w];
        const int blk = w >> 2;
        const float s = f16_to_f32(sc[int64_t(n) * nb + blk]);
        const int64_t zi = int64_t(n) * zr + (blk >> 1);
        const uint32_t zb = (zp[zi >> 2] >> ((zi & 3) * 8)) & 255u;     // kernels.js:16-19
        const float z = float((zb >> ((blk & 1) * 4)) & 15u);
        float a = 0.0f;
        for (int i = 0; i < 8; ++i) {
          const float q = float((word >> (i * 4)) & 15u);
          a += f16_to_f32(x[w * 8 + i]) * (q - z);
        }
        acc += a * s;
      }
      red[lane] = acc;
    }
    for (int s = 16; s > 0; s >>= 1)  // kernels.js:61-65
      for (int l = 0; l < s; ++l) red[l] += red[l + s];
    y[y_off + n] = f32_to_f16(red[0]);  // kernels.js:66
  }
}

// kernels.js:70-145 (GEMM, the prompt-chunk form of the same MatMulNBits projection):
// Y[m * y_stride + y_off + n] = f16(sum_k f32(X[m][k]) * W[n][k]) with the dequantised weight
// W[n][k] = (f32(q) - zp) * scale rounded to f32 first (kernels.js:116-121), and the sum taken
// over k in increasing order, one product and one addition at a time (kernels.js:125-133: every
// thread adds its 32 k of a block in order, block after block).
void p2p_or_gemm_q4(int m_rows, int k, int n_rows, const uint16_t* x, const uint32_t* wq,
                    const uint16_t* sc, const uint32_t* zp, uint16_t* y, int64_t y_stride,
                    int64_t y_off) {
  const int nb = k / 32, zr = (nb + 1) / 2, wpr = k / 8;
  std::vector<float> wd(size_t(n_rows) * k);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < n_rows; ++n)
    for (int kb = 0; kb < nb; ++kb) {
      const float s = f16_to_f32(sc[int64_t(n) * nb + kb]);
      const int64_t zi = int64_t(n) * zr + (kb >> 1);
      const uint32_t zb = (zp[zi >> 2] >> ((zi & 3) * 8)) & 255u;  // kernels.js:16-19
      const float z = float((zb >> ((kb & 1) * 4)) & 15u);
      for (int wi = 0; wi < 4; ++wi) {
        const uint32_t word = wq[int64_t(n) * wpr + kb * 4 + wi];
        for (int i = 0; i < 8; ++i)
          wd[size_t(n) * k + kb * 32 + wi * 8 + i] = (float((word >> (i * 4)) & 15u) - z) * s;
      }
    }
#pragma omp parallel for schedule(static)
  for (int m = 0; m < m_rows; ++m)
    for (int n = 0; n < n_rows; ++n) {
      float c = 0.0f;
      const float* w = wd.data() + size_t(n) * k;
      for (int kk = 0; kk < k; ++kk) c += f16_to_f32(x[int64_t(m) * k + kk]) * w[kk];
      y[int64_t(m) * y_stride + y_off + n] = f32_to_f16(c);
    }
}

void p2p_or_quantize_q8(const uint16_t* src, int8_t* dst, int64_t rows, int hkv, int d,
                        const float* scale, int per_channel) {
  const int64_t chan = int64_t(hkv) * d;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < chan; ++c)
      dst[r * chan + c] = quantize_q8(f16_to_f32(src[r * chan + c]), per_channel ? scale[c] : scale[0]);
}

void p2p_or_attn_ragged_q8(int hq, int hkv, int d, float scale, const uint16_t* q, int64_t ld_q,
                           const int8_t* kc, const int8_t* vc, const float* ks, const float* vs,
                           int per_channel, const int64_t* offsets, const int32_t* past,
                           int nseq, uint16_t* out, int64_t ld_o) {
  const int group = hq / hkv;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int i = 0; i < nseq; ++i)
    for (int h = 0; h < hq; ++h) {
      const int64_t base = offsets[i] * hkv * d;
      attn_row_q8(hkv, d, group, scale, q + int64_t(i) * ld_q, kc + base, vc + base, ks, vs,
                  per_channel, h, past[i], out + int64_t(i) * ld_o);
    }
}

void p2p_or_attn_ragged_h(int hq, int hkv, int d, float scale, const uint16_t* q, int64_t ld_q,
                          const uint16_t* kc, const uint16_t* vc, const int64_t* offsets,
                          const int32_t* past, int nseq, uint16_t* out, int64_t ld_o) {
  const int group = hq / hkv;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int i = 0; i < nseq; ++i)
    for (int h = 0; h < hq; ++h) {
      const int64_t base = offsets[i] * hkv * d;
      attn_row<Half>(hkv, d, group, scale, q + int64_t(i) * ld_q, kc + base, vc + base, h,
                     past[i], out + int64_t(i) * ld_o);
    }
}

// vision-kernels.js:176-258 for every (image, head, token).
void p2p_or_vision_attn_h(int nh, int d, float scale, int batch, int s_tokens,
                          const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          uint16_t* out, int64_t ld) {
  constexpr int CH = 64;
#pragma omp parallel for collapse(3) schedule(dynamic, 4)
  for (int b = 0; b < batch; ++b)
    for (int m = 0; m < s_tokens; ++m)
      for (int h = 0; h < nh; ++h) {
        const int64_t img = int64_t(b) * s_tokens * ld;
        const uint16_t* qb = q + img;
        const uint16_t* kb = k + img;
        const uint16_t* vb = v + img;
        const int64_t q_base = int64_t(m) * ld + int64_t(h) * d;  // :198
        float qs[256];
        float sc[CH];
        std::vector<float> acc(d, 0.0f);
        for (int e = 0; e < d; ++e) qs[e] = f16_to_f32(qb[q_base + e]) * scale;  // :199
        float running_max = -1e30f;
        float running_sum = 0.0f;
        for (int j0 = 0; j0 < s_tokens; j0 += CH) {  // :206
          for (int t = 0; t < CH; ++t) {              // :207-217
            const int j = j0 + t;
            float dot = -1e30f;
            if (j < s_tokens) {
              const int64_t k_base = int64_t(j) * ld + int64_t(h) * d;
              float sum_d = 0.0f;
              for (int e = 0; e < d; ++e) sum_d += qs[e] * f16_to_f32(kb[k_base + e]);
              dot = sum_d;
            }
            sc[t] = dot;
          }
          float chunk_max = sc[0];  // :220-223
          for (int t = 1; t < CH; ++t) chunk_max = std::fmax(chunk_max, sc[t]);
          float mx;
          if (j0 == 0) {  // :225-235
            running_max = chunk_max;
            mx = chunk_max;
          } else {  // :236-241
            const float new_max = std::fmax(running_max, chunk_max);
            const float alpha = std::exp(running_max - new_max);
            running_sum = running_sum * alpha;
            for (int e = 0; e < d; ++e) acc[e] = acc[e] * alpha;
            mx = new_max;
          }
          for (int t = 0; t < CH; ++t) {  // :227-234 / :242-250
            const int j2 = j0 + t;
            if (j2 < s_tokens) {
              const float p = std::exp(sc[t] - mx);
              running_sum += p;
              const int64_t v_base = int64_t(j2) * ld + int64_t(h) * d;
              for (int e = 0; e < d; ++e) acc[e] += p * f16_to_f32(vb[v_base + e]);
            }
          }
          running_max = mx;  // :251
        }
        for (int e = 0; e < d; ++e)  // :256
          out[img + q_base + e] = f32_to_f16(acc[e] / running_sum);
      }
}

void p2p_or_attn_exact(int hq, int hkv, int d, double scale, const uint16_t* q, int64_t ld_q,
                       const uint16_t* kc, const uint16_t* vc, double* out, int64_t ld_o,
                       int pos0, int m_tokens) {
  const int group = hq / hkv;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int m = 0; m < m_tokens; ++m)
    for (int h = 0; h < hq; ++h) {
      const int64_t pos = int64_t(pos0) + m;
      const int kh = h / group;
      std::vector<double> s(size_t(pos + 1));
      double mx = -INFINITY;
      for (int64_t j = 0; j <= pos; ++j) {
        double dot = 0.0;
        for (int e = 0; e < d; ++e)
          dot += double(f16_to_f32(q[int64_t(m) * ld_q + int64_t(h) * d + e])) *
                 double(f16_to_f32(kc[(j * hkv + kh) * d + e]));
        s[size_t(j)] = dot * scale;
        mx = std::fmax(mx, s[size_t(j)]);
      }
      double l = 0.0;
      std::vector<double> acc(d, 0.0);
      for (int64_t j = 0; j <= pos; ++j) {
        const double p = std::exp(s[size_t(j)] - mx);
        l += p;
        for (int e = 0; e < d; ++e) acc[e] += p * double(f16_to_f32(vc[(j * hkv + kh) * d + e]));
      }
      for (int e = 0; e < d; ++e) out[int64_t(m) * ld_o + int64_t(h) * d + e] = acc[e] / l;
    }
}

int p2p_or_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}


// kernels.js:362-399 (ARGMAX), dispatched as one workgroup of 256 (engine.js:239-240, 265-266):
// invocation t scans logits[t], logits[t+256], ... keeping the first strictly larger value
// (seeded -3e38 and index 0); the workgroup tree over 128, 64, ..., 1 keeps the larger value,
// ties to the smaller index; invocation 0 stores the token in tok[0] and outTok[mt[2]] and
// advances mt[2] (step) and mt[0] (position) by one.
void p2p_or_argmax_h(const uint16_t* logits, uint32_t v, uint32_t* tok, uint32_t* mt,
                     uint32_t* out_tok) {
  float bv[256];
  uint32_t bi[256];
  for (uint32_t t = 0; t < 256u; ++t) {
    float best = -3.0e38f;
    uint32_t bidx = 0u;
    for (uint32_t i = t; i < v; i += 256u) {
      const float x = p2p_or_f16_to_f32(logits[i]);
      if (x > best) {
        best = x;
        bidx = i;
      }
    }
    bv[t] = best;
    bi[t] = bidx;
  }
  for (uint32_t s = 128u; s > 0u; s >>= 1u)
    for (uint32_t t = 0; t < s; ++t) {
      const float ov = bv[t + s];
      const uint32_t oi = bi[t + s];
      if (ov > bv[t] || (ov == bv[t] && oi < bi[t])) {
        bv[t] = ov;
        bi[t] = oi;
      }
    }
  tok[0] = bi[0];
  out_tok[mt[2]] = bi[0];
  mt[2] = mt[2] + 1u;
  mt[0] = mt[0] + 1u;
}

}  // extern "C"
