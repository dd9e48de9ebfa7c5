// decode.cu -- split-KV decode attention for sm_100a (ATTN at M = 1,
// src/scripts/lfm-engine/kernels.js:268-319, optionally fused with QK_PREP, :216-266).
//
// Grid (splits, Hkv * head_chunks, Z).  Z is either the attention layers of one decode step
// (all at the same position, engine.js:425-429) or the sequences of a ragged batch.  One CTA
// streams one contiguous key range of ONE kv head and serves up to 4 of its G = Hq/Hkv query
// heads, so for G <= 4 every K/V byte is read from HBM exactly once (the shader reads each kv
// head once per q head, kernels.js:282).
//
// Memory pipeline (both kernels): a cp.async ring of 64-key tiles in shared memory; every
// warp instruction copies four whole 128-byte K (or V) rows with 16-byte copies.
//
// f16 kernel (decode_mma_kernel): each warp owns 16 keys of a tile and runs the two
// contractions on the tensor cores with warp-level mma.sync.m16n8k16 (f16 in, f32 out):
//     S^T[16 keys x 8]   = K[16 x 64] . Q^T[64 x 8]         (the G query heads, zero padded)
//     O^T[64 dims x 8]  += V^T[64 x 16] . P^T[16 x 8]
// K/V fragments come from the ring with ldmatrix (rows XOR-swizzled in 16-byte chunks, so
// the 128-byte rows are bank-conflict free); P^T is the S^T accumulator rounded to f16 and
// transposed in registers with movmatrix.  The softmax runs on the accumulator fragment:
// per-head block max by xor-shuffle over the 8 lanes holding a head's keys, exp2 on the MUFU,
// running max / sum kept per lane.  That is ~4 warp instructions per key instead of ~60 for
// a CUDA-core dot-product formulation, so the kernel is bound by HBM, not by issue.
//
// f32 kernel (decode_simt_kernel, the fp32 storage case): CUDA-core formulation, lane =
// 8*slot + part, each slot of 8 lanes holds one key row, dot products completed with a
// 3-level xor-shuffle, per-slot online softmax.
//
// Both finish the same way: warps merge through shared memory; a CTA whose sequence needs
// more than one split writes its partial (acc, max, sum) to the workspace, and the last CTA
// of the (sequence, head chunk) to arrive -- counted with one atomic -- runs the second pass
// that combines the partials and writes the output, then resets its counter.  Nothing ever
// waits on another CTA.
//
// Cluster form (f16, one decode step over the layers): the splits of one (layer, head chunk)
// are the CTAs of one thread-block cluster (up to 8).  Head g's combine is owned by cluster
// rank g % nsplit; every split pushes its partial for head g straight into the owner's shared
// memory with st.async, which completes bytes on the owner's mbarrier.  The owner waits on
// that mbarrier (bounded), combines and writes the output; every other CTA exits as soon as it
// has pushed.  No workspace, no atomics, no global fences and no cluster barrier at the end.
#include <map>
#include <mutex>
#include <set>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace p2p {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = 4;
constexpr int kStageKeys = 64;  // keys per pipeline stage
constexpr float kNegBig = -1e30f;
constexpr int kPartialStride = kHeadDim + 2;  // acc[64], max, sum

template <class T>
struct Ring {
  static constexpr int kStages = sizeof(T) == 2 ? 4 : 2;
  static constexpr int kTileElems = kStageKeys * kHeadDim;
  static constexpr int kBytes = 2 * kStages * kTileElems * int(sizeof(T));  // K and V
};

// ---- per-sequence view ------------------------------------------------------------------------
// T: element of q / out / rope / norm weights; TC: element of the KV cache (T, or int8_t).
template <class T, class TC>
struct Seq {
  int past;
  const T* qrow;
  const T* nw;
  TC* kc;  // kLayers / kRagged: the sequence's row 0; kPaged: the page pool
  TC* vc;
  T* orow;
  const int32_t* tbl;  // kPaged: the sequence's block-table row
};

template <class T, class TC, int MODE>
__device__ __forceinline__ Seq<T, TC> resolve(const DecodeArgs& a, int z) {
  Seq<T, TC> q;
  q.tbl = nullptr;
  if (MODE == kLayers) {
    const DecodeLayer& L = a.layers[z];
    q.past = a.meta ? int(a.meta[0]) : a.pos_host;
    q.qrow = static_cast<const T*>(L.qkv);
    q.nw = static_cast<const T*>(L.norm_w);
    q.kc = static_cast<TC*>(L.k_cache);
    q.vc = static_cast<TC*>(L.v_cache);
    q.orow = static_cast<T*>(L.out);
  } else {
    q.past = a.past[z];
    q.qrow = static_cast<const T*>(a.qkv) + int64_t(z) * a.ld_qkv;
    q.nw = static_cast<const T*>(a.norm_w);
    const int64_t row0 = MODE == kPaged ? 0 : int64_t(a.offsets[z]) * a.hkv * kHeadDim;
    q.kc = static_cast<TC*>(a.k_cache) + row0;
    q.vc = static_cast<TC*>(a.v_cache) + row0;
    q.orow = static_cast<T*>(a.out) + int64_t(z) * a.ld_o;
    if (MODE == kPaged) q.tbl = a.block_table + int64_t(z) * a.max_blocks;
  }
  return q;
}

// Whether sequence z must be refused before any of its rows is touched: a decode-step
// position at or beyond the cache (kLayers); a ragged entry that is negative, longer than
// max_past (the rope table's bound) or reaching past the cache's kv_cap rows (kRagged); a
// paged sequence with more pages than its block-table row holds or a block-table entry
// outside the kv_cap pages (kPaged; every thread takes part, every CTA of the sequence reads
// the same entries and decides alike).  One CTA per sequence records the refusal in the device
// error word, which p2p_sync reports.
template <int MODE>
__device__ __forceinline__ bool refused(const DecodeArgs& a, int z) {
  bool bad;
  if (MODE == kLayers) {
    const int pos = a.meta ? int(a.meta[0]) : a.pos_host;
    bad = pos < 0 || int64_t(pos) >= a.kv_cap;
  } else if (MODE == kRagged) {
    const int off = a.offsets[z], past = a.past[z];
    bad = off < 0 || past < 0 || past > a.max_past || int64_t(off) + past >= a.kv_cap;
  } else {
    const int past = a.past[z];
    bad = past < 0 || past > a.max_past || (past >> a.block_shift) >= a.max_blocks;
    if (!bad) {
      const int32_t* tbl = a.block_table + int64_t(z) * a.max_blocks;
      const int n = (past >> a.block_shift) + 1;
      bool mine = false;
      for (int b = threadIdx.x; b < n; b += blockDim.x) {
        const int32_t pg = tbl[b];
        mine |= pg < 0 || int64_t(pg) >= a.kv_cap;
      }
      bad = __syncthreads_or(mine) != 0;
    }
  }
  if (bad && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
    atomicOr(a.err, kErrPosBeyondCache);
  return bad;
}

// int8 cache: the scale of (kv head kh, dim d) and the quantisation of one value,
// q = clamp(roundeven(x / scale), -128, 127) (the GroupQueryAttention int8 cache append).
__device__ __forceinline__ float kv_scale(const float* sc, int per_channel, int kh, int d) {
  return per_channel ? sc[kh * kHeadDim + d] : sc[0];
}
__device__ __forceinline__ int8_t quantize_q8(float x, float scale) {
  const float q = rintf(__fdiv_rn(x, scale));
  return static_cast<int8_t>(fminf(fmaxf(q, -128.f), 127.f));
}
template <class TC>
__device__ __forceinline__ float cache_f32(TC x) { return to_f32(x); }
template <>
__device__ __forceinline__ float cache_f32<int8_t>(int8_t x) { return float(x); }

// Rotated query heads head0..head0+GC-1 into q_s (times `qscale`), and for the split that
// holds the new token its normed/rotated k and raw v (QK_PREP's k and v units) into
// knew_s/vnew_s and, by head chunk 0, into cache row `new_row` (an int8 cache stores them
// quantised, and knew_s/vnew_s then hold the quantised integers).  Unfused: q is read as given.
// The prologue's inputs in registers, per lane.
struct PrologueIn {
  float cs, sn;   // fused: this lane's rope row entries (lane, lane + 32)
  float x[2][2];  // fused: unit (warp + 4i)'s values at lane and lane + 32; else q_s values
  float w[2][2];  // fused: that unit's norm weights (q and k units)
  float ks[2];    // int8 cache: the key scales that fold into q (per channel) or the one scale
};

// Where the prologue reads its inputs: the global rows, or the CTA's shared-memory copy of
// them (PrologueStage).
template <class T>
struct PrologueSrc {
  const T* q;       // the split's GC q heads, 64 values each, consecutive
  const T* k;       // fused: the new token's k head and v head (64 values each)
  const T* v;
  const T* nw;      // [q norm | k norm] or nullptr
  const T* rope;    // fused: the position's rope row
  const float* ks;  // int8 caches: the kv head's 64 key scales, or the one scale
};

template <class T, class TC>
__device__ __forceinline__ PrologueSrc<T> prologue_global(const DecodeArgs& a,
                                                          const Seq<T, TC>& sq, int kh,
                                                          int head0) {
  constexpr int D = kHeadDim;
  PrologueSrc<T> src;
  src.q = sq.qrow + int64_t(head0) * D;
  src.k = sq.qrow + int64_t(a.hq + kh) * D;
  src.v = sq.qrow + int64_t(a.hq + a.hkv + kh) * D;
  src.nw = sq.nw;
  src.rope = static_cast<const T*>(a.rope) + int64_t(sq.past) * D;
  src.ks = a.k_scale ? a.k_scale + (a.scale_per_channel ? kh * D : 0) : nullptr;
  return src;
}

// The prologue's inputs copied into shared memory as the CTA's first cp.async group, ahead
// of the K/V tiles: loads issued behind a CTA's tile burst return only after it (about 2 us
// with three CTAs per SM), and the prologue would then hold up the ring's refills.  16-byte
// pieces: the q heads, k and v (fused, new token), the norm weights, the rope row, the key
// scales (int8 per channel); the host enables it when every source is 16-byte aligned.
// Layout (bytes): q GC*128 | k 128 | v 128 | nw 256 | rope 128 | ks 256 = GC*128 + 896.
template <int GC>
constexpr int prologue_stage_bytes() {
  return GC * 128 + 896;
}

template <class T, class TC, int GC, bool FUSED>
__device__ __forceinline__ PrologueSrc<T> prologue_stage(const DecodeArgs& a,
                                                         const PrologueSrc<T>& g,
                                                         bool has_new, bool do_q,
                                                         unsigned char* stage) {
  constexpr bool kQ8 = sizeof(TC) == 1;
  const int tid = threadIdx.x;
  const int c = tid;  // one 16-byte piece per thread (at most GC*8 + 56 <= 88 pieces)
  const void* from = nullptr;
  int at = 0;
  if (c < GC * 8) {
    if (do_q) from = g.q + c * 8, at = c * 16;
  } else if (c < GC * 8 + 16) {
    const int e = c - GC * 8;
    if (FUSED && has_new) from = (e < 8 ? g.k : g.v) + (e & 7) * 8, at = GC * 128 + e * 16;
  } else if (c < GC * 8 + 32) {
    const int e = c - GC * 8 - 16;
    if (g.nw != nullptr) from = g.nw + e * 8, at = GC * 128 + 256 + e * 16;
  } else if (c < GC * 8 + 40) {
    const int e = c - GC * 8 - 32;
    if (FUSED) from = g.rope + e * 8, at = GC * 128 + 512 + e * 16;
  } else if (c < GC * 8 + 56) {
    const int e = c - GC * 8 - 40;
    if (kQ8 && a.scale_per_channel) from = g.ks + e * 4, at = GC * 128 + 640 + e * 16;
  }
  if (from != nullptr) cp_async16(stage + at, from, true);
  cp_async_commit();
  PrologueSrc<T> s;
  s.q = reinterpret_cast<const T*>(stage);
  s.k = reinterpret_cast<const T*>(stage + GC * 128);
  s.v = reinterpret_cast<const T*>(stage + GC * 128 + 128);
  s.nw = g.nw != nullptr ? reinterpret_cast<const T*>(stage + GC * 128 + 256) : nullptr;
  s.rope = reinterpret_cast<const T*>(stage + GC * 128 + 512);
  s.ks = (kQ8 && a.scale_per_channel) ? reinterpret_cast<const float*>(stage + GC * 128 + 640)
                                      : g.ks;
  return s;
}

template <class T, class TC, int GC, bool FUSED>
__device__ __forceinline__ PrologueIn prologue_load(const DecodeArgs& a, const PrologueSrc<T>& src,
                                                    bool has_new, bool do_q) {
  constexpr int D = kHeadDim;
  constexpr bool kQ8 = sizeof(TC) == 1;
  static_assert(kWarps == 4 && GC <= 4, "the warp's units are warp and warp + 4");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  PrologueIn in{};
  if (FUSED) {
    in.cs = to_f32(src.rope[lane]);
    in.sn = to_f32(src.rope[32 + lane]);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int u = warp + i * kWarps;
      if (u >= GC + 2 || (u < GC ? !do_q : !has_new)) continue;
      const T* x = u < GC ? src.q + u * D : (u == GC ? src.k : src.v);
      in.x[i][0] = to_f32(x[lane]);
      in.x[i][1] = to_f32(x[lane + 32]);
      if (src.nw != nullptr && u <= GC) {  // q units take the q norm, the k unit the k norm
        const T* w = src.nw + (u < GC ? 0 : D);
        in.w[i][0] = to_f32(w[lane]);
        in.w[i][1] = to_f32(w[lane + 32]);
      }
    }
  } else if (do_q) {
#pragma unroll
    for (int i = 0; i < 2; ++i)
      if (tid + i * kThreads < GC * D) in.x[i][0] = to_f32(src.q[tid + i * kThreads]);
  }
  if constexpr (kQ8) {
    if (a.scale_per_channel) {
#pragma unroll
      for (int i = 0; i < 2; ++i)
        if (tid + i * kThreads < GC * D) in.ks[i] = src.ks[(tid + i * kThreads) % D];
    } else {
      in.ks[0] = src.ks[0];
    }
  }
  return in;
}

// QK_PREP of the split's q heads (and, in the CTA holding the new token, its k and v) from
// the loaded inputs: the normed, rotated q (times qscale) into q_s; k/v into knew_s / vnew_s
// and, for head chunk 0, into cache row new_row (int8 caches: quantised).
template <class T, class TC, int GC, bool FUSED>
__device__ __forceinline__ void prologue(const DecodeArgs& a, const Seq<T, TC>& sq, int kh,
                                         int hc, int head0, bool has_new, int64_t new_row,
                                         float qscale, float (*q_s)[kHeadDim], float* knew_s,
                                         float* vnew_s, const PrologueIn& in, bool do_q = true) {
  constexpr int D = kHeadDim;
  constexpr bool kQ8 = sizeof(TC) == 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (FUSED) {
    const int64_t kv_stride = int64_t(a.hkv) * D;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int u = warp + i * kWarps;
      if (u >= GC + 2 || (u < GC ? !do_q : !has_new)) continue;
      if (u < GC) {  // QK_PREP q unit (kernels.js:255-263), f16 rounding of the stored q
        float r0, r1;
        norm_rope_vals<T>(in.x[i][0], in.x[i][1], in.w[i][0], in.w[i][1], sq.nw != nullptr,
                          a.eps, in.cs, in.sn, r0, r1);
        q_s[u][lane] = round_st<T>(r0) * qscale;
        q_s[u][lane + 32] = round_st<T>(r1) * qscale;
        continue;
      }
      // QK_PREP k unit (normed, rotated) or v unit (raw copy) -> cache row `new_row`
      const bool is_k = u == GC;
      float x0 = in.x[i][0], x1 = in.x[i][1];
      if (is_k) {
        float r0, r1;
        norm_rope_vals<T>(x0, x1, in.w[i][0], in.w[i][1], sq.nw != nullptr, a.eps, in.cs,
                          in.sn, r0, r1);
        x0 = round_st<T>(r0);
        x1 = round_st<T>(r1);
      }
      TC c0, c1;
      if constexpr (kQ8) {
        const float* sc = is_k ? a.k_scale : a.v_scale;
        c0 = quantize_q8(x0, kv_scale(sc, a.scale_per_channel, kh, lane));
        c1 = quantize_q8(x1, kv_scale(sc, a.scale_per_channel, kh, lane + 32));
      } else {
        c0 = from_f32<TC>(x0);
        c1 = from_f32<TC>(x1);
      }
      if (hc == 0) {
        TC* dst = (is_k ? sq.kc : sq.vc) + new_row * kv_stride + kh * D;
        dst[lane] = c0;
        dst[lane + 32] = c1;
      }
      float* dst_s = is_k ? knew_s : vnew_s;
      dst_s[lane] = cache_f32<TC>(c0);
      dst_s[lane + 32] = cache_f32<TC>(c1);
    }
  } else if (do_q) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int e = tid + i * kThreads;
      if (e < GC * D) q_s[e / D][e % D] = in.x[i][0] * qscale;
    }
  }
}

// Cross-warp merge of (red_m, red_l, red_acc) and the split-KV second pass.
template <class T, int GC>
__device__ __forceinline__ void finish(const DecodeArgs& a, T* out_h, int pair, int split,
                                       int nsplit, int ngrid, const float (*red_m)[GC],
                                       const float (*red_l)[GC],
                                       const float (*red_acc)[GC][kHeadDim], int* s_last) {
  constexpr int D = kHeadDim;
  const int tid = threadIdx.x;
  float* part_base = a.partials + int64_t(pair) * ngrid * (GC * kPartialStride);
  for (int idx = tid; idx < GC * D; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float mx = red_m[0][g];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, red_m[w][g]);
    float l = 0.f, ac = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float c = fast_exp2(red_m[w][g] - mx);
      l = fmaf(red_l[w][g], c, l);
      ac = fmaf(red_acc[w][g][d], c, ac);
    }
    if (nsplit == 1) {
      out_h[idx] = from_f32<T>(ac / l);  // kernels.js:317
    } else {
      float* p = part_base + int64_t(split) * (GC * kPartialStride) + g * kPartialStride;
      p[d] = ac;
      if (d == 0) {
        p[D] = mx;
        p[D + 1] = l;
      }
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&a.counters[pair], 1);
    *s_last = (prev == nsplit - 1);
  }
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  for (int idx = tid; idx < GC * D; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    const float* p0 = part_base + g * kPartialStride;
    float mx = kNegBig;
    for (int sp = 0; sp < nsplit; ++sp)
      mx = fmaxf(mx, __ldcg(p0 + int64_t(sp) * (GC * kPartialStride) + D));
    float l = 0.f, ac = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float* p = p0 + int64_t(sp) * (GC * kPartialStride);
      const float c = fast_exp2(__ldcg(p + D) - mx);
      l = fmaf(__ldcg(p + D + 1), c, l);
      ac = fmaf(__ldcg(p + d), c, ac);
    }
    out_h[idx] = from_f32<T>(ac / l);
  }
  if (tid == 0) a.counters[pair] = 0;
}

// ---- cluster push-combine ---------------------------------------------------------------------
constexpr int kMaxCluster = 16;         // non-portable sizes above 8: few (layer, head) rows
constexpr int kPortableCluster = 8;
constexpr int kPushStride = kHeadDim + 4;  // acc[64], max, sum, 2 pad: 17 16-byte chunks
constexpr int kPushChunks = kPushStride / 4;
// receive slots of a cluster of up to `cl` CTAs: ceil(GC / n) * n <= cl for GC <= 4, n <= cl
constexpr int recv_slots(int cl) { return cl > kPortableCluster ? kMaxCluster : kPortableCluster; }
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Address of the same shared-memory variable in cluster CTA `rank` (shared::cluster window).
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}
// 16 bytes into a cluster peer's shared memory; completes 16 bytes of transaction count on the
// peer's mbarrier when they have landed.
__device__ __forceinline__ void st_async16(uint32_t dst, const uint4& v, uint32_t bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, "
      "[%5];" ::"r"(dst),
      "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void recv_bar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void recv_bar_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool recv_bar_try_wait(uint64_t* bar) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar))
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Cluster form of finish().  Split `split` (= cluster rank) of `nsplit` active splits merges
// its warps into stage_s, pushes head g's partial to slot (g / nsplit) * nsplit + split of
// rank g % nsplit, and, if it owns heads, waits for all nsplit partials of each and writes
// them combined.  Splits >= nsplit (empty key ranges) push nothing and own nothing.  Every
// CTA must have called cluster_arrive_relaxed() after recv_bar_init().
template <class T, int GC>
__device__ __forceinline__ void finish_push(const DecodeArgs& a, T* out_h, int split, int nsplit,
                                            const float (*red_m)[GC], const float (*red_l)[GC],
                                            const float (*red_acc)[GC][kHeadDim],
                                            float (*stage_s)[kPushStride],
                                            float (*recv_s)[kPushStride], uint64_t* recv_bar,
                                            bool start_waited) {
  constexpr int D = kHeadDim;
  const int tid = threadIdx.x;
  const bool active = split < nsplit;
  if (active) {
    for (int idx = tid; idx < GC * D; idx += kThreads) {
      const int g = idx / D, d = idx % D;
      float mx = red_m[0][g];
#pragma unroll
      for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, red_m[w][g]);
      float l = 0.f, ac = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float c = fast_exp2(red_m[w][g] - mx);
        l = fmaf(red_l[w][g], c, l);
        ac = fmaf(red_acc[w][g][d], c, ac);
      }
      stage_s[g][d] = ac;
      if (d == 0) {
        stage_s[g][D] = mx;
        stage_s[g][D + 1] = l;
        stage_s[g][D + 2] = 0.f;
        stage_s[g][D + 3] = 0.f;
      }
    }
    __syncthreads();
  }
  if (!start_waited) cluster_wait();  // every rank's receive mbarrier is initialised
  if (!active) return;
  for (int i = tid; i < GC * kPushChunks; i += kThreads) {
    const int g = i / kPushChunks, c = i % kPushChunks;
    const uint32_t owner = uint32_t(g % nsplit);
    const int slot = (g / nsplit) * nsplit + split;
    const uint4 v = *reinterpret_cast<const uint4*>(&stage_s[g][4 * c]);
    st_async16(map_rank(smem_addr(&recv_s[slot][4 * c]), owner), v,
               map_rank(smem_addr(recv_bar), owner));
  }
  // heads owned by this rank: g = split, split + nsplit, ...
  const int owned = split < GC ? (GC - 1 - split) / nsplit + 1 : 0;
  if (owned == 0) return;
  if (tid == 0)
    recv_bar_expect(recv_bar, uint32_t(owned * nsplit * kPushStride * 4 + a.wait_deficit));
  if (!recv_bar_try_wait(recv_bar)) {
    const uint64_t t0 = now_ns();
    while (!recv_bar_try_wait(recv_bar)) {
      if (now_ns() - t0 > kWaitLimitNs) {  // a peer never delivered: report, write nothing
        if (tid == 0) atomicOr(a.err, kErrTimeout);
        return;
      }
    }
  }
  for (int idx = tid; idx < owned * D; idx += kThreads) {
    const int h = idx / D, d = idx % D;
    const float(*src)[kPushStride] = recv_s + h * nsplit;
    float mx = kNegBig;  // the partials are read straight from shared memory (few registers)
    for (int r = 0; r < nsplit; ++r) mx = fmaxf(mx, src[r][D]);
    float lt = 0.f, at = 0.f;
    for (int r = 0; r < nsplit; ++r) {
      const float c = fast_exp2(src[r][D] - mx);
      lt = fmaf(src[r][D + 1], c, lt);
      at = fmaf(src[r][d], c, at);
    }
    out_h[(split + h * nsplit) * D + d] = from_f32<T>(at / lt);  // kernels.js:317
  }
}

// ---- warp-level MMA helpers -------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Byte offset of 16-byte chunk `c` of row `r` in a 64-element f16 tile whose rows are 128
// bytes and whose chunks are XOR-swizzled with the row's low 3 bits.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return uint32_t(r * 128 + ((c ^ (r & 7)) << 4));
}

// int8 caches: per stage a K and a V tile of 64 rows x 64 bytes, 8 stages (the f16 ring's 64
// KB).  Row r's four 16-byte pieces are XOR-swizzled with (r >> 1) & 3, so the eight rows one
// ldmatrix phase reads hit all 32 banks.
struct RingQ8 {
  static constexpr int kStages = 8;
  static constexpr int kTileBytes = kStageKeys * kHeadDim;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kBytes = kStages * kStageBytes;
};
__device__ __forceinline__ uint32_t swz8(int r, int c) {
  return uint32_t(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// Four int8 values (one 32-bit word, dims 4k..4k+3) -> two f16x2 words, exactly: the byte
// x ^ 0x80 under the f16 pattern 0x64xx is 1024 + 128 + x; subtracting 1152 leaves x.
__device__ __forceinline__ void s8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;
  uint32_t l = __byte_perm(x, 0x64646464u, 0x5140);
  uint32_t h = __byte_perm(x, 0x64646464u, 0x7362);
  const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
  const __half2 lh = __hsub2(*reinterpret_cast<const __half2*>(&l), bias);
  const __half2 hh = __hsub2(*reinterpret_cast<const __half2*>(&h), bias);
  lo = *reinterpret_cast<const uint32_t*>(&lh);
  hi = *reinterpret_cast<const uint32_t*>(&hh);
}

// CL: 0 (no cluster: workspace combine) or the largest cluster the instance serves (8 or 16;
// the larger receive buffer of 16 would cost the 8-CTA form its third CTA per SM).
template <int G, bool FUSED, int MODE, int CL, int KVF>
__global__ void __launch_bounds__(kThreads, 3)
    decode_mma_kernel(const __grid_constant__ DecodeArgs a) {
  using T = __half;
  constexpr bool kQ8 = KVF == kKvI8;
  using TC = typename std::conditional<kQ8, int8_t, __half>::type;
  constexpr bool kPg = MODE == kPaged;
  constexpr int D = kHeadDim;
  constexpr int GC = G > 4 ? 4 : G;
  constexpr int NHC = G / GC;
  constexpr int kStages = kQ8 ? RingQ8::kStages : Ring<T>::kStages;
  constexpr int kTile = Ring<T>::kTileElems;       // f16 elements of one 64-key K (or V) tile
  constexpr uint32_t kVOff = kStages * kTile * 2;  // f16 ring: byte offset of the V ring
  extern __shared__ __align__(128) unsigned char smem_raw[];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, z = blockIdx.z;
  const int kh = blockIdx.y / NHC, hc = blockIdx.y % NHC;
  const int head0 = kh * G + hc * GC;
  const int ngrid = gridDim.x;
  // Launched early behind the previous kernel of the stream (programmatic dependent launch):
  // nothing of global memory is read or written before that kernel has completed.
  grid_dependency_wait();
  if (a.pdl == 1) launch_dependents();
  if (refused<MODE>(a, z)) return;  // rows beyond the cache: touch nothing
  const Seq<T, TC> sq = resolve<T, TC, MODE>(a, z);
  const int len = sq.past + 1;  // keys 0..past, key `past` is the new token
  // Splits sized over the cache rows (fused: the new key is computed, not streamed), so that
  // 4096 rows in 8 splits are 8 whole 64-key tiles each; the last split also takes the rest
  // (at most one key more than split_len).
  const int rows = FUSED ? len - 1 : len;
  const int split_len = max(a.min_split, (ceil_div(max(rows, 1), ngrid) + 15) & ~15);
  const int nsplit = min(ceil_div(len, split_len), ngrid);
  if (kPg && (split_len >> a.block_shift) + 2 > kPagedTableCap) {
    // a split longer than the block-table copy holds (the host sizes the grid so that this
    // does not happen); the same for every CTA of the sequence, so none of them starts
    if (tid == 0 && split == 0 && blockIdx.y == 0) atomicOr(a.err, kErrPosBeyondCache);
    return;
  }
  // A cluster CTA past the last split still takes part in the cluster barriers (empty range).
  if (!CL && split >= nsplit) return;
  const int j0 = min(split * split_len, len);
  const int j1 = split == nsplit - 1 ? len : min(j0 + split_len, len);
  const bool has_new = FUSED && j0 < j1 && j1 == len;
  const int jcopy = has_new ? sq.past : j1;  // rows streamed from the cache
  const int64_t kv_stride = int64_t(a.hkv) * D;

  // paged: this split's block-table entries, pages j0 >> shift .. (j1 - 1) >> shift
  __shared__ int32_t tbl_s[kPg ? kPagedTableCap : 1];
  const int bshift = kPg ? a.block_shift : 0;
  const int blk0 = kPg ? (j0 >> bshift) : 0;
  if constexpr (kPg) {
    const int nblk = j1 > j0 ? ((j1 - 1) >> bshift) - blk0 + 1 : 0;
    for (int b = tid; b < nblk; b += kThreads) tbl_s[b] = sq.tbl[blk0 + b];
    __syncthreads();
  }
  // cache row of key j of this split
  auto row_of = [&](int j) -> int64_t {
    if constexpr (kPg)
      return (int64_t(tbl_s[(j >> bshift) - blk0]) << bshift) | int64_t(j & ((1 << bshift) - 1));
    else
      return int64_t(j);
  };

  __shared__ __align__(16) float stage_s[CL ? GC : 1][kPushStride];
  __shared__ __align__(16) float recv_s[CL ? recv_slots(CL) : 1][kPushStride];
  __shared__ __align__(8) uint64_t recv_bar;
  __shared__ __align__(8) uint64_t q_bar;
  if constexpr (CL) {
    if (tid == 0) {
      recv_bar_init(&recv_bar);
      recv_bar_init(&q_bar);
    }
    cluster_arrive_relaxed();  // matched by one cluster_wait(): after the prologue or at finish
  }
  __shared__ __align__(16) float q_s[GC][D];
  __shared__ float knew_s[D];
  __shared__ float vnew_s[D];
  __shared__ float red_m[kWarps][GC];
  __shared__ float red_l[kWarps][GC];
  __shared__ float red_acc[kWarps][GC][D];
  __shared__ int s_last;

  const TC* kbase = sq.kc + kh * D;
  const TC* vbase = sq.vc + kh * D;
  const int n_tiles = ceil_div(j1 - j0, kStageKeys);
  const uint32_t ring = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  auto issue_tile = [&](int tile) {
    if (tile < n_tiles) {
      const int jt = j0 + tile * kStageKeys;
      if constexpr (kQ8) {  // 64-byte rows, four 16-byte pieces each, row-contiguous staging
        const uint32_t st = (tile % kStages) * RingQ8::kStageBytes;
        const int c = tid & 3;
#pragma unroll
        for (int i = 0; i < kStageKeys / 32; ++i) {
          const int r = (tid >> 2) + 32 * i;
          const bool ok = jt + r < jcopy;
          const int64_t src = row_of(ok ? jt + r : j0) * kv_stride + c * 16;
          cp_async16(smem_raw + st + swz8(r, c), kbase + src, ok);
          cp_async16(smem_raw + st + RingQ8::kTileBytes + swz8(r, c), vbase + src, ok);
        }
      } else {
        const uint32_t off = (tile % kStages) * (kTile * 2);
        const int c = tid & 7;
#pragma unroll
        for (int i = 0; i < kStageKeys / 16; ++i) {
          const int r = (tid >> 3) + 16 * i;
          const bool ok = jt + r < jcopy;
          const int64_t src = row_of(ok ? jt + r : j0) * kv_stride + c * 8;
          cp_async16(smem_raw + off + swz(r, c), kbase + src, ok);
          cp_async16(smem_raw + kVOff + off + swz(r, c), vbase + src, ok);
        }
      }
    }
    cp_async_commit();
  };
  const bool q_bcast = CL != 0 && a.q_bcast;
  const bool do_q = !q_bcast || split == 0;
  PrologueSrc<T> psrc = prologue_global<T, TC>(a, sq, kh, head0);
  static_assert(prologue_stage_bytes<GC>() <= int(sizeof(red_acc)), "stage fits red_acc");
  if (a.pro_async)  // red_acc is free until the warp merge after the key loop
    psrc = prologue_stage<T, TC, GC, FUSED>(a, psrc, has_new, do_q,
                                            reinterpret_cast<unsigned char*>(&red_acc[0][0][0]));
#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) issue_tile(t);
  if (a.pro_async) {
    cp_async_wait<kStages - 1>();  // the prologue's group, the oldest, has landed
    __syncthreads();               // ... for every thread's pieces
  }
  const PrologueIn pin = prologue_load<T, TC, GC, FUSED>(a, psrc, has_new, do_q);

  // Cluster form with the qkv rows in host memory: the query rows are the same for every split
  // of a (layer, head chunk), so rank 0 alone reads them across the host link and rotates
  // them, and pushes the result into every peer's q_s (st.async, completing on the peer's
  // q_bar); the first K/V tiles are already in flight meanwhile.
  prologue<T, TC, GC, FUSED>(a, sq, kh, hc, head0, has_new, has_new ? row_of(sq.past) : 0,
                             1.0f, q_s, knew_s, vnew_s, pin, do_q);
  if (q_bcast) {
    cluster_wait();  // every rank's q_bar and recv_bar are initialised
    constexpr int kQChunks = GC * D * 4 / 16;  // 16-byte pieces of q_s
    if (split == 0) {
      __syncthreads();  // q_s complete
      for (int i = tid; i < (ngrid - 1) * kQChunks; i += kThreads) {
        const uint32_t peer = uint32_t(1 + i / kQChunks);
        const int c = i % kQChunks;
        const uint4 v = reinterpret_cast<const uint4*>(&q_s[0][0])[c];
        st_async16(map_rank(smem_addr(&q_s[0][0]) + 16u * c, peer), v,
                   map_rank(smem_addr(&q_bar), peer));
      }
    } else {
      if (tid == 0) recv_bar_expect(&q_bar, uint32_t(GC * D * 4));
      if (!recv_bar_try_wait(&q_bar)) {
        const uint64_t t0 = now_ns();
        bool ok = true;
        while (ok && !recv_bar_try_wait(&q_bar)) ok = now_ns() - t0 <= kWaitLimitNs;
        // Rank 0 never delivered: report it and carry on with whatever q_s holds, so that
        // this CTA still takes its part in the combine (no peer writes into a CTA that left).
        if (!ok && tid == 0) atomicOr(a.err, kErrTimeout);
      }
    }
  }
  __syncthreads();
  // int8 cache: the key scales fold into q (one per channel) or into the score scale
  float sl2 = a.scale_log2;
  if constexpr (kQ8) {
    if (a.scale_per_channel) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = tid + i * kThreads;
        if (e < GC * D) q_s[e / D][e % D] *= pin.ks[i];
      }
      __syncthreads();
    } else {
      sl2 *= pin.ks[0];
    }
  }

  // Q^T as the B operand (k = dims, n = heads): lane holds head n = lane/4 (zero when
  // n >= GC), dims 2(lane%4)+{0,1} and +8 of every 16-dim k-step.
  // int8 keys are read four dims per register (dims 4t..4t+3 of a 16-dim step), so there the
  // k index of the MMA runs over the dims in the order 4t, 4t+1 (k = 2t, 2t+1) and 4t+2, 4t+3
  // (k = 2t+8, 2t+9); q takes the same order (a permutation of the summed index).
  const int gid = lane >> 2, tig = lane & 3;
  uint32_t qb[4][2];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int d0 = kQ8 ? kk * 16 + 4 * tig : kk * 16 + 2 * tig;
    const int d1 = kQ8 ? d0 + 2 : d0 + 8;
    if (gid < GC) {
      qb[kk][0] = pack_h2(q_s[gid][d0], q_s[gid][d0 + 1]);
      qb[kk][1] = pack_h2(q_s[gid][d1], q_s[gid][d1 + 1]);
    } else {
      qb[kk][0] = qb[kk][1] = 0u;
    }
  }
  // Running state for heads 2*tig, 2*tig+1 (columns of the accumulator fragments).
  float m_run[2] = {kNegBig, kNegBig}, l_run[2] = {0.f, 0.f};
  float o[4][4];  // O^T tiles: dims 16i + gid (+8), heads 2*tig + {0,1}
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int mi = lane >> 3;

  for (int tile = 0; tile < n_tiles; ++tile) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // tile landed for every thread; slot (tile-1) % kStages is free again
    issue_tile(tile + kStages - 1);
    const int jt = j0 + tile * kStageKeys;
    // byte offsets (from smem_raw) of the K and V tiles the MMAs read
    uint32_t koff, voff;
    if constexpr (kQ8) {
      koff = (tile % kStages) * RingQ8::kStageBytes;
      voff = koff + RingQ8::kTileBytes;
    } else {
      koff = (tile % kStages) * (kTile * 2);
      voff = kVOff + koff;
    }
    if (FUSED && has_new && sq.past >= jt && sq.past < jt + kStageKeys) {
      // the new token's k/v (computed in the prologue) replace the zero-filled tile row
      const int r = sq.past - jt;
      if constexpr (kQ8) {
        if (tid < 8) {  // the quantised integers, 16 bytes per thread
          const int c = tid & 3;
          const float* src = (tid < 4 ? knew_s : vnew_s) + c * 16;
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k)
            w[k] = (uint32_t(int32_t(src[4 * k]) & 255)) |
                   (uint32_t(int32_t(src[4 * k + 1]) & 255) << 8) |
                   (uint32_t(int32_t(src[4 * k + 2]) & 255) << 16) |
                   (uint32_t(int32_t(src[4 * k + 3]) & 255) << 24);
          *reinterpret_cast<uint4*>(smem_raw + (tid < 4 ? koff : voff) + swz8(r, c)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else if (tid < 16) {
        const int c = tid & 7;
        const float* src = (tid < 8 ? knew_s : vnew_s) + c * 8;
        const uint4 val = make_uint4(pack_h2(src[0], src[1]), pack_h2(src[2], src[3]),
                                     pack_h2(src[4], src[5]), pack_h2(src[6], src[7]));
        *reinterpret_cast<uint4*>(smem_raw + (tid < 8 ? koff : voff) + swz(r, c)) = val;
      }
      __syncthreads();
    }
    const int rw = warp * 16;  // this warp's 16 keys of the tile
    // ---- S^T = K Q^T (4 k-steps over the 64 dims)
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (kQ8) {
      // one ldmatrix.x4 of int8 rows covers 16 keys x 32 dims: register 0 = key gid, dims
      // 4t..4t+3 of the first 16; 1 = key gid + 8; 2, 3 = the same for the next 16 dims
      const int r = rw + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int kk2 = 0; kk2 < 2; ++kk2) {
        uint32_t kr[4];
        ldsm_x4(ring + koff + swz8(r, kk2 * 2 + (lane >> 4)), kr);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t af[4];
          s8x4_to_f16x4(kr[2 * h], af[0], af[2]);
          s8x4_to_f16x4(kr[2 * h + 1], af[1], af[3]);
          mma16816(sacc, af, qb[kk2 * 2 + h][0], qb[kk2 * 2 + h][1]);
        }
      }
    } else {
      const int r = rw + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t af[4];
        ldsm_x4(ring + koff + swz(r, kk * 2 + (mi >> 1)), af);
        mma16816(sacc, af, qb[kk][0], qb[kk][1]);
      }
    }
    // ---- online softmax on the fragment: keys rw+gid (sacc 0,1) and rw+gid+8 (sacc 2,3)
    const bool v0 = jt + rw + gid < j1, v1 = jt + rw + gid + 8 < j1;
    const float t0 = v0 ? sacc[0] * sl2 : -INFINITY;
    const float t1 = v0 ? sacc[1] * sl2 : -INFINITY;
    const float t2 = v1 ? sacc[2] * sl2 : -INFINITY;
    const float t3 = v1 ? sacc[3] * sl2 : -INFINITY;
    float mb0 = fmaxf(t0, t2), mb1 = fmaxf(t1, t3);
#pragma unroll
    for (int sh = 4; sh <= 16; sh <<= 1) {
      mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, sh));
      mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, sh));
    }
    const float mn0 = fmaxf(m_run[0], mb0), mn1 = fmaxf(m_run[1], mb1);
    const float c0 = fast_exp2(m_run[0] - mn0), c1 = fast_exp2(m_run[1] - mn1);
    m_run[0] = mn0;
    m_run[1] = mn1;
    const float p0 = fast_exp2(t0 - mn0), p1 = fast_exp2(t1 - mn1);
    const float p2 = fast_exp2(t2 - mn0), p3 = fast_exp2(t3 - mn1);
    l_run[0] = fmaf(l_run[0], c0, p0 + p2);
    l_run[1] = fmaf(l_run[1], c1, p1 + p3);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[i][0] *= c0;
      o[i][1] *= c1;
      o[i][2] *= c0;
      o[i][3] *= c1;
    }
    // P^T as the B operand: the accumulator fragment transposed in registers, as f16 pairs
    // p = hi + lo (hi = f16(p), lo = f16(p - hi)): two MMAs per V fragment carry p to ~22
    // bits, so the weights that multiply V keep the f32 precision of the reference's p
    // (kernels.js:306-310) instead of f16's 11 bits; the tensor pipe has room (HBM bound).
    const uint32_t h01 = pack_h2(p0, p1), h23 = pack_h2(p2, p3);
    const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
    const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
    const uint32_t pb0 = movmatrix_trans(h01);
    const uint32_t pb1 = movmatrix_trans(h23);
    const uint32_t pl0 = movmatrix_trans(pack_h2(p0 - f01.x, p1 - f01.y));
    const uint32_t pl1 = movmatrix_trans(pack_h2(p2 - f23.x, p3 - f23.y));
    // ---- O^T += V^T P^T (4 m-tiles of 16 dims)
    if constexpr (kQ8) {
      // int8 V rows (keys) read four dims per register, converted to f16 pairs (dims 4t, 4t+1
      // and 4t+2, 4t+3 of key gid) and transposed with movmatrix into V^T fragments whose rows
      // are the dims 4(g>>1) + (g&1) (first 8 rows) and that + 2 (last 8) of each 16-dim tile
      const int r = rw + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int i2 = 0; i2 < 2; ++i2) {
        uint32_t vr[4];
        ldsm_x4(ring + voff + swz8(r, i2 * 2 + (lane >> 4)), vr);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t lo0, hi0, lo1, hi1;  // keys 0-7 and keys 8-15 of the warp's 16
          s8x4_to_f16x4(vr[2 * h], lo0, hi0);
          s8x4_to_f16x4(vr[2 * h + 1], lo1, hi1);
          const uint32_t af[4] = {movmatrix_trans(lo0), movmatrix_trans(hi0),
                                  movmatrix_trans(lo1), movmatrix_trans(hi1)};
          mma16816(o[i2 * 2 + h], af, pb0, pb1);
          mma16816(o[i2 * 2 + h], af, pl0, pl1);
        }
      }
    } else {
      const int r = rw + (mi >> 1) * 8 + (lane & 7);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t af[4];
        ldsm_x4_trans(ring + voff + swz(r, 2 * i + (mi & 1)), af);
        mma16816(o[i], af, pb0, pb1);
        mma16816(o[i], af, pl0, pl1);
      }
    }
  }
  cp_async_wait<0>();
  if (a.pdl == 2) launch_dependents();
  // output dims of the accumulator rows gid and gid + 8 of tile i: 16i + gid and 16i + gid + 8
  // for f16 caches; 16i + 4(gid>>1) + (gid&1) and that + 2 for int8 (the V^T row order above)
  const int dlo = kQ8 ? 4 * (gid >> 1) + (gid & 1) : gid;
  const int dhi = kQ8 ? dlo + 2 : gid + 8;
  if constexpr (kQ8) {  // the value scales, per output dim
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float s0 = kv_scale(a.v_scale, a.scale_per_channel, kh, 16 * i + dlo);
      const float s1 = kv_scale(a.v_scale, a.scale_per_channel, kh, 16 * i + dhi);
      o[i][0] *= s0;
      o[i][1] *= s0;
      o[i][2] *= s1;
      o[i][3] *= s1;
    }
  }

  // ---- warp totals: sum l over the 8 lanes that share a head column, then publish
#pragma unroll
  for (int sh = 4; sh <= 16; sh <<= 1) {
    l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], sh);
    l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], sh);
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int g = 2 * tig + e;
    if (g < GC) {
      if (gid == 0) {
        red_m[warp][g] = m_run[e];
        red_l[warp][g] = l_run[e];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        red_acc[warp][g][16 * i + dlo] = o[i][e];
        red_acc[warp][g][16 * i + dhi] = o[i][2 + e];
      }
    }
  }
  __syncthreads();
  if constexpr (CL) {
    finish_push<T, GC>(a, sq.orow + int64_t(head0) * D, split, nsplit, red_m, red_l, red_acc,
                       stage_s, recv_s, &recv_bar, q_bcast);
  } else {
    finish<T, GC>(a, sq.orow + int64_t(head0) * D, z * gridDim.y + blockIdx.y, split, nsplit,
                  ngrid, red_m, red_l, red_acc, &s_last);
  }
}

// ---- CUDA-core kernel (fp32 storage) ----------------------------------------------------------
template <int G, int NU>
__device__ __forceinline__ void softmax_update(float (&s)[NU][G], const bool (&valid)[NU],
                                               const float (&vf)[NU][8], float (&m_run)[G],
                                               float (&l_run)[G], float (&acc)[G][8]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float mb = kNegBig;
#pragma unroll
    for (int u = 0; u < NU; ++u)
      if (valid[u]) mb = fmaxf(mb, s[u][g]);
    const float mn = fmaxf(m_run[g], mb);
    const float c = fast_exp2(m_run[g] - mn);
    m_run[g] = mn;
    float psum = 0.f;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      s[u][g] = valid[u] ? fast_exp2(s[u][g] - mn) : 0.f;  // s now holds p
      psum += s[u][g];
    }
    l_run[g] = fmaf(l_run[g], c, psum);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[g][i] *= c;
  }
#pragma unroll
  for (int u = 0; u < NU; ++u)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[g][i] = fmaf(s[u][g], vf[u][i], acc[g][i]);
}

template <int G>
__device__ __forceinline__ void qk_partial(const float (&qr)[G][8], const float (&kf)[8],
                                           float (&s)[G]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      d0 = fmaf(qr[g][i], kf[i], d0);
      d1 = fmaf(qr[g][i + 1], kf[i + 1], d1);
    }
    s[g] = d0 + d1;
  }
}

template <int G>
__device__ __forceinline__ void reduce_slot(float (&s)[G]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    s[g] += __shfl_xor_sync(0xffffffffu, s[g], 1);
    s[g] += __shfl_xor_sync(0xffffffffu, s[g], 2);
    s[g] += __shfl_xor_sync(0xffffffffu, s[g], 4);
  }
}

template <int G, bool FUSED, int MODE>
__global__ void __launch_bounds__(kThreads, 2)
    decode_simt_kernel(const __grid_constant__ DecodeArgs a) {
  using T = float;
  constexpr int D = kHeadDim;
  constexpr int GC = G > 4 ? 4 : G;
  constexpr int NHC = G / GC;
  constexpr int kStages = Ring<T>::kStages;
  constexpr int kTile = Ring<T>::kTileElems;
  constexpr int kKeysPerThread = kStageKeys / 16;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* k_s = reinterpret_cast<T*>(smem_raw);
  T* v_s = k_s + kStages * kTile;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int slot = lane >> 3, part = lane & 7;
  const int split = blockIdx.x, z = blockIdx.z;
  const int kh = blockIdx.y / NHC, hc = blockIdx.y % NHC;
  const int head0 = kh * G + hc * GC;
  const int ngrid = gridDim.x;
  if (refused<MODE>(a, z)) return;
  const Seq<T, T> sq = resolve<T, T, MODE>(a, z);
  const int len = sq.past + 1;
  const int split_len = max(a.min_split, (ceil_div(len, ngrid) + 15) & ~15);
  const int nsplit = ceil_div(len, split_len);
  if (split >= nsplit) return;
  const int j0 = split * split_len;
  const int j1 = min(j0 + split_len, len);
  const bool has_new = FUSED && (j1 == len);
  const int jend = has_new ? sq.past : j1;
  const int64_t kv_stride = int64_t(a.hkv) * D;

  __shared__ float q_s[GC][D];
  __shared__ float knew_s[D];
  __shared__ float vnew_s[D];
  __shared__ float red_m[kWarps][GC];
  __shared__ float red_l[kWarps][GC];
  __shared__ float red_acc[kWarps][GC][D];
  __shared__ int s_last;

  const T* kbase = sq.kc + kh * D;
  const T* vbase = sq.vc + kh * D;
  const int n_tiles = ceil_div(max(jend - j0, 0), kStageKeys);
  auto issue_tile = [&](int tile) {
    if (tile < n_tiles) {
      T* ks = k_s + (tile % kStages) * kTile;
      T* vs = v_s + (tile % kStages) * kTile;
      const int jt = j0 + tile * kStageKeys;
#pragma unroll
      for (int i = 0; i < kStageKeys / 16; ++i) {
        const int r = (tid >> 3) + 16 * i;
        const bool ok = jt + r < jend;
        const int64_t src = int64_t(ok ? jt + r : j0) * kv_stride;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int e = part * 8 + c * 4;
          cp_async16(ks + r * D + e, kbase + src + e, ok);
          cp_async16(vs + r * D + e, vbase + src + e, ok);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) issue_tile(t);

  prologue<T, T, GC, FUSED>(a, sq, kh, hc, head0, has_new, sq.past, a.scale_log2, q_s, knew_s,
                            vnew_s,
                            prologue_load<T, T, GC, FUSED>(
                                a, prologue_global<T, T>(a, sq, kh, head0), has_new, true));
  __syncthreads();

  float qr[GC][8];
#pragma unroll
  for (int g = 0; g < GC; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) qr[g][i] = q_s[g][part * 8 + i];
  float m_run[GC], l_run[GC], acc[GC][8];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m_run[g] = kNegBig;
    l_run[g] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[g][i] = 0.f;
  }

  for (int tile = 0; tile < n_tiles; ++tile) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    issue_tile(tile + kStages - 1);
    const T* ks = k_s + (tile % kStages) * kTile;
    const T* vs = v_s + (tile % kStages) * kTile;
    const int jt = j0 + tile * kStageKeys;
    float s[kKeysPerThread][GC];
    bool valid[kKeysPerThread];
#pragma unroll
    for (int u = 0; u < kKeysPerThread; ++u) {
      const int r = warp * 4 + slot + 16 * u;
      float kf[8];
      load8_shared(ks + r * D + part * 8, kf);
      qk_partial<GC>(qr, kf, s[u]);
      valid[u] = jt + r < jend;
    }
#pragma unroll
    for (int u = 0; u < kKeysPerThread; ++u) reduce_slot<GC>(s[u]);
    float vf[kKeysPerThread][8];
#pragma unroll
    for (int u = 0; u < kKeysPerThread; ++u)
      load8_shared(vs + (warp * 4 + slot + 16 * u) * D + part * 8, vf[u]);
    softmax_update<GC, kKeysPerThread>(s, valid, vf, m_run, l_run, acc);
  }
  cp_async_wait<0>();

  if (FUSED && has_new && warp == 0) {  // the new token: its k/v are in shared memory
    float kf[8], vfn[1][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      kf[i] = knew_s[part * 8 + i];
      vfn[0][i] = vnew_s[part * 8 + i];
    }
    float s1[1][GC];
    qk_partial<GC>(qr, kf, s1[0]);
    reduce_slot<GC>(s1[0]);
    const bool v1[1] = {slot == 0};
    softmax_update<GC, 1>(s1, v1, vfn, m_run, l_run, acc);
  }

#pragma unroll
  for (int off = 8; off <= 16; off <<= 1) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m_run[g], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l_run[g], off);
      const float mn = fmaxf(m_run[g], mo);
      const float c1 = fast_exp2(m_run[g] - mn), c2 = fast_exp2(mo - mn);
      l_run[g] = l_run[g] * c1 + lo * c2;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float ao = __shfl_xor_sync(0xffffffffu, acc[g][i], off);
        acc[g][i] = acc[g][i] * c1 + ao * c2;
      }
      m_run[g] = mn;
    }
  }
  if (slot == 0) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
#pragma unroll
      for (int i = 0; i < 8; ++i) red_acc[warp][g][part * 8 + i] = acc[g][i];
      if (part == 0) {
        red_m[warp][g] = m_run[g];
        red_l[warp][g] = l_run[g];
      }
    }
  }
  __syncthreads();
  finish<T, GC>(a, sq.orow + int64_t(head0) * D, z * gridDim.y + blockIdx.y, split, nsplit,
                ngrid, red_m, red_l, red_acc, &s_last);
}

struct KernelInfo {
  const void* fn;
  int smem;
};

template <int G, bool FUSED, int MODE, int CL, int KVF>
KernelInfo info_h() {
  return {reinterpret_cast<const void*>(&decode_mma_kernel<G, FUSED, MODE, CL, KVF>),
          KVF == kKvI8 ? RingQ8::kBytes : Ring<__half>::kBytes};
}
template <int G, bool FUSED, int MODE>
KernelInfo info_f() {
  return {reinterpret_cast<const void*>(&decode_simt_kernel<G, FUSED, MODE>),
          Ring<float>::kBytes};
}

template <int G, bool FUSED>
KernelInfo pick_h(int mode, int cl, int kvf) {
  if (cl) {  // cluster combine: decode steps over layers only (f16 caches)
    if (mode != kLayers || kvf != kKvF16) return {nullptr, 0};
    return cl > kPortableCluster ? info_h<G, FUSED, kLayers, kMaxCluster, kKvF16>()
                                 : info_h<G, FUSED, kLayers, kPortableCluster, kKvF16>();
  }
  if (mode == kLayers) return kvf == kKvF16 ? info_h<G, FUSED, kLayers, 0, kKvF16>()
                                            : KernelInfo{nullptr, 0};
  if (mode == kRagged) return kvf == kKvF16 ? info_h<G, FUSED, kRagged, 0, kKvF16>()
                                            : info_h<G, FUSED, kRagged, 0, kKvI8>();
  return kvf == kKvF16 ? info_h<G, FUSED, kPaged, 0, kKvF16>()
                       : info_h<G, FUSED, kPaged, 0, kKvI8>();
}

template <int G>
KernelInfo pick_fm(bool half, bool fused, int mode, int cl, int kvf) {
  if (half) return fused ? pick_h<G, true>(mode, cl, kvf) : pick_h<G, false>(mode, cl, kvf);
  if (cl || kvf != kKvF16 || mode == kPaged) return {nullptr, 0};
  if (mode == kLayers) return fused ? info_f<G, true, kLayers>() : info_f<G, false, kLayers>();
  return fused ? info_f<G, true, kRagged>() : info_f<G, false, kRagged>();
}

// cl: 0 (workspace combine) or the cluster size
KernelInfo pick(int group, bool half, bool fused, int mode, int cl, int kvf = kKvF16) {
  switch (group) {
    case 1: return pick_fm<1>(half, fused, mode, cl, kvf);
    case 2: return pick_fm<2>(half, fused, mode, cl, kvf);
    case 4: return pick_fm<4>(half, fused, mode, cl, kvf);
    case 8: return pick_fm<8>(half, fused, mode, cl, kvf);
    default: return {nullptr, 0};
  }
}

// One-time attribute setup per kernel (dynamic shared memory; cluster kernels may use
// clusters above the portable 8 CTAs).
cudaError_t configure(const KernelInfo& k, bool cl) {
  static std::mutex mu;
  static std::set<const void*> configured;
  std::lock_guard<std::mutex> lk(mu);
  if (configured.count(k.fn)) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
  if (e != cudaSuccess) return e;
  if (cl) {
    e = cudaFuncSetAttribute(k.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  configured.insert(k.fn);
  return cudaSuccess;
}

int head_chunks(int group) { return group > 4 ? group / 4 : 1; }

}  // namespace

size_t decode_partials_bytes(int max_splits, int hkv, int nz, int group) {
  const int gc = group > 4 ? 4 : group;
  return size_t(max_splits) * hkv * head_chunks(group) * nz * gc * kPartialStride *
         sizeof(float);
}
size_t decode_counters_bytes(int hkv, int nz) {
  return size_t(hkv) * 2 /* up to 2 head chunks */ * nz * sizeof(int32_t);
}

int decode_max_splits(int64_t max_len, int hkv, int nz, int num_sms, int* min_split) {
  // Few (sequence, kv head) pairs: split every sequence so the CTAs fill each SM once
  // (3 resident per SM), rounding splits to whole 16-key passes.  Many pairs: fixed 1024-key
  // splits so long sequences spread over many CTAs and the block scheduler balances them.
  const int64_t pairs = int64_t(hkv) * nz;
  const int64_t slots = int64_t(num_sms) * 3;
  const int64_t by_len = (max_len + 15) / 16;
  if (pairs * 2 <= slots) {
    *min_split = 16;
    int64_t g = slots / pairs;
    if (g > by_len) g = by_len;
    return int(g < 1 ? 1 : g);
  }
  *min_split = 1024;
  const int64_t g = (max_len + 1023) / 1024;
  return int(g < 1 ? 1 : g);
}

// Clusters of `c` CTAs of kernel `k` the device can hold at once (cudaOccupancyMaxActiveClusters
// does not depend on the grid size); asked once per (kernel, c) and remembered, since the
// query costs host time and a decode step is launched once per token.
int max_active_clusters(const KernelInfo& k, int c) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(k.fn, c);
  const auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(c), 1, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = size_t(k.smem);
  cudaLaunchAttribute at{};
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = unsigned(c);
  at.val.clusterDim.y = 1;
  at.val.clusterDim.z = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, k.fn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache.emplace(key, n);
  return n;
}

int decode_cluster_splits(int64_t max_len, int hkv, int group, int nz, bool fused,
                          int num_sms) {
  // One wave: the (layer, head chunk) rows times the cluster size fill the 3 CTA slots of every
  // SM at most; at most kMaxCluster CTAs per cluster and one 16-key pass per CTA at least.  The
  // size is then lowered until the device reports that all clusters are resident at once.
  const int rows = hkv * head_chunks(group) * nz;
  const int64_t slots = int64_t(num_sms) * 3;
  int64_t c = slots / rows;
  const int64_t by_len = (max_len + 15) / 16;
  if (c > by_len) c = by_len;
  // Non-portable clusters (up to 16) only when portable ones would leave most SMs idle (one
  // layer: 8 kv heads x 8 splits = 64 CTAs on 148 SMs); with more rows they schedule worse.
  const int cap = int64_t(rows) * kPortableCluster * 2 <= num_sms ? kMaxCluster : kPortableCluster;
  if (c > cap) c = cap;
  if (c < 2) return 1;
  for (; c >= 2; --c) {
    const KernelInfo k = pick(group, true, fused, kLayers, int(c));
    if (!k.fn || configure(k, true) != cudaSuccess) return 1;
    if (max_active_clusters(k, int(c)) >= rows) return int(c);
  }
  return 1;
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether every input the prologue copies with 16-byte cp.async is 16-byte aligned and in
// device memory (host rows, the q_bcast form, keep plain loads).
bool prologue_async_ok(const DecodeArgs& a, int mode, bool fused, int nz) {
  if (a.q_bcast) return false;
  if (fused && !aligned16(a.rope)) return false;
  if (a.kv_format == kKvI8 && a.scale_per_channel && !aligned16(a.k_scale)) return false;
  if (mode == kLayers) {
    for (int l = 0; l < nz; ++l)
      if (!aligned16(a.layers[l].qkv) || (a.layers[l].norm_w && !aligned16(a.layers[l].norm_w)))
        return false;
    return true;
  }
  return aligned16(a.qkv) && (a.ld_qkv % 8) == 0 && (!a.norm_w || aligned16(a.norm_w));
}
}  // namespace

cudaError_t launch_decode(const DecodeArgs& args_in, int mode, bool fused, int dtype,
                          int max_splits, int nz, cudaStream_t s, int cluster) {
  DecodeArgs a = args_in;
  a.pro_async = dtype == 0 && prologue_async_ok(a, mode, fused, nz) ? 1 : 0;
  const int group = a.hq / a.hkv;
  const bool cl = cluster > 1;
  if (cl && (cluster > kMaxCluster || cluster != max_splits)) return cudaErrorInvalidValue;
  const KernelInfo k = pick(group, dtype == 0, fused, mode, cl ? cluster : 0, a.kv_format);
  if (!k.fn) return cudaErrorInvalidValue;
  cudaError_t e = configure(k, cl);
  if (e != cudaSuccess) return e;
  dim3 grid(max_splits, a.hkv * head_chunks(group), nz);
  void* args[] = {&a};
  if (!cl && !a.pdl) return cudaLaunchKernel(k.fn, grid, dim3(kThreads), args, size_t(k.smem), s);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = size_t(k.smem);
  cfg.stream = s;
  cudaLaunchAttribute at[2] = {};
  int n_at = 0;
  if (cl) {
    at[n_at].id = cudaLaunchAttributeClusterDimension;
    at[n_at].val.clusterDim.x = unsigned(cluster);
    at[n_at].val.clusterDim.y = 1;
    at[n_at].val.clusterDim.z = 1;
    ++n_at;
  }
  if (a.pdl) {
    at[n_at].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n_at].val.programmaticStreamSerializationAllowed = 1;
    ++n_at;
  }
  cfg.attrs = at;
  cfg.numAttrs = unsigned(n_at);
  return cudaLaunchKernelExC(&cfg, k.fn, args);
}

}  // namespace p2p
