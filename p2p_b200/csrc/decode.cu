// decode.cu -- split-KV decode attention for sm_100a (ATTN at M = 1,
// src/scripts/lfm-engine/kernels.js:268-319, optionally fused with QK_PREP, :216-266).
//
// Grid (splits, Hkv * head_chunks, Z).  Z is either the attention layers of one decode step
// (all at the same position, engine.js:425-429) or the sequences of a ragged batch.  One CTA
// streams one contiguous key range of ONE kv head and serves up to 4 of its G = Hq/Hkv query
// heads, so for G <= 4 every K/V byte is read from HBM exactly once (the shader reads each kv
// head once per q head, kernels.js:282).
//
// Memory pipeline: a kStages-deep cp.async ring of 64-key tiles in shared memory; every warp
// instruction copies four whole 128-byte K (or V) rows.  Compute: lane = 8*slot + part; the 8
// lanes of a slot hold one key row's 8-element chunks, complete the dot products with a
// 3-level xor-shuffle, and each slot keeps its own online-softmax state (running max and sum,
// 8 accumulator dims per q head) in the log2 domain.  Slots merge with shuffles, warps through
// shared memory.  A CTA whose sequence needs more than one split writes its partial
// (acc, max, sum) to the workspace; the last CTA of the (sequence, head chunk) to arrive --
// counted with one atomic -- runs the second pass that combines the partials and writes the
// output, then resets its counter.  Nothing ever waits on another CTA.
#include <mutex>
#include <set>

#include "common.cuh"
#include "kernels.h"

namespace p2p {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = 4;
constexpr int kStageKeys = 64;                   // keys per pipeline stage
constexpr int kKeysPerThread = kStageKeys / 16;  // 4 warps x 4 slots cover 16 rows per pass
constexpr float kNegBig = -1e30f;
constexpr int kPartialStride = kHeadDim + 2;  // acc[64], max, sum

template <class T>
struct Ring {
  static constexpr int kStages = sizeof(T) == 2 ? 4 : 2;
  static constexpr int kTileElems = kStageKeys * kHeadDim;
  static constexpr int kBytes = 2 * kStages * kTileElems * int(sizeof(T));  // K and V
};

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
    const float c = exp2f(m_run[g] - mn);
    m_run[g] = mn;
    float psum = 0.f;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      s[u][g] = valid[u] ? exp2f(s[u][g] - mn) : 0.f;  // s now holds p
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

// G: query heads per kv head; GC: query heads handled by one CTA (G / GC head chunks).
template <class T, int G, bool FUSED, int MODE>
__global__ void __launch_bounds__(kThreads, 3) decode_kernel(const __grid_constant__ DecodeArgs a) {
  constexpr int D = kHeadDim;
  constexpr int GC = G > 4 ? 4 : G;
  constexpr int NHC = G / GC;
  constexpr int kStages = Ring<T>::kStages;
  constexpr int kTile = Ring<T>::kTileElems;
  constexpr int kCopies = int(sizeof(T)) * 8 / 16;  // 16-byte copies per 8-element chunk
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* k_s = reinterpret_cast<T*>(smem_raw);
  T* v_s = k_s + kStages * kTile;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int slot = lane >> 3, part = lane & 7;
  const int split = blockIdx.x, z = blockIdx.z;
  const int kh = blockIdx.y / NHC, hc = blockIdx.y % NHC;
  const int head0 = kh * G + hc * GC;  // first q head of this CTA
  const int ngrid = gridDim.x;

  int past;
  const T* qrow;
  const T* nw;
  T* kc;
  T* vc;
  T* orow;
  if (MODE == kLayers) {
    const DecodeLayer& L = a.layers[z];
    past = a.meta ? int(a.meta[0]) : a.pos_host;
    qrow = static_cast<const T*>(L.qkv);
    nw = static_cast<const T*>(L.norm_w);
    kc = static_cast<T*>(L.k_cache);
    vc = static_cast<T*>(L.v_cache);
    orow = static_cast<T*>(L.out);
  } else {
    past = a.past[z];
    qrow = static_cast<const T*>(a.qkv) + int64_t(z) * a.ld_qkv;
    nw = static_cast<const T*>(a.norm_w);
    const int64_t row0 = int64_t(a.offsets[z]) * a.hkv * D;
    kc = static_cast<T*>(a.k_cache) + row0;
    vc = static_cast<T*>(a.v_cache) + row0;
    orow = static_cast<T*>(a.out) + int64_t(z) * a.ld_o;
  }
  if (MODE == kLayers && int64_t(past) >= a.kv_cap) {  // refuse rows beyond the cache
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.err, kErrPosBeyondCache);
    return;
  }
  const int len = past + 1;  // keys 0..past, key `past` is the new token
  const int split_len = max(a.min_split, (ceil_div(len, ngrid) + 15) & ~15);
  const int nsplit = ceil_div(len, split_len);
  if (split >= nsplit) return;
  const int j0 = split * split_len;
  const int j1 = min(j0 + split_len, len);
  const bool has_new = FUSED && (j1 == len);
  const int jend = has_new ? past : j1;  // keys streamed from the cache
  const int64_t kv_stride = int64_t(a.hkv) * D;

  __shared__ float q_s[GC][D];
  __shared__ float knew_s[D];
  __shared__ float vnew_s[D];
  __shared__ float red_m[kWarps][GC];
  __shared__ float red_l[kWarps][GC];
  __shared__ float red_acc[kWarps][GC][D];
  __shared__ int s_last;

  // ---- start streaming K/V rows [j0, jend) of kv head kh --------------------------------
  const T* kbase = kc + kh * D;
  const T* vbase = vc + kh * D;
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
        for (int c = 0; c < kCopies; ++c) {
          const int e = part * 8 + c * (16 / int(sizeof(T)));
          cp_async16(ks + r * D + e, kbase + src + e, ok);
          cp_async16(vs + r * D + e, vbase + src + e, ok);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) issue_tile(t);

  // ---- prologue (overlaps the first copies): rotated q heads and, fused, the new k/v -----
  if (FUSED) {
    const T* rope = static_cast<const T*>(a.rope) + int64_t(past) * D;
    const float cs = to_f32(rope[lane]);
    const float sn = to_f32(rope[32 + lane]);
    const int units = GC + (has_new ? 2 : 0);
    for (int u = warp; u < units; u += kWarps) {
      if (u < GC) {  // QK_PREP q unit, then ATTN's f32(q) * scale (kernels.js:255-263, :283)
        const int64_t off = int64_t(head0 + u) * D;
        float r0, r1;
        norm_rope_head<T>(to_f32(qrow[off + lane]), to_f32(qrow[off + lane + 32]), nw,
                          nw != nullptr, a.eps, cs, sn, r0, r1);
        q_s[u][lane] = round_st<T>(r0) * a.scale_log2;
        q_s[u][lane + 32] = round_st<T>(r1) * a.scale_log2;
      } else if (u == GC) {  // QK_PREP k unit -> cache row `past`
        const int64_t off = int64_t(a.hq + kh) * D;
        float r0, r1;
        norm_rope_head<T>(to_f32(qrow[off + lane]), to_f32(qrow[off + lane + 32]),
                          nw ? nw + D : nullptr, nw != nullptr, a.eps, cs, sn, r0, r1);
        const T k0 = from_f32<T>(r0), k1 = from_f32<T>(r1);
        if (hc == 0) {
          T* dst = kc + int64_t(past) * kv_stride + kh * D;
          dst[lane] = k0;
          dst[lane + 32] = k1;
        }
        knew_s[lane] = to_f32(k0);
        knew_s[lane + 32] = to_f32(k1);
      } else {  // QK_PREP v unit: raw copy -> cache row `past`
        const int64_t off = int64_t(a.hq + a.hkv + kh) * D;
        const T x0 = qrow[off + lane], x1 = qrow[off + lane + 32];
        if (hc == 0) {
          T* dst = vc + int64_t(past) * kv_stride + kh * D;
          dst[lane] = x0;
          dst[lane + 32] = x1;
        }
        vnew_s[lane] = to_f32(x0);
        vnew_s[lane + 32] = to_f32(x1);
      }
    }
  } else {
    for (int i = tid; i < GC * D; i += kThreads)
      q_s[i / D][i % D] = to_f32(qrow[int64_t(head0) * D + i]) * a.scale_log2;
  }
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

  // ---- main loop over the ring ------------------------------------------------------------
  for (int tile = 0; tile < n_tiles; ++tile) {
    cp_async_wait<kStages - 2>();
    __syncthreads();  // tile landed for every thread; slot (tile-1) % kStages is free again
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

  // ---- the new token (fused, last split): its k/v are in shared memory -------------------
  if (FUSED && has_new && warp == 0) {
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

  // ---- merge the 4 slots of each warp, then the 4 warps ----------------------------------
#pragma unroll
  for (int off = 8; off <= 16; off <<= 1) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m_run[g], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l_run[g], off);
      const float mn = fmaxf(m_run[g], mo);
      const float c1 = exp2f(m_run[g] - mn), c2 = exp2f(mo - mn);
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

  T* out_h = orow + int64_t(head0) * D;
  const int pair = z * gridDim.y + blockIdx.y;
  float* part_base = a.partials + int64_t(pair) * ngrid * (GC * kPartialStride);
  for (int idx = tid; idx < GC * D; idx += kThreads) {
    const int g = idx / D, d = idx % D;
    float mx = red_m[0][g];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, red_m[w][g]);
    float l = 0.f, ac = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float c = exp2f(red_m[w][g] - mx);
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

  // ---- second pass: the last CTA of this (sequence, head chunk) combines the partials ----
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&a.counters[pair], 1);
    s_last = (prev == nsplit - 1);
  }
  __syncthreads();
  if (!s_last) return;
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
      const float c = exp2f(__ldcg(p + D) - mx);
      l = fmaf(__ldcg(p + D + 1), c, l);
      ac = fmaf(__ldcg(p + d), c, ac);
    }
    out_h[idx] = from_f32<T>(ac / l);
  }
  if (tid == 0) a.counters[pair] = 0;
}

struct KernelInfo {
  const void* fn;
  int smem;
};

template <class T, int G, bool FUSED, int MODE>
KernelInfo info() {
  return {reinterpret_cast<const void*>(&decode_kernel<T, G, FUSED, MODE>), Ring<T>::kBytes};
}

template <class T, int G>
KernelInfo pick_fm(bool fused, int mode) {
  if (mode == kLayers) return fused ? info<T, G, true, kLayers>() : info<T, G, false, kLayers>();
  return fused ? info<T, G, true, kRagged>() : info<T, G, false, kRagged>();
}

template <class T>
KernelInfo pick_g(int group, bool fused, int mode) {
  switch (group) {
    case 1: return pick_fm<T, 1>(fused, mode);
    case 2: return pick_fm<T, 2>(fused, mode);
    case 4: return pick_fm<T, 4>(fused, mode);
    case 8: return pick_fm<T, 8>(fused, mode);
    default: return {nullptr, 0};
  }
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

cudaError_t launch_decode(const DecodeArgs& a, int mode, bool fused, int dtype, int max_splits,
                          int nz, cudaStream_t s) {
  const int group = a.hq / a.hkv;
  const KernelInfo k =
      dtype == 0 ? pick_g<__half>(group, fused, mode) : pick_g<float>(group, fused, mode);
  if (!k.fn) return cudaErrorInvalidValue;
  static std::mutex mu;
  static std::set<const void*> configured;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!configured.count(k.fn)) {
      cudaError_t e =
          cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem);
      if (e != cudaSuccess) return e;
      configured.insert(k.fn);
    }
  }
  dim3 grid(max_splits, a.hkv * head_chunks(group), nz);
  void* args[] = {const_cast<DecodeArgs*>(&a)};
  return cudaLaunchKernel(k.fn, grid, dim3(kThreads), args, size_t(k.smem), s);
}

}  // namespace p2p
