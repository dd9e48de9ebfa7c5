// qk_prep.cu -- QK_PREP (src/scripts/lfm-engine/kernels.js:216-266) for sm_100a.
//
// Units [0,Hq) are q heads, [Hq,Hq+Hkv) k heads, [Hq+Hkv,Hq+2Hkv) v heads, exactly the shader's
// unit numbering generalised from 16/8.  Two kernels:
//  * qk_prep_rows_kernel (16-byte aligned buffers, the normal case): one THREAD per (q or k
//    head, token) row.  A warp stages its 32 rows through shared memory with row-contiguous
//    16-byte loads; each thread then sums the squares of its row in
//    the shader's tree order (pairs 32 apart, then 16, 8, 4, 2, 1: the same IEEE additions, so
//    the result is bit-identical), and computes inverseSqrt, the f16-rounded norm and the
//    rotate-half RoPE per element pair (i, i + 32), storing 16 bytes at a time.  The per-row
//    scalar work (divide, square root, reciprocal) is paid once per row instead of once per
//    row by a whole warp, which made the one-warp-per-row form instruction-bound (~130 warp
//    instructions per row, 8 % of DRAM bandwidth).  v heads are copied by further threads.
//  * qk_prep_kernel (any alignment): one warp per (head unit, token); lane l owns elements l
//    and l+32 (the rotate-half partners), so RoPE needs no exchange and the RMS sum is a
//    5-level butterfly that reproduces the shader's tree sum bit for bit.
#include "common.cuh"
#include "kernels.h"
#include "qk_row.cuh"

namespace p2p {
namespace {

constexpr int kWarpsPerBlock = 8;

template <class T>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    qk_prep_kernel(const QkPrepArgs a) {
  const int lane = threadIdx.x & 31;
  const int unit = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const int m = blockIdx.y;
  const int units = a.hq + 2 * a.hkv;
  if (unit >= units) return;
  const int64_t pos = int64_t(a.meta ? a.meta[0] : uint32_t(a.pos0)) + m;
  if (pos >= a.kv_cap) {  // the cache cannot hold this row: touch nothing, report it
    if ((threadIdx.x & 31) == 0) atomicOr(a.err, kErrPosBeyondCache);
    return;
  }
  const T* row = static_cast<const T*>(a.qkv) + int64_t(m) * a.ld_qkv;
  const int64_t kv_stride = int64_t(a.hkv) * kHeadDim;
  if (unit >= a.hq + a.hkv) {  // kernels.js:237-241: v heads are copied unchanged
    const int kh = unit - a.hq - a.hkv;
    const T* src = row + int64_t(a.hq + a.hkv) * kHeadDim + kh * kHeadDim;
    T* dst = static_cast<T*>(a.v_cache) + pos * kv_stride + kh * kHeadDim;
    dst[lane] = src[lane];
    dst[lane + 32] = src[lane + 32];
    return;
  }
  const bool isq = unit < a.hq;
  const int64_t off = int64_t(unit) * kHeadDim;  // q heads then k heads are contiguous
  const float v0 = to_f32(row[off + lane]);
  const float v1 = to_f32(row[off + lane + 32]);
  const T* nw = a.norm_w ? static_cast<const T*>(a.norm_w) + (isq ? 0 : kHeadDim) : nullptr;
  const T* rope = static_cast<const T*>(a.rope) + pos * kHeadDim;
  const float cs = to_f32(rope[lane]);
  const float sn = to_f32(rope[32 + lane]);
  float r0, r1;
  norm_rope_head<T>(v0, v1, nw, nw != nullptr, a.eps, cs, sn, r0, r1);
  T* dst = isq ? static_cast<T*>(a.q_out) + int64_t(m) * a.ld_q + off
               : static_cast<T*>(a.k_cache) + pos * kv_stride + (unit - a.hq) * kHeadDim;
  dst[lane] = from_f32<T>(r0);
  dst[lane + 32] = from_f32<T>(r1);
}


constexpr int kRowsPerBlock = 128;  // 4 warps; one q/k row per thread

// Threads [0, round_up(M*(Hq+Hkv), 32)) take the q and k rows, one per thread, token-major and
// unit-minor; threads beyond take the v rows, 16 bytes each.  A warp's 32 rows are staged
// through shared memory (row stride padded by 16 bytes, so the per-thread 16-byte reads and
// writes are conflict-free): global loads and stores then cover whole 128-byte rows per 8
// lanes instead of 32 different rows per instruction.
template <class T>
__global__ void __launch_bounds__(kRowsPerBlock)
    qk_prep_rows_kernel(const QkPrepArgs a) {
  // the attention that follows may launch now; it waits for this kernel to complete before
  // it reads anything
  launch_dependents();
  constexpr int kVec = 16 / sizeof(T);             // elements per 16-byte access
  constexpr int kPieces = kHeadDim / kVec;         // 16-byte pieces per row
  constexpr int kStride = kHeadDim * sizeof(T) + 16;  // staged row stride in bytes
  __shared__ float nw_s[2 * kHeadDim];
  __shared__ __align__(16) uint8_t stage[kRowsPerBlock / 32][32][kStride];
  const bool has_norm = a.norm_w != nullptr;
  if (has_norm)
    for (int i = threadIdx.x; i < 2 * kHeadDim; i += blockDim.x)
      nw_s[i] = to_f32(static_cast<const T*>(a.norm_w)[i]);
  __syncthreads();
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t pos0 = int64_t(a.meta ? a.meta[0] : uint32_t(a.pos0));
  const int qk_units = a.hq + a.hkv;
  const int64_t n_qk = int64_t(a.m_tokens) * qk_units;
  const int64_t n_qk_pad = (n_qk + 31) & ~int64_t(31);
  const int64_t kv_stride = int64_t(a.hkv) * kHeadDim;
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const T* qkv = static_cast<const T*>(a.qkv);
  if (idx >= n_qk_pad) {
    // v heads (kernels.js:237-241): copied unchanged, one 16-byte piece per thread (32-bit
    // index arithmetic: the host launches this kernel only for fewer than 2^31 threads)
    const uint32_t v = uint32_t(idx - n_qk_pad);
    if (v >= uint32_t(a.m_tokens) * uint32_t(a.hkv) * kPieces) return;
    const int piece = int(v % kPieces);
    const uint32_t vr = v / kPieces;
    const int kh = int(vr % uint32_t(a.hkv));
    const int m = int(vr / uint32_t(a.hkv));
    const int64_t pos = pos0 + m;
    if (pos >= a.kv_cap) {  // the cache cannot hold this row: touch nothing, report it
      atomicOr(a.err, kErrPosBeyondCache);
      return;
    }
    const T* src = qkv + int64_t(m) * a.ld_qkv + int64_t(qk_units + kh) * kHeadDim + piece * kVec;
    T* dst = static_cast<T*>(a.v_cache) + pos * kv_stride + kh * kHeadDim + piece * kVec;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    return;
  }
  // the whole warp is in the q/k range from here on (n_qk_pad is a multiple of 32); each lane
  // decodes its own row once, and the staged copies take row r's values from lane r
  const int64_t row0 = idx - lane;  // first row of this warp
  const int64_t row = row0 + lane;
  const int unit = int(uint32_t(row) % uint32_t(qk_units));
  const int m = int(uint32_t(row) / uint32_t(qk_units));
  const int64_t pos = pos0 + m;
  const bool mine = row < n_qk;
  const bool ok = mine && pos < a.kv_cap;
  if (mine && !ok) atomicOr(a.err, kErrPosBeyondCache);  // the cache cannot hold this row
  // staged load: flat piece f = i * 32 + lane -> row f / kPieces, piece f % kPieces
#pragma unroll
  for (int i = 0; i < kPieces; ++i) {
    const int f = i * 32 + lane, r = f / kPieces, pc = f % kPieces;
    const int mr = __shfl_sync(0xffffffffu, m, r), ur = __shfl_sync(0xffffffffu, unit, r);
    if (__shfl_sync(0xffffffffu, ok ? 1 : 0, r))
      *reinterpret_cast<uint4*>(&stage[wib][r][pc * 16]) = *reinterpret_cast<const uint4*>(
          qkv + int64_t(mr) * a.ld_qkv + int64_t(ur) * kHeadDim + pc * kVec);
  }
  __syncwarp();
  if (ok) {
    const bool isq = unit < a.hq;
    Row64<T> x;
    x.load(reinterpret_cast<const T*>(&stage[wib][lane][0]));
    T* out = reinterpret_cast<T*>(&stage[wib][lane][0]);  // results replace the staged row
    rotate_row<T>(x, has_norm ? nw_s + (isq ? 0 : kHeadDim) : nullptr, a.eps,
                  static_cast<const T*>(a.rope) + pos * kHeadDim,
                  [&](int k, const float(&v)[8]) { store8(out + 8 * k, v); });
  }
  __syncwarp();
  // staged store: q rows to q_out[m][unit], k rows to the cache row `pos`
#pragma unroll
  for (int i = 0; i < kPieces; ++i) {
    const int f = i * 32 + lane, r = f / kPieces, pc = f % kPieces;
    const int mr = __shfl_sync(0xffffffffu, m, r), ur = __shfl_sync(0xffffffffu, unit, r);
    if (__shfl_sync(0xffffffffu, ok ? 1 : 0, r)) {
      T* dst = ur < a.hq ? static_cast<T*>(a.q_out) + int64_t(mr) * a.ld_q + int64_t(ur) * kHeadDim
                         : static_cast<T*>(a.k_cache) + (pos0 + mr) * kv_stride +
                               int64_t(ur - a.hq) * kHeadDim;
      *reinterpret_cast<uint4*>(dst + pc * kVec) =
          *reinterpret_cast<const uint4*>(&stage[wib][r][pc * 16]);
    }
  }
}

}  // namespace

cudaError_t launch_qk_prep(const QkPrepArgs& a, int dtype, cudaStream_t s) {
  if (a.m_tokens <= 0) return cudaSuccess;
  const int units = a.hq + 2 * a.hkv;
  const size_t es = dtype == 0 ? 2 : 4;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int64_t n_qk = int64_t(a.m_tokens) * (a.hq + a.hkv);
  const int64_t threads = ((n_qk + 31) & ~int64_t(31)) +
                          int64_t(a.m_tokens) * a.hkv * int64_t(kHeadDim * es / 16);
  if (al16(a.qkv) && al16(a.q_out) && al16(a.k_cache) && al16(a.v_cache) && al16(a.rope) &&
      (a.ld_qkv * es) % 16 == 0 && (a.ld_q * es) % 16 == 0 &&
      threads + kRowsPerBlock <= INT32_MAX) {
    const int64_t blocks = (threads + kRowsPerBlock - 1) / kRowsPerBlock;
    if (dtype == 0) qk_prep_rows_kernel<__half><<<unsigned(blocks), kRowsPerBlock, 0, s>>>(a);
    else qk_prep_rows_kernel<float><<<unsigned(blocks), kRowsPerBlock, 0, s>>>(a);
    return cudaGetLastError();
  }
  dim3 grid(ceil_div(units, kWarpsPerBlock), a.m_tokens);
  if (dtype == 0) qk_prep_kernel<__half><<<grid, kWarpsPerBlock * 32, 0, s>>>(a);
  else qk_prep_kernel<float><<<grid, kWarpsPerBlock * 32, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace p2p
