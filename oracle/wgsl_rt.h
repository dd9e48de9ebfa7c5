// wgsl_rt.h -- host execution model for WGSL compute shaders translated by oracle/wgsl2cpp.py
// (TEST INFRASTRUCTURE ONLY; used to run the reference's own shader text on host cores).
//
// Each shader invocation becomes a C++20 coroutine.  workgroupBarrier() suspends it; a
// workgroup is executed by resuming every invocation of the group in turn until all of them
// reach the barrier (or finish), which is exactly the WGSL barrier semantics for the
// workgroup-uniform control flow that WGSL requires.  Workgroups are independent and are
// distributed over OpenMP threads; workgroup-address-space variables are thread_local and
// zeroed at the start of every workgroup (WGSL zero-initialises workgroup memory).
//
// Scalar semantics: f32 is IEEE single; f16 storage is binary16 with round-to-nearest-even
// conversion (the same rule as engine.js:28-50); exp/inverseSqrt use the C library in single
// precision; no FMA contraction (compile with -ffp-contract=off).
#ifndef P2P_WGSL_RT_H
#define P2P_WGSL_RT_H

#include <coroutine>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace wgsl {

struct h16 {
  uint16_t bits;
};

inline uint16_t to_half_bits(float v) {
  uint32_t x;
  std::memcpy(&x, &v, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t e = int32_t((x >> 23) & 0xffu) - 112;
  uint32_t m = x & 0x7fffffu;
  if (((x >> 23) & 0xffu) == 0xffu) return uint16_t(sign | 0x7c00u | (m ? 0x200u : 0u));
  if (e >= 31) return uint16_t(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return uint16_t(sign);
    m |= 0x800000u;
    const int sh = 14 - e;
    uint32_t h = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u);
    if (rem > (1u << (sh - 1)) || (rem == (1u << (sh - 1)) && (h & 1u))) h++;
    return uint16_t(sign | h);
  }
  uint32_t h = (uint32_t(e) << 10) | (m >> 13);
  const uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return uint16_t(sign | h);
}

inline float from_half_bits(uint16_t h) {
  const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
  if (e == 0) {
    const float mag = std::ldexp(float(m), -24);
    return (h & 0x8000u) ? -mag : mag;
  }
  const uint32_t bits = (uint32_t(h & 0x8000u) << 16) |
                        (e == 31 ? (0x7f800000u | (m << 13)) : (((e + 112u) << 23) | (m << 13)));
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// WGSL value constructors / conversions used by the shaders.
inline float f32(h16 x) { return from_half_bits(x.bits); }
inline float f32(float x) { return x; }
inline float f32(uint32_t x) { return float(x); }
inline float f32(int32_t x) { return float(x); }
inline h16 f16(float x) { return h16{to_half_bits(x)}; }
inline h16 f16(h16 x) { return x; }
inline uint32_t u32(float x) { return x <= 0.0f ? 0u : uint32_t(x); }
inline uint32_t u32(uint32_t x) { return x; }
inline uint32_t u32(int32_t x) { return uint32_t(x); }

// Builtins.
inline float exp_(float x) { return std::exp(x); }
inline float inverseSqrt(float x) { return 1.0f / std::sqrt(x); }
inline float max_(float a, float b) { return std::fmax(a, b); }
inline float min_(float a, float b) { return std::fmin(a, b); }
inline uint32_t max_(uint32_t a, uint32_t b) { return a > b ? a : b; }
inline uint32_t min_(uint32_t a, uint32_t b) { return a < b ? a : b; }

struct uvec3 {
  uint32_t x, y, z;
};

// vec4<f32> and array<vec4<f32>, 4> (the GEMM's 4x4 accumulators): componentwise, every
// operation separately rounded.
struct vec4f {
  float c[4];
  explicit vec4f(float v) : c{v, v, v, v} {}
  vec4f(float a, float b, float d, float e) : c{a, b, d, e} {}
  float& operator[](uint32_t i) { return c[i]; }
  float operator[](uint32_t i) const { return c[i]; }
};
inline vec4f operator*(float s, const vec4f& v) {
  return vec4f(s * v.c[0], s * v.c[1], s * v.c[2], s * v.c[3]);
}
inline vec4f& operator+=(vec4f& a, const vec4f& b) {
  for (int i = 0; i < 4; ++i) a.c[i] += b.c[i];
  return a;
}
struct array4v {
  vec4f v[4];
  array4v(const vec4f& a, const vec4f& b, const vec4f& d, const vec4f& e) : v{a, b, d, e} {}
  vec4f& operator[](uint32_t i) { return v[i]; }
};

// One invocation = one coroutine.
struct Task {
  struct promise_type {
    Task get_return_object() {
      return Task{std::coroutine_handle<promise_type>::from_promise(*this)};
    }
    std::suspend_always initial_suspend() noexcept { return {}; }
    std::suspend_always final_suspend() noexcept { return {}; }
    void return_void() noexcept {}
    void unhandled_exception() noexcept { std::terminate(); }
  };
  std::coroutine_handle<promise_type> h;
};

struct Barrier {
  bool await_ready() const noexcept { return false; }
  void await_suspend(std::coroutine_handle<>) const noexcept {}
  void await_resume() const noexcept {}
};

// Runs every workgroup of a (gx, gy, gz) dispatch.  make(wid, local_index) creates the
// invocation coroutine; reset() zeroes the workgroup variables of the calling thread.
// Returns 0, or -1 if some invocation left a barrier phase early (non-uniform barrier).
template <class Make, class Reset>
int dispatch(uint32_t gx, uint32_t gy, uint32_t gz, uint32_t wg_size, Make make, Reset reset) {
  const int64_t groups = int64_t(gx) * gy * gz;
  int bad = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
  for (int64_t g = 0; g < groups; ++g) {
    const uvec3 wid{uint32_t(g % gx), uint32_t((g / gx) % gy), uint32_t(g / (int64_t(gx) * gy))};
    reset();
    std::vector<Task> inv;
    inv.reserve(wg_size);
    for (uint32_t t = 0; t < wg_size; ++t) inv.push_back(make(wid, t));
    for (;;) {
      uint32_t finished = 0;
      for (auto& tk : inv) {
        if (!tk.h.done()) tk.h.resume();
        if (tk.h.done()) ++finished;
      }
      if (finished == wg_size) break;
      // Every invocation must be at the same barrier: none may finish while others wait.
      for (auto& tk : inv)
        if (tk.h.done()) bad = 1;
      if (bad) break;
    }
    for (auto& tk : inv) tk.h.destroy();
  }
  return bad ? -1 : 0;
}

}  // namespace wgsl

#endif
