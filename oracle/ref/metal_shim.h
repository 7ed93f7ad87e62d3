// metal_shim.h -- just enough of the Metal Shading Language's vocabulary for
// the MSL text that tiny-metal-nn generates to compile as host C++.
//
// TEST INFRASTRUCTURE: used only by oracle/ref_build.py to execute the
// reference's own generated kernels on the CPU (oracle/_ref), so the CPU
// restatement in oracle/tmnn_oracle.c can be pinned against them.
//
// Semantics: vectors are plain value types with component-wise operators;
// address-space qualifiers vanish; atomics map to std::atomic; a threadgroup
// is emulated by running its threads as std::threads that meet at a
// std::barrier (the driver sets the current barrier per thread); the
// simdgroup operations of the SIMD training kernel are emulated per lane
// (below).
#pragma once
#include <atomic>
#include <barrier>
#include <cmath>
#include <cstdint>

typedef unsigned int uint;

namespace metal {

template <class T> struct V2 {
  T x, y;
  V2() = default;
  explicit V2(T s) : x(s), y(s) {}
  V2(T a, T b) : x(a), y(b) {}
  template <class U> explicit V2(const V2<U> &o) : x(T(o.x)), y(T(o.y)) {}
};
template <class T> struct V3 {
  T x, y, z;
  V3() = default;
  explicit V3(T s) : x(s), y(s), z(s) {}
  V3(T a, T b, T c) : x(a), y(b), z(c) {}
  template <class U> explicit V3(const V3<U> &o) : x(T(o.x)), y(T(o.y)), z(T(o.z)) {}
};
template <class T> struct V4 {
  T x, y, z, w;
  V4() = default;
  explicit V4(T s) : x(s), y(s), z(s), w(s) {}
  V4(T a, T b, T c, T d) : x(a), y(b), z(c), w(d) {}
  template <class U> explicit V4(const V4<U> &o)
      : x(T(o.x)), y(T(o.y)), z(T(o.z)), w(T(o.w)) {}
};

#define SHIM_VEC_OPS(V, APPLY)                                                  \
  template <class T> V<T> operator+(V<T> a, V<T> b) { return APPLY(a, b, +); } \
  template <class T> V<T> operator-(V<T> a, V<T> b) { return APPLY(a, b, -); } \
  template <class T> V<T> operator*(V<T> a, V<T> b) { return APPLY(a, b, *); } \
  template <class T> V<T> operator/(V<T> a, V<T> b) { return APPLY(a, b, /); } \
  template <class T> V<T> operator*(T s, V<T> b) { return V<T>(s) * b; }       \
  template <class T> V<T> operator*(V<T> a, T s) { return a * V<T>(s); }       \
  template <class T> V<T> operator+(V<T> a, T s) { return a + V<T>(s); }       \
  template <class T> V<T> &operator+=(V<T> &a, V<T> b) { return a = a + b; }   \
  template <class T> V<T> &operator-=(V<T> &a, V<T> b) { return a = a - b; }   \
  template <class T> V<T> &operator*=(V<T> &a, V<T> b) { return a = a * b; }   \
  template <class T> V<T> &operator*=(V<T> &a, T s) { return a = a * s; }

#define SHIM_AP2(a, b, op) V2<T>(a.x op b.x, a.y op b.y)
#define SHIM_AP3(a, b, op) V3<T>(a.x op b.x, a.y op b.y, a.z op b.z)
#define SHIM_AP4(a, b, op) V4<T>(a.x op b.x, a.y op b.y, a.z op b.z, a.w op b.w)
SHIM_VEC_OPS(V2, SHIM_AP2)
SHIM_VEC_OPS(V3, SHIM_AP3)
SHIM_VEC_OPS(V4, SHIM_AP4)

typedef V2<float> float2;
typedef V3<float> float3;
typedef V4<float> float4;
typedef V2<int> int2;
typedef V3<int> int3;
typedef V4<int> int4;
typedef V2<uint> uint2;
typedef V3<uint> uint3;
typedef V4<uint> uint4;
typedef _Float16 half;
typedef V2<half> half2;
typedef V4<half> half4;

inline float floor(float x) { return std::floor(x); }
inline float sqrt(float x) { return std::sqrt(x); }
inline float pow(float x, float y) { return std::pow(x, y); }
inline float exp(float x) { return std::exp(x); }
inline float log(float x) { return std::log(x); }
inline float sin(float x) { return std::sin(x); }
inline float cos(float x) { return std::cos(x); }
inline float abs(float x) { return std::fabs(x); }
inline int abs(int x) { return x < 0 ? -x : x; }
inline float max(float a, float b) { return std::fmax(a, b); }
inline float min(float a, float b) { return std::fmin(a, b); }
inline int max(int a, int b) { return a > b ? a : b; }
inline int min(int a, int b) { return a < b ? a : b; }
inline uint max(uint a, uint b) { return a > b ? a : b; }
inline uint min(uint a, uint b) { return a < b ? a : b; }
inline float clamp(float x, float lo, float hi) { return min(max(x, lo), hi); }
inline bool isnan(float x) { return std::isnan(x); }
inline bool isinf(float x) { return std::isinf(x); }
inline bool isfinite(float x) { return std::isfinite(x); }
inline float2 floor(float2 v) { return float2(floor(v.x), floor(v.y)); }
inline float3 floor(float3 v) { return float3(floor(v.x), floor(v.y), floor(v.z)); }
inline float4 floor(float4 v) {
  return float4(floor(v.x), floor(v.y), floor(v.z), floor(v.w));
}
inline float4 max(float4 a, float4 b) {
  return float4(max(a.x, b.x), max(a.y, b.y), max(a.z, b.z), max(a.w, b.w));
}
inline float dot(float4 a, float4 b) {
  return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}
inline float dot(float3 a, float3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
inline float dot(float2 a, float2 b) { return a.x * b.x + a.y * b.y; }

typedef std::atomic<int> atomic_int;
typedef std::atomic<uint> atomic_uint;
typedef std::atomic<float> atomic_float;
constexpr std::memory_order memory_order_relaxed = std::memory_order_relaxed;
template <class A, class T>
inline auto atomic_fetch_add_explicit(A *a, T v, std::memory_order o) {
  return a->fetch_add(v, o);
}
template <class A, class T>
inline auto atomic_fetch_or_explicit(A *a, T v, std::memory_order o) {
  return a->fetch_or(v, o);
}
template <class A, class T>
inline void atomic_store_explicit(A *a, T v, std::memory_order o) {
  a->store(v, o);
}
template <class A>
inline auto atomic_load_explicit(A *a, std::memory_order o) {
  return a->load(o);
}

enum class mem_flags { mem_none, mem_device, mem_threadgroup };
extern thread_local std::barrier<> *g_tg_barrier;
inline void threadgroup_barrier(mem_flags) {
  if (g_tg_barrier) g_tg_barrier->arrive_and_wait();
}

// ---- simdgroup operations (the reference's SIMD training kernel) ----------
// A simdgroup is 32 consecutive threads of the emulated threadgroup, which
// meet at their own std::barrier (set per thread by the driver, with the
// lane index and 32 floats of per-simdgroup scratch).  MSL executes these
// operations collectively; here every lane holds a full copy of each 8x8
// matrix (all lanes load the same elements), computes the product itself,
// and one lane writes results back, with a simdgroup barrier before every
// collective load, sum and store so the lanes' earlier writes are visible.
// The summation order inside a product is row-by-column in k order, so
// results agree with the hardware's to rounding, not bit for bit.
extern thread_local std::barrier<> *g_simd_barrier;
extern thread_local unsigned g_simd_lane;
extern thread_local float *g_simd_scratch;
inline void simd_sync() {
  if (g_simd_barrier) g_simd_barrier->arrive_and_wait();
}

typedef V2<unsigned long> ulong2;

template <class T> struct simdgroup_matrix8 {
  T e[8][8];
};
typedef simdgroup_matrix8<float> simdgroup_float8x8;
typedef simdgroup_matrix8<half> simdgroup_half8x8;

// m(r, c) = src[(origin.y + r) * elements_per_row + origin.x + c], or with
// transpose the element at (c, r) of the source block.
template <class T, class S>
inline void simdgroup_load(simdgroup_matrix8<T> &m, const S *src,
                           unsigned long elements_per_row,
                           ulong2 origin = ulong2(0ul, 0ul),
                           bool transpose = false) {
  simd_sync();
  for (int r = 0; r < 8; ++r)
    for (int c = 0; c < 8; ++c) {
      const unsigned long rr = transpose ? c : r, cc = transpose ? r : c;
      m.e[r][c] = T(src[(origin.y + rr) * elements_per_row + origin.x + cc]);
    }
}

template <class T, class D>
inline void simdgroup_store(const simdgroup_matrix8<T> &m, D *dst,
                            unsigned long elements_per_row,
                            ulong2 origin = ulong2(0ul, 0ul),
                            bool transpose = false) {
  simd_sync();
  if (g_simd_lane == 0)
    for (int r = 0; r < 8; ++r)
      for (int c = 0; c < 8; ++c) {
        const unsigned long rr = transpose ? c : r, cc = transpose ? r : c;
        dst[(origin.y + rr) * elements_per_row + origin.x + cc] = D(m.e[r][c]);
      }
  simd_sync();
}

template <class T>
inline void simdgroup_multiply_accumulate(simdgroup_matrix8<T> &d,
                                          const simdgroup_matrix8<T> &a,
                                          const simdgroup_matrix8<T> &b,
                                          const simdgroup_matrix8<T> &c) {
  simdgroup_matrix8<T> out;
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 8; ++j) {
      T acc = c.e[i][j];
      for (int k = 0; k < 8; ++k) acc = acc + a.e[i][k] * b.e[k][j];
      out.e[i][j] = acc;
    }
  d = out;
}

template <class T>
inline void simdgroup_multiply(simdgroup_matrix8<T> &d,
                               const simdgroup_matrix8<T> &a,
                               const simdgroup_matrix8<T> &b) {
  simdgroup_matrix8<T> z{};
  simdgroup_multiply_accumulate(d, a, b, z);
}

// Sum over the 32 lanes of the simdgroup, in lane order.
inline float simd_sum(float x) {
  g_simd_scratch[g_simd_lane] = x;
  simd_sync();
  float s = 0.0f;
  for (int l = 0; l < 32; ++l) s = s + g_simd_scratch[l];
  simd_sync();
  return s;
}

}  // namespace metal

