// Host C++ stand-ins for the Metal Shading Language 3.1 vocabulary, so that the
// reference's serial kernel functions (pure integer / float32 code) compile with
// g++ and can be called on the CPU as an independent cross-check of the oracle.
//
// TEST INFRASTRUCTURE ONLY. Nothing in the product links this. Only the
// functions that are serial in the reference (one thread does the whole job,
// no SIMD-group or threadgroup cooperation for the outputs that are read) are
// ever called through it; the SIMD/atomic stand-ins below give single-lane,
// single-thread semantics so that the surrounding file parses and those
// serial functions run unchanged.
//
// Address spaces: `device` and `thread` vanish. `threadgroup` becomes
// `volatile` where the reference overloads on device vs threadgroup pointers
// (the add64 pair at the top of boost.metal) and vanishes elsewhere; the
// wrapper headers in wrap/ switch it at the reference's own #include points.
// Kernels become function templates with a defaulted parameter, so the ones
// the harness never calls are parsed but not instantiated.
#pragma once
#include <algorithm>
#include <atomic>
#include <bit>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <type_traits>

// Address spaces and function qualifiers.
#define kernel template <class ShimKernel = void>
#define device
#define thread
#define threadgroup volatile
#define constant const
#define METAL_FUNC inline

using uchar = std::uint8_t;
using ushort = std::uint16_t;
using uint = std::uint32_t;
using ulong = std::uint64_t;
// IEEE binary16 storage with a widening conversion (only parsed by the harness).
struct half {
  ushort bits;
  operator float() const {
    uint sign = uint(bits & 0x8000u) << 16, e = (bits >> 10) & 31, m = bits & 0x3ffu;
    uint out;
    if (e == 31) out = sign | 0x7f800000u | (m << 13);
    else if (e) out = sign | ((e + 112) << 23) | (m << 13);
    else if (!m) out = sign;
    else {
      int shift = std::countl_zero(m) - 21;
      out = sign | (uint(113 - shift) << 23) | (((m << shift) & 0x3ffu) << 13);
    }
    float f;
    std::memcpy(&f, &out, 4);
    return f;
  }
};

template <class T, int N>
struct vec;

// Read-only two-component swizzle (.xy, .zw, .yz, .yx) overlaid on a vector.
template <class T, int N, int I, int J>
struct swizzle2 {
  T v[N];
  operator vec<T, 2>() const;
};

// Metal vectors: two components align to their size, three and four components
// to four times the component size (a three-component vector has a pad lane).
template <class T>
struct alignas(2 * sizeof(T)) vec<T, 2> {
  union {
    struct { T x, y; };
    swizzle2<T, 2, 1, 0> yx;
  };
  constexpr vec() : x(), y() {}
  constexpr vec(T s) : x(s), y(s) {}
  template <class A, class B>
  constexpr vec(A a, B b) : x(T(a)), y(T(b)) {}
  template <class U>
  explicit constexpr vec(vec<U, 2> o) : x(T(o.x)), y(T(o.y)) {}
  constexpr vec(const vec& o) : x(o.x), y(o.y) {}
  vec(const volatile vec& o) : x(o.x), y(o.y) {}
  vec(const volatile vec&& o) : x(o.x), y(o.y) {}
  vec& operator=(const vec& o) { x = o.x; y = o.y; return *this; }
  void operator=(const vec& o) volatile { x = o.x; y = o.y; }
  T& operator[](int i) { return i ? y : x; }
  T operator[](int i) const { return i ? y : x; }
};
template <class T>
struct alignas(4 * sizeof(T)) vec<T, 3> {
  T x, y, z, pad_;
  constexpr vec() : x(), y(), z(), pad_() {}
  constexpr vec(T s) : x(s), y(s), z(s), pad_() {}
  template <class A, class B, class C>
  constexpr vec(A a, B b, C c) : x(T(a)), y(T(b)), z(T(c)), pad_() {}
  template <class U>
  explicit constexpr vec(vec<U, 3> o) : x(T(o.x)), y(T(o.y)), z(T(o.z)), pad_() {}
  constexpr vec(const vec& o) = default;
  vec(const volatile vec& o) : x(o.x), y(o.y), z(o.z), pad_() {}
  vec(const volatile vec&& o) : x(o.x), y(o.y), z(o.z), pad_() {}
  vec& operator=(const vec&) = default;
  void operator=(const vec& o) volatile { x = o.x; y = o.y; z = o.z; }
  T& operator[](int i) { return i == 0 ? x : i == 1 ? y : z; }
  T operator[](int i) const { return i == 0 ? x : i == 1 ? y : z; }
};
template <class T>
struct alignas(4 * sizeof(T)) vec<T, 4> {
  union {
    struct { T x, y, z, w; };
    swizzle2<T, 4, 0, 1> xy;
    swizzle2<T, 4, 2, 3> zw;
    swizzle2<T, 4, 1, 2> yz;
  };
  constexpr vec() : x(), y(), z(), w() {}
  constexpr vec(T s) : x(s), y(s), z(s), w(s) {}
  template <class A, class B, class C, class D>
  constexpr vec(A a, B b, C c, D d) : x(T(a)), y(T(b)), z(T(c)), w(T(d)) {}
  template <class A>
  constexpr vec(A a, vec<T, 3> b) : x(T(a)), y(b.x), z(b.y), w(b.z) {}
  template <class U>
  constexpr vec(vec<U, 2> a, vec<U, 2> b) : x(T(a.x)), y(T(a.y)), z(T(b.x)), w(T(b.y)) {}
  template <class U>
  explicit constexpr vec(vec<U, 4> o) : x(T(o.x)), y(T(o.y)), z(T(o.z)), w(T(o.w)) {}
  constexpr vec(const vec& o) : x(o.x), y(o.y), z(o.z), w(o.w) {}
  vec(const volatile vec& o) : x(o.x), y(o.y), z(o.z), w(o.w) {}
  vec(const volatile vec&& o) : x(o.x), y(o.y), z(o.z), w(o.w) {}
  vec& operator=(const vec& o) { x = o.x; y = o.y; z = o.z; w = o.w; return *this; }
  void operator=(const vec& o) volatile { x = o.x; y = o.y; z = o.z; w = o.w; }
  T& operator[](int i) { return i == 0 ? x : i == 1 ? y : i == 2 ? z : w; }
  T operator[](int i) const { return i == 0 ? x : i == 1 ? y : i == 2 ? z : w; }
};
template <class T, int N, int I, int J>
inline swizzle2<T, N, I, J>::operator vec<T, 2>() const { return vec<T, 2>(v[I], v[J]); }

#define SHIM_BINOP(op)                                                            \
  template <class T, int N>                                                       \
  inline vec<T, N> operator op(vec<T, N> a, vec<T, N> b) {                        \
    for (int i = 0; i < N; ++i) a[i] = T(a[i] op b[i]);                           \
    return a;                                                                     \
  }                                                                               \
  template <class T, int N, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> \
  inline vec<T, N> operator op(vec<T, N> a, S b) {                                \
    for (int i = 0; i < N; ++i) a[i] = T(a[i] op T(b));                           \
    return a;                                                                     \
  }                                                                               \
  template <class T, int N, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> \
  inline vec<T, N> operator op(S a, vec<T, N> b) {                                \
    for (int i = 0; i < N; ++i) b[i] = T(T(a) op b[i]);                           \
    return b;                                                                     \
  }                                                                               \
  template <class T, int N, class R>                                              \
  inline vec<T, N>& operator op##=(vec<T, N>& a, R b) {                           \
    a = a op b;                                                                   \
    return a;                                                                     \
  }                                                                               \
  template <class T, int N, class R>                                              \
  inline void operator op##=(volatile vec<T, N>& a, R b) {                        \
    vec<T, N> t(a);                                                               \
    a = t op b;                                                                   \
  }
SHIM_BINOP(+)
SHIM_BINOP(-)
SHIM_BINOP(*)
SHIM_BINOP(/)
SHIM_BINOP(&)
SHIM_BINOP(|)
SHIM_BINOP(^)
SHIM_BINOP(<<)
SHIM_BINOP(>>)
#undef SHIM_BINOP
template <class T, int N>
inline vec<T, N> operator-(vec<T, N> a) {
  for (int i = 0; i < N; ++i) a[i] = -a[i];
  return a;
}
template <class T, int N>
inline vec<T, N> operator~(vec<T, N> a) {
  for (int i = 0; i < N; ++i) a[i] = ~a[i];
  return a;
}
#define SHIM_CMP(op)                                                   \
  template <class T, int N>                                            \
  inline vec<bool, N> operator op(vec<T, N> a, vec<T, N> b) {          \
    vec<bool, N> r;                                                    \
    for (int i = 0; i < N; ++i) r[i] = a[i] op b[i];                   \
    return r;                                                          \
  }
template <class T, int N>
inline T dot(vec<T, N> a, vec<T, N> b) {
  T r = 0;
  for (int i = 0; i < N; ++i) r += a[i] * b[i];
  return r;
}
template <class T, int N>
inline vec<T, N> ldexp(vec<T, N> v, vec<int, N> e) {
  for (int i = 0; i < N; ++i) v[i] = std::ldexp(v[i], e[i]);
  return v;
}
SHIM_CMP(==)
SHIM_CMP(!=)
SHIM_CMP(<)
SHIM_CMP(<=)
SHIM_CMP(>)
SHIM_CMP(>=)
#undef SHIM_CMP

#define SHIM_VEC(name, T)  \
  using name##2 = vec<T, 2>; \
  using name##3 = vec<T, 3>; \
  using name##4 = vec<T, 4>;
SHIM_VEC(float, float)
SHIM_VEC(int, int)
SHIM_VEC(uint, std::uint32_t)
SHIM_VEC(long, std::int64_t)
SHIM_VEC(ulong, std::uint64_t)
SHIM_VEC(bool, bool)
SHIM_VEC(uchar, std::uint8_t)
SHIM_VEC(ushort, std::uint16_t)
SHIM_VEC(short, std::int16_t)
#undef SHIM_VEC

template <int N>
inline bool all(vec<bool, N> v) {
  for (int i = 0; i < N; ++i)
    if (!v[i]) return false;
  return true;
}
template <int N>
inline bool any(vec<bool, N> v) {
  for (int i = 0; i < N; ++i)
    if (v[i]) return true;
  return false;
}
inline bool all(bool v) { return v; }
inline bool any(bool v) { return v; }

// as_type<T>: a bit cast between equally sized scalars or vectors.
template <class To, class From>
inline To as_type(From v) {
  static_assert(sizeof(To) == sizeof(From), "as_type size mismatch");
  To out;
  std::memcpy(&out, &v, sizeof(To));
  return out;
}

// Integer intrinsics with Metal's definitions (clz(0) is the bit width).
inline uint clz(uint v) { return v ? uint(std::countl_zero(v)) : 32u; }
inline ulong clz(ulong v) { return v ? ulong(std::countl_zero(v)) : 64u; }
inline int clz(int v) { return int(clz(uint(v))); }
inline long clz(long v) { return long(clz(ulong(v))); }
inline uint ctz(uint v) { return v ? uint(std::countr_zero(v)) : 32u; }
inline ulong ctz(ulong v) { return v ? ulong(std::countr_zero(v)) : 64u; }
inline uint popcount(uint v) { return uint(std::popcount(v)); }
inline ulong popcount(ulong v) { return ulong(std::popcount(v)); }
inline ulong mulhi(ulong a, ulong b) { return ulong((unsigned __int128)a * b >> 64); }
inline uint mulhi(uint a, uint b) { return uint((ulong)a * b >> 32); }

// Scalar helpers. Metal's min/max/clamp take one type; mixed literal calls in
// the reference rely on implicit conversion to the non-literal argument.
template <class T, class U>
inline auto min(T a, U b) -> std::common_type_t<T, U> {
  using C = std::common_type_t<T, U>;
  return C(b) < C(a) ? C(b) : C(a);
}
template <class T, class U>
inline auto max(T a, U b) -> std::common_type_t<T, U> {
  using C = std::common_type_t<T, U>;
  return C(a) < C(b) ? C(b) : C(a);
}
inline float min(float a, float b) { return std::fmin(a, b); }
inline float max(float a, float b) { return std::fmax(a, b); }
template <class T, int N>
inline vec<T, N> min(vec<T, N> a, vec<T, N> b) {
  for (int i = 0; i < N; ++i) a[i] = min(a[i], b[i]);
  return a;
}
template <class T, int N>
inline vec<T, N> max(vec<T, N> a, vec<T, N> b) {
  for (int i = 0; i < N; ++i) a[i] = max(a[i], b[i]);
  return a;
}
template <class T, class L, class H>
inline T clamp(T v, L lo, H hi) {
  return min(max(v, T(lo)), T(hi));
}
inline float fabs(float v) { return std::fabs(v); }
inline float rint(float v) { return std::nearbyint(v); }
inline double rint(double v) { return std::nearbyint(v); }
inline float fma(float a, float b, float c) { return std::fma(a, b, c); }
inline float ldexp(float v, int e) { return std::ldexp(v, e); }
inline float frexp(float v, int& e) { return std::frexp(v, &e); }
using std::isfinite;
using std::isinf;
using std::isnan;
inline float exp(float v) { return std::exp(v); }
inline float log(float v) { return std::log(v); }
inline float sqrt(float v) { return std::sqrt(v); }
inline float floor(float v) { return std::floor(v); }
inline float ceil(float v) { return std::ceil(v); }
inline float trunc(float v) { return std::trunc(v); }
inline float copysign(float a, float b) { return std::copysign(a, b); }
template <class T>
inline T select(T a, T b, bool c) { return c ? b : a; }

#ifndef INFINITY
#define INFINITY (std::numeric_limits<float>::infinity())
#endif
#ifndef NAN
#define NAN (std::numeric_limits<float>::quiet_NaN())
#endif
#ifndef FLT_MAX
#define FLT_MAX (std::numeric_limits<float>::max())
#endif

// Atomics: only ever touched by cooperative kernels, which the harness never
// runs; sequential semantics suffice for parsing and for single-thread use.
using atomic_uint = uint;
using atomic_int = int;
enum memory_order { memory_order_relaxed };
template <class T, class V>
inline T atomic_fetch_add_explicit(T* p, V v, memory_order) {
  T old = *p;
  *p = T(old + T(v));
  return old;
}
template <class T, class V>
inline T atomic_fetch_or_explicit(T* p, V v, memory_order) {
  T old = *p;
  *p = T(old | T(v));
  return old;
}
template <class T, class V>
inline T atomic_fetch_max_explicit(T* p, V v, memory_order) {
  T old = *p;
  *p = old < T(v) ? T(v) : old;
  return old;
}
template <class T, class V>
inline T atomic_fetch_min_explicit(T* p, V v, memory_order) {
  T old = *p;
  *p = T(v) < old ? T(v) : old;
  return old;
}
template <class T, class V>
inline void atomic_store_explicit(T* p, V v, memory_order) { *p = T(v); }
template <class T>
inline T atomic_load_explicit(const T* p, memory_order) { return *p; }
template <class T, class V>
inline bool atomic_compare_exchange_weak_explicit(T* p, T* expected, V desired, memory_order, memory_order) {
  if (*p == *expected) {
    *p = T(desired);
    return true;
  }
  *expected = *p;
  return false;
}

namespace mem_flags {
enum flags { mem_none = 0, mem_device = 1, mem_threadgroup = 2 };
}
inline mem_flags::flags operator|(mem_flags::flags a, mem_flags::flags b) {
  return mem_flags::flags(int(a) | int(b));
}
// Barriers and SIMD-group operations with single-lane semantics: each call
// behaves as if its SIMD group held only the calling thread. The harness calls
// only kernels whose per-thread outputs do not depend on other lanes (their
// SIMD use feeds flags or certificates that the harness ignores), and runs
// them one thread at a time.
inline void threadgroup_barrier(mem_flags::flags) {}
inline void simdgroup_barrier(mem_flags::flags) {}
template <class T> inline T simd_sum(T v) { return v; }
template <class T> inline T simd_min(T v) { return v; }
template <class T> inline T simd_max(T v) { return v; }
template <class T> inline T simd_or(T v) { return v; }
template <class T> inline T simd_and(T v) { return v; }
template <class T> inline T simd_xor(T v) { return v; }
template <class T> inline T simd_prefix_exclusive_sum(T) { return T(0); }
template <class T> inline T simd_prefix_inclusive_sum(T v) { return v; }
template <class T> inline T simd_broadcast_first(T v) { return v; }
template <class T, class U> inline T simd_shuffle(T v, U) { return v; }
template <class T, class U> inline T simd_shuffle_up(T v, U) { return v; }
template <class T, class U> inline T simd_shuffle_down(T v, U) { return v; }
template <class T, class U> inline T simd_shuffle_xor(T v, U) { return v; }
template <class T, class U> inline T simd_broadcast(T v, U) { return v; }
inline bool simd_is_first() { return true; }
inline bool simd_any(bool v) { return v; }
inline bool simd_all(bool v) { return v; }
struct simd_vote {
  using vote_t = ulong;
  vote_t bits;
  explicit simd_vote(vote_t b) : bits(b) {}
  explicit operator vote_t() const { return bits; }
  bool all() const { return bits & 1; }
  bool any() const { return bits & 1; }
};
inline simd_vote simd_ballot(bool v) { return simd_vote(v ? 1 : 0); }
