// Runtime for WGSL compute shaders translated to C++ by oracle/wgsl2cpp.py.
// TEST INFRASTRUCTURE ONLY: it runs the reference's own shader sources on the host cores
// so that the oracle restatement can be checked against them. Nothing in the product
// links or loads it.
//
// What it provides:
//   * the WGSL value types: f32/u32/i32, vec2/vec3/vec4<T>, mat4x4<T>, array<T, N>, and
//     Buf<T> for runtime-sized storage arrays, with the WGSL operators;
//   * the builtins the translated shaders call (W_exp, W_inverseSqrt, W_pack2x16float ...);
//     transcendentals come from the host libm in f32, as in oracle/oracle.cpp;
//   * a dispatcher: the invocations of a workgroup run as fibers on one host thread,
//     workgroupBarrier() as a switch back to a scheduler that releases them together;
//     workgroups run on several host threads at once (workgroup memory is per thread and
//     zeroed before each workgroup, as WGSL zero-initializes it).
// Out-of-bounds array or buffer accesses, which WGSL would clamp or discard, are
// recorded (the dispatch then fails) so a harness mistake is never mistaken for a result.
#pragma once
#include <atomic>
#include <ucontext.h>

#include <algorithm>
#include <memory>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <thread>
#include <type_traits>
#include <vector>

namespace wgsl {

using f32 = float;
using u32 = uint32_t;
using i32 = int32_t;

inline std::atomic<uint64_t> g_oob{0};
inline void oob() { g_oob.fetch_add(1, std::memory_order_relaxed); }

template <class T>
struct vec2 {
  T x{}, y{};
  vec2() = default;
  explicit vec2(T s) : x(s), y(s) {}
  vec2(T a, T b) : x(a), y(b) {}
  T& operator[](u32 i) { return i == 0 ? x : (i == 1 ? y : (oob(), y)); }
  const T& operator[](u32 i) const { return i == 0 ? x : (i == 1 ? y : (oob(), y)); }
};
template <class T>
struct vec3 {
  T x{}, y{}, z{};
  vec3() = default;
  explicit vec3(T s) : x(s), y(s), z(s) {}
  vec3(T a, T b, T c) : x(a), y(b), z(c) {}
  T& operator[](u32 i) { return i == 0 ? x : i == 1 ? y : i == 2 ? z : (oob(), z); }
  const T& operator[](u32 i) const { return i == 0 ? x : i == 1 ? y : i == 2 ? z : (oob(), z); }
};
template <class T>
struct vec4 {
  T x{}, y{}, z{}, w{};
  vec4() = default;
  explicit vec4(T s) : x(s), y(s), z(s), w(s) {}
  vec4(T a, T b, T c, T d) : x(a), y(b), z(c), w(d) {}
  T& operator[](u32 i) { return i == 0 ? x : i == 1 ? y : i == 2 ? z : i == 3 ? w : (oob(), w); }
  const T& operator[](u32 i) const { return i == 0 ? x : i == 1 ? y : i == 2 ? z : i == 3 ? w : (oob(), w); }
};
static_assert(sizeof(vec4<u32>) == 16 && sizeof(vec4<f32>) == 16, "vec4 is 16 bytes in storage");

// Component-wise arithmetic, vector-vector and vector-scalar (both orders).
#define WGSL_VEC_OPS(V, N, ...)                                                                  \
  template <class T> V<T> operator+(V<T> a, V<T> b) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] + b[i]; return r; } \
  template <class T> V<T> operator-(V<T> a, V<T> b) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] - b[i]; return r; } \
  template <class T> V<T> operator*(V<T> a, V<T> b) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] * b[i]; return r; } \
  template <class T> V<T> operator/(V<T> a, V<T> b) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] / b[i]; return r; } \
  template <class T, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> V<T> operator*(V<T> a, S s) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] * (T)s; return r; } \
  template <class T, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> V<T> operator*(S s, V<T> a) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = (T)s * a[i]; return r; } \
  template <class T, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> V<T> operator/(V<T> a, S s) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] / (T)s; return r; } \
  template <class T, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> V<T> operator+(V<T> a, S s) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] + (T)s; return r; } \
  template <class T, class S, class = std::enable_if_t<std::is_arithmetic_v<S>>> V<T> operator-(V<T> a, S s) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = a[i] - (T)s; return r; } \
  template <class T> V<T> operator-(V<T> a) { V<T> r; for (u32 i = 0; i < N; i++) r[i] = -a[i]; return r; } \
  template <class T, class B> V<T>& operator+=(V<T>& a, B b) { a = a + b; return a; } \
  template <class T, class B> V<T>& operator-=(V<T>& a, B b) { a = a - b; return a; } \
  template <class T, class B> V<T>& operator*=(V<T>& a, B b) { a = a * b; return a; } \
  template <class T, class B> V<T>& operator/=(V<T>& a, B b) { a = a / b; return a; }
WGSL_VEC_OPS(vec2, 2)
WGSL_VEC_OPS(vec3, 3)
WGSL_VEC_OPS(vec4, 4)
#undef WGSL_VEC_OPS

// mat4x4<T>: four column vectors; m[j] is column j.
template <class T>
struct mat4x4 {
  vec4<T> c[4];
  mat4x4() = default;
  mat4x4(vec4<T> a, vec4<T> b, vec4<T> d, vec4<T> e) : c{a, b, d, e} {}
  vec4<T>& operator[](u32 j) { return j < 4 ? c[j] : (oob(), c[3]); }
  const vec4<T>& operator[](u32 j) const { return j < 4 ? c[j] : (oob(), c[3]); }
};
template <class T> mat4x4<T> operator+(mat4x4<T> a, const mat4x4<T>& b) {
  for (u32 j = 0; j < 4; j++) a.c[j] = a.c[j] + b.c[j];
  return a;
}
template <class T> mat4x4<T>& operator+=(mat4x4<T>& a, const mat4x4<T>& b) { a = a + b; return a; }

// Fixed-size arrays (function-scope, workgroup, values).
template <class T, u32 N>
struct array {
  T v[N]{};
  array() = default;
  template <class... A, class = std::enable_if_t<sizeof...(A) == N && (N > 1 || sizeof...(A) == 1)>>
  array(A... a) : v{T(a)...} {}
  T& operator[](u32 i) { return i < N ? v[i] : (oob(), v[N - 1]); }
  const T& operator[](u32 i) const { return i < N ? v[i] : (oob(), v[N - 1]); }
};

// Runtime-sized storage buffer binding.
template <class T>
struct Buf {
  T* p = nullptr;
  uint64_t n = 0;
  T& operator[](uint64_t i) {
    static T dummy{};
    if (i >= n) { oob(); return dummy; }
    return p[i];
  }
};

// ---- builtins ----
inline f32 W_exp(f32 v) { return expf(v); }
inline f32 W_log(f32 v) { return logf(v); }
inline f32 W_pow(f32 a, f32 b) { return powf(a, b); }
inline f32 W_sin(f32 v) { return sinf(v); }
inline f32 W_cos(f32 v) { return cosf(v); }
inline f32 W_tanh(f32 v) { return tanhf(v); }
inline f32 W_sqrt(f32 v) { return sqrtf(v); }
inline f32 W_inverseSqrt(f32 v) { return 1.0f / sqrtf(v); }
inline f32 W_abs(f32 v) { return fabsf(v); }
template <class A, class B> inline std::common_type_t<A, B> W_max(A a, B b) {
  using T = std::common_type_t<A, B>;
  return (T)a < (T)b ? (T)b : (T)a;
}
template <class A, class B> inline std::common_type_t<A, B> W_min(A a, B b) {
  using T = std::common_type_t<A, B>;
  return (T)b < (T)a ? (T)b : (T)a;
}
template <class T, class L, class H> inline T W_clamp(T v, L lo, H hi) { return W_min(W_max(v, (T)lo), (T)hi); }
template <class T> inline T W_select(T f, T t, bool c) { return c ? t : f; }
template <class T> inline T W_dot(vec2<T> a, vec2<T> b) { return a.x * b.x + a.y * b.y; }
template <class T> inline T W_dot(vec3<T> a, vec3<T> b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
template <class T> inline T W_dot(vec4<T> a, vec4<T> b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

// f32 -> f16 bits, round to nearest even (IEEE 754 binary16), and back.
inline uint16_t f32_to_f16(f32 f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520: infinity
  if (ax < 0x38800000u) {                                     // below the smallest normal half
    const float a = std::fabs(f);
    // subnormal halves are multiples of 2^-24; nearbyint rounds half to even
    const float q = std::nearbyint(a * 16777216.0f);
    return (uint16_t)(sign | (uint32_t)q);
  }
  const uint32_t mant = ax & 0x7fffffu;
  uint32_t h = ((ax >> 23) - 112u) << 10 | (mant >> 13);
  const uint32_t rest = mant & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}
inline f32 f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    const float v = std::ldexp((float)m, -24);
    std::memcpy(&x, &v, 4);
    x |= sign;
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  f32 r;
  std::memcpy(&r, &x, 4);
  return r;
}
inline u32 W_pack2x16float(vec2<f32> v) { return (u32)f32_to_f16(v.x) | ((u32)f32_to_f16(v.y) << 16); }
inline vec2<f32> W_unpack2x16float(u32 w) { return vec2<f32>(f16_to_f32((uint16_t)(w & 0xffffu)), f16_to_f32((uint16_t)(w >> 16))); }

// ---- dispatch ----
struct Builtins {
  vec3<u32> global_invocation_id, local_invocation_id, workgroup_id, num_workgroups;
  u32 local_invocation_index;
};

// The invocations of one workgroup run as fibers (ucontext) on one host thread:
// workgroupBarrier() switches back to the scheduler, which resumes every invocation only
// after all of them have reached the barrier (or returned). Workgroup variables are
// thread_local, so host threads run different workgroups at the same time, as a GPU does.
struct FiberSet {
  static constexpr size_t kStack = 64 * 1024;
  u32 W = 0, cur = 0;
  std::vector<ucontext_t> ctx;
  std::vector<std::unique_ptr<char[]>> stk;
  std::vector<uint8_t> done;
  std::vector<Builtins> bi;
  ucontext_t main{};
  const std::function<void(const Builtins&)>* entry = nullptr;
  explicit FiberSet(u32 w) : W(w), ctx(w), done(w), bi(w) {
    for (u32 i = 0; i < w; i++) stk.emplace_back(new char[kStack]);
  }
};
inline thread_local FiberSet* tl_fs = nullptr;
inline void fiber_main() {
  FiberSet* fs = tl_fs;
  const u32 i = fs->cur;
  (*fs->entry)(fs->bi[i]);
  fs->done[i] = 1;  // uc_link returns to the scheduler
}
inline void W_workgroupBarrier() {
  FiberSet* fs = tl_fs;
  swapcontext(&fs->ctx[fs->cur], &fs->main);
}
inline void W_storageBarrier() { W_workgroupBarrier(); }

// Runs entry over the grid; zero_wg clears the calling thread's workgroup variables.
// Returns the number of out-of-bounds accesses seen (0 on success).
inline uint64_t dispatch(const std::function<void(const Builtins&)>& entry, const std::function<void()>& zero_wg,
                         u32 gx, u32 gy, u32 gz, u32 wx, u32 wy, u32 wz) {
  g_oob.store(0);
  const u32 W = wx * wy * wz;
  const uint64_t nwg = (uint64_t)gx * gy * gz;
  std::atomic<uint64_t> next{0};
  auto worker = [&]() {
    FiberSet fs(W);
    fs.entry = &entry;
    tl_fs = &fs;
    for (;;) {
      const uint64_t g = next.fetch_add(1);
      if (g >= nwg) break;
      const u32 x = (u32)(g % gx), y = (u32)((g / gx) % gy), z = (u32)(g / ((uint64_t)gx * gy));
      zero_wg();
      for (u32 i = 0; i < W; i++) {
        Builtins& b = fs.bi[i];
        b.local_invocation_index = i;
        b.local_invocation_id = vec3<u32>(i % wx, (i / wx) % wy, i / (wx * wy));
        b.num_workgroups = vec3<u32>(gx, gy, gz);
        b.workgroup_id = vec3<u32>(x, y, z);
        b.global_invocation_id = vec3<u32>(x * wx + b.local_invocation_id.x, y * wy + b.local_invocation_id.y,
                                           z * wz + b.local_invocation_id.z);
        getcontext(&fs.ctx[i]);
        fs.ctx[i].uc_stack.ss_sp = fs.stk[i].get();
        fs.ctx[i].uc_stack.ss_size = FiberSet::kStack;
        fs.ctx[i].uc_link = &fs.main;
        makecontext(&fs.ctx[i], fiber_main, 0);
        fs.done[i] = 0;
      }
      // One pass runs every live invocation to its next barrier or its end.
      for (bool live = true; live;) {
        live = false;
        for (u32 i = 0; i < W; i++) {
          if (fs.done[i]) continue;
          fs.cur = i;
          swapcontext(&fs.main, &fs.ctx[i]);
          live = true;
        }
      }
    }
    tl_fs = nullptr;
  };
  const u32 hw = std::max(1u, std::thread::hardware_concurrency());
  const u32 T = (u32)std::min<uint64_t>(std::min<u32>(hw, 16), nwg);
  std::vector<std::thread> th;
  for (u32 t = 1; t < T; t++) th.emplace_back(worker);
  worker();
  for (auto& t : th) t.join();
  return g_oob.load();
}

}  // namespace wgsl
