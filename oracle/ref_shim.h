// ref_shim.h -- the host environment in which oracle/_ref compiles the reference's own
// Metal source text for the affine quantize / dequantize / qmv_fast kernels as C++.
//
// TEST INFRASTRUCTURE ONLY: nothing in the product library includes or links this.
//
// What it provides (all written for this checker, nothing taken from Apple's headers):
//  * the Metal address-space qualifiers and function attributes as no-ops;
//  * the vector index types the kernels take (uint2, uint3);
//  * `bfloat16_t` -- a bf16 storage type whose arithmetic follows Metal's rules for
//    `bfloat`: bfloat op bfloat (or op an integer) is computed in float and rounded
//    to bf16 (round to nearest even); bfloat op float promotes to float;
//  * min / max / round / abs for float, and Limits<T>::max;
//  * the SIMD-group collectives simd_min / simd_max / simd_sum / simd_shuffle_down.
//    A SIMD group is 32 cooperative fibers (ucontext) on one OS thread: each lane runs
//    the kernel body until it reaches a collective, and the collective completes once
//    all 32 lanes have arrived.  simd_sum adds in lane order (Metal leaves the order
//    unspecified), so sums are compared within fp32 tolerance, not bit for bit.
#pragma once

#include <ucontext.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <type_traits>

#define device
#define thread
#define threadgroup
#define constant
#define METAL_FUNC inline

using std::abs;
using std::round;

inline float min(float a, float b) { return std::fmin(a, b); }
inline float max(float a, float b) { return std::fmax(a, b); }

namespace metal {
template <bool B, class T, class F>
using conditional_t = typename std::conditional<B, T, F>::type;
}

struct uint2 {
  uint32_t x, y;
};
struct uint3 {
  uint32_t x, y, z;
};

struct bfloat16_t {
  uint16_t bits;
  bfloat16_t() : bits(0) {}
  bfloat16_t(float f) { bits = from_float(f); }
  operator float() const {
    uint32_t u = (uint32_t)bits << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  }
  static uint16_t from_float(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
    const uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
  }
};

#define VMLX_BF_OP(op)                                                                             \
  inline bfloat16_t operator op(bfloat16_t a, bfloat16_t b) { return bfloat16_t((float)a op(float) b); } \
  template <class I, class = typename std::enable_if<std::is_integral<I>::value>::type>            \
  inline bfloat16_t operator op(bfloat16_t a, I b) {                                                \
    return bfloat16_t((float)a op(float) bfloat16_t((float)b));                                     \
  }                                                                                                 \
  template <class I, class = typename std::enable_if<std::is_integral<I>::value>::type>            \
  inline bfloat16_t operator op(I a, bfloat16_t b) {                                                \
    return bfloat16_t((float)bfloat16_t((float)a) op(float) b);                                     \
  }                                                                                                 \
  inline float operator op(bfloat16_t a, float b) { return (float)a op b; }                         \
  inline float operator op(float a, bfloat16_t b) { return a op(float) b; }
VMLX_BF_OP(+)
VMLX_BF_OP(-)
VMLX_BF_OP(*)
VMLX_BF_OP(/)
#undef VMLX_BF_OP

template <typename T>
struct Limits;
template <>
struct Limits<float> {
  static constexpr float max = 3.40282347e+38f;
};
template <>
struct Limits<bfloat16_t> {
  static constexpr float max = 3.38953139e+38f;  // largest finite bf16
};

// ---- SIMD-group emulation -------------------------------------------------------------

namespace simdemu {

constexpr int kLanes = 32;
constexpr size_t kStack = 256 * 1024;

struct Group {
  ucontext_t sched;
  ucontext_t lane_ctx[kLanes];
  char* stacks[kLanes] = {};
  bool done[kLanes];
  int cur = 0;
  int arrived = 0;
  double in[kLanes];
  double out[kLanes];
  const std::function<void(int)>* body = nullptr;
  ~Group() {
    for (auto* s : stacks) delete[] s;
  }
};

inline Group& group() {
  static thread_local Group g;
  return g;
}

inline void trampoline() {
  Group& g = group();
  (*g.body)(g.cur);
  g.done[g.cur] = true;
  // returning switches to uc_link (the scheduler)
}

// Run body(lane) for the 32 lanes of one SIMD group to completion.
inline void run(const std::function<void(int)>& body) {
  Group& g = group();
  g.body = &body;
  for (int l = 0; l < kLanes; l++) {
    if (!g.stacks[l]) g.stacks[l] = new char[kStack];
    getcontext(&g.lane_ctx[l]);
    g.lane_ctx[l].uc_stack.ss_sp = g.stacks[l];
    g.lane_ctx[l].uc_stack.ss_size = kStack;
    g.lane_ctx[l].uc_link = &g.sched;
    makecontext(&g.lane_ctx[l], (void (*)())trampoline, 0);
    g.done[l] = false;
  }
  bool all_done = false;
  while (!all_done) {
    g.arrived = 0;
    for (int l = 0; l < kLanes; l++) {
      if (g.done[l]) continue;
      g.cur = l;
      swapcontext(&g.sched, &g.lane_ctx[l]);
    }
    all_done = true;
    for (int l = 0; l < kLanes; l++) all_done &= g.done[l];
  }
}

// A collective: deposit this lane's value, yield until every lane has deposited,
// then the last lane to arrive computes every lane's result.
template <class F>
inline double collective(double v, F combine) {
  Group& g = group();
  const int me = g.cur;
  g.in[me] = v;
  g.arrived++;
  if (g.arrived == kLanes) combine(g.in, g.out);
  swapcontext(&g.lane_ctx[me], &g.sched);
  // resumed in the next scheduler pass, after all lanes arrived
  return g.out[me];
}

}  // namespace simdemu

inline float simd_sum(float v) {
  return (float)simdemu::collective(v, [](const double* in, double* out) {
    float s = 0.f;
    for (int l = 0; l < simdemu::kLanes; l++) s += (float)in[l];
    for (int l = 0; l < simdemu::kLanes; l++) out[l] = s;
  });
}
inline float simd_min(float v) {
  return (float)simdemu::collective(v, [](const double* in, double* out) {
    float s = (float)in[0];
    for (int l = 1; l < simdemu::kLanes; l++) s = std::fmin(s, (float)in[l]);
    for (int l = 0; l < simdemu::kLanes; l++) out[l] = s;
  });
}
inline float simd_max(float v) {
  return (float)simdemu::collective(v, [](const double* in, double* out) {
    float s = (float)in[0];
    for (int l = 1; l < simdemu::kLanes; l++) s = std::fmax(s, (float)in[l]);
    for (int l = 0; l < simdemu::kLanes; l++) out[l] = s;
  });
}
// Lane l reads lane l + delta; lanes past the end keep their own value.
template <class V>
inline V simd_shuffle_down(V v, int delta) {
  static thread_local int d;
  d = delta;
  return (V)simdemu::collective((double)v, [](const double* in, double* out) {
    for (int l = 0; l < simdemu::kLanes; l++) out[l] = l + d < simdemu::kLanes ? in[l + d] : in[l];
  });
}
