// qmv_util.cuh -- device helpers shared by the decode GEMV kernels: code unpacking
// and the RMSNorm / SwiGLU transforms applied to x while it is staged.
#pragma once
#include "kernels.cuh"

namespace vmlx {

// Unpack one 8-bit word (4 consecutive k) into two bf16 pairs holding q exactly
// (the 2^23 float trick, then a packed convert; q <= 255 is exact in bf16).
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t (&p)[2]) {
  const float MAGIC = 8388608.0f;
  const uint32_t K4B = 0x4B000000u;
  float f0 = __uint_as_float(prmt(w, K4B, 0x7540)) - MAGIC;
  float f1 = __uint_as_float(prmt(w, K4B, 0x7541)) - MAGIC;
  float f2 = __uint_as_float(prmt(w, K4B, 0x7542)) - MAGIC;
  float f3 = __uint_as_float(prmt(w, K4B, 0x7543)) - MAGIC;
  p[0] = bf162_as_u32(__floats2bfloat162_rn(f0, f1));
  p[1] = bf162_as_u32(__floats2bfloat162_rn(f2, f3));
}

__device__ __forceinline__ unsigned long long pack_f2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ unsigned long long pack_u2(uint32_t a, uint32_t b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float2 unpack_f2(unsigned long long v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
// acc.xy += a.xy * b.xy (packed fp32 FMA, sm_100)
__device__ __forceinline__ void ffma2(unsigned long long& acc, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

// RMSNorm applied to 8 consecutive bf16 of x at column k0 (same rounding as
// rms_norm_kernel: n = bf16(x * inv), out = bf16(w * n)).
__device__ __forceinline__ uint4 norm8(uint4 v, float inv, const bf16* w) {
  const uint4 ww = *reinterpret_cast<const uint4*>(w);
  const uint32_t u[4] = {v.x, v.y, v.z, v.w}, wu[4] = {ww.x, ww.y, ww.z, ww.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
    const float2 n = __bfloat1622float2(__floats2bfloat162_rn(f.x * inv, f.y * inv));
    const float2 wf = __bfloat1622float2(u32_as_bf162(wu[j]));
    o[j] = bf162_as_u32(__floats2bfloat162_rn(wf.x * n.x, wf.y * n.y));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
__device__ __forceinline__ uint2 norm4(uint2 v, float inv, const bf16* w) {
  const uint2 ww = *reinterpret_cast<const uint2*>(w);
  const uint32_t u[2] = {v.x, v.y}, wu[2] = {ww.x, ww.y};
  uint32_t o[2];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
    const float2 n = __bfloat1622float2(__floats2bfloat162_rn(f.x * inv, f.y * inv));
    const float2 wf = __bfloat1622float2(u32_as_bf162(wu[j]));
    o[j] = bf162_as_u32(__floats2bfloat162_rn(wf.x * n.x, wf.y * n.y));
  }
  return make_uint2(o[0], o[1]);
}

// SwiGLU of a gate||up row on load: bf16(bf16(silu(g)) * u), the rounding of
// compiledSwiGLU and of the standalone silu_mul kernel.
__device__ __forceinline__ uint32_t swiglu2(uint32_t g, uint32_t u) {
  const float2 gf = __bfloat1622float2(u32_as_bf162(g)), uf = __bfloat1622float2(u32_as_bf162(u));
  const float s0 = __bfloat162float(__float2bfloat16_rn(gf.x / (1.f + __expf(-gf.x))));
  const float s1 = __bfloat162float(__float2bfloat16_rn(gf.y / (1.f + __expf(-gf.y))));
  return bf162_as_u32(__floats2bfloat162_rn(s0 * uf.x, s1 * uf.y));
}
// 8 (or 4) x values at xrow[off]: plain, or the SwiGLU of gate xrow[off] and up xrow[K + off]
__device__ __forceinline__ uint4 load_x8(const QmvArgs& p, const bf16* xrow) {
  const uint4 v = *reinterpret_cast<const uint4*>(xrow);
  if (!p.x_swiglu) return v;
  const uint4 u = *reinterpret_cast<const uint4*>(xrow + p.K);
  return make_uint4(swiglu2(v.x, u.x), swiglu2(v.y, u.y), swiglu2(v.z, u.z), swiglu2(v.w, u.w));
}
__device__ __forceinline__ uint2 load_x4(const QmvArgs& p, const bf16* xrow) {
  const uint2 v = *reinterpret_cast<const uint2*>(xrow);
  if (!p.x_swiglu) return v;
  const uint2 u = *reinterpret_cast<const uint2*>(xrow + p.K);
  return make_uint2(swiglu2(v.x, u.x), swiglu2(v.y, u.y));
}

}  // namespace vmlx
