// quant.cu -- affine quantize / dequantize on sm_100a.
//
// Bit-exact with MLX's affine_quantize / affine_dequantize
// (Source/Cmlx/mlx-generated/metal/quantized.h:2393-2558): the same fp32
// min/max/edge rule, IEEE division, round-half-away-from-zero (roundf) and
// LSB-first packing.  This file must not be built with fast-math.
//
// Layout: one thread per group (groups are contiguous in a row-major matrix);
// it reads its g values, derives scale/bias and writes g*bits/32 packed words.
// Quantization runs at load time only, so the kernel is simple rather than
// bandwidth-tuned.
#include "common.cuh"

namespace vmlx {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<bf16>(bf16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ bf16 from_f32<bf16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T>
__device__ __forceinline__ float type_max();
template <>
__device__ __forceinline__ float type_max<float>() {
  return 3.402823466e+38f;
}
template <>
__device__ __forceinline__ float type_max<bf16>() {
  return __uint_as_float(0x7f7f0000u);
}

// One thread quantizes one group of GS values (GS in {32, 64, 128}).
template <typename T, int GS, int BITS>
__global__ void quantize_kernel(const T* __restrict__ w, uint32_t* __restrict__ wq,
                                T* __restrict__ scales, T* __restrict__ biases, int64_t n_groups) {
  int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gid >= n_groups) return;
  constexpr int PER = 32 / BITS;  // values per word
  constexpr float n_bins = (float)((1 << BITS) - 1);
  const float eps = 1e-7f;
  const T* src = w + gid * GS;
  float v[GS];
#pragma unroll
  for (int i = 0; i < GS; i++) v[i] = to_f32<T>(src[i]);
  float w_min = type_max<T>(), w_max = 0.0f;
#pragma unroll
  for (int i = 0; i < GS; i++) {
    w_min = fminf(w_min, v[i]);
    w_max = fmaxf(w_max, v[i]);
  }
  float scale = fmaxf(__fdiv_rn(w_max - w_min, n_bins), eps);
  bool side = fabsf(w_min) > fabsf(w_max);
  scale = side ? scale : -scale;
  float edge = side ? w_min : w_max;
  float q0 = roundf(__fdiv_rn(edge, scale));
  bool at_zero = q0 == 0.0f;
  scale = at_zero ? scale : __fdiv_rn(edge, q0);
  float bias = at_zero ? 0.0f : edge;
  scales[gid] = from_f32<T>(scale);
  biases[gid] = from_f32<T>(bias);
  uint32_t* dst = wq + gid * (GS / PER);
#pragma unroll
  for (int wi = 0; wi < GS / PER; wi++) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < PER; j++) {
      float q = fminf(roundf(__fdiv_rn(__fsub_rn(v[wi * PER + j], bias), scale)), n_bins);
      uint32_t c = q > 0.0f ? (uint32_t)q : 0u;  // saturating float -> uint8
      word |= c << (BITS * j);
    }
    dst[wi] = word;
  }
}

// One thread dequantizes one packed word.
template <typename TS, typename TO, int BITS>
__global__ void dequantize_kernel(const uint32_t* __restrict__ wq, const TS* __restrict__ scales,
                                  const TS* __restrict__ biases, TO* __restrict__ out,
                                  int64_t n_words, int group_size) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_words) return;
  constexpr int PER = 32 / BITS;
  int64_t k0 = i * PER;
  int64_t g = k0 / group_size;
  float s = to_f32<TS>(scales[g]);
  float b = to_f32<TS>(biases[g]);
  uint32_t word = wq[i];
#pragma unroll
  for (int j = 0; j < PER; j++) {
    float q = (float)((word >> (BITS * j)) & ((1u << BITS) - 1u));
    // affine_dequantize (quantized.h:2498-2560) computes `scale * d + bias` in the scales'
    // type T: for T = float that is an unfused fp32 multiply and add; for T = bfloat each
    // operation rounds to bf16 (round to nearest even), so a bf16 result from bf16
    // scales rounds the product before the add.  A float result keeps the exact value.
    float prod = __fmul_rn(s, q);
    if constexpr (sizeof(TS) == 2 && sizeof(TO) == 2) prod = __bfloat162float(__float2bfloat16_rn(prod));
    out[k0 + j] = from_f32<TO>(__fadd_rn(prod, b));
  }
}

static int check_qargs(int64_t rows, int64_t cols, int group_size, int bits, const char* mode) {
  if (!mode_is_affine(mode)) return set_error(VMLX_E_UNSUPPORTED, "mode '%s' not supported", mode);
  if (bits != 2 && bits != 4 && bits != 8)
    return set_error(VMLX_E_UNSUPPORTED, "bits=%d not supported (2, 4, 8)", bits);
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return set_error(VMLX_E_UNSUPPORTED, "group_size=%d not supported (32, 64, 128)", group_size);
  if (rows < 0 || cols <= 0 || cols % group_size)
    return set_error(VMLX_E_INVALID, "cols=%lld must be a positive multiple of group_size=%d",
                     (long long)cols, group_size);
  return VMLX_OK;
}

template <typename T, int GS>
static void launch_quantize_bits(int bits, const T* w, uint32_t* wq, T* s, T* b, int64_t ng,
                                 cudaStream_t st) {
  int threads = 128;
  int64_t blocks = (ng + threads - 1) / threads;
  if (bits == 2) quantize_kernel<T, GS, 2><<<(unsigned)blocks, threads, 0, st>>>(w, wq, s, b, ng);
  if (bits == 4) quantize_kernel<T, GS, 4><<<(unsigned)blocks, threads, 0, st>>>(w, wq, s, b, ng);
  if (bits == 8) quantize_kernel<T, GS, 8><<<(unsigned)blocks, threads, 0, st>>>(w, wq, s, b, ng);
}

template <typename T>
static void launch_quantize(int gs, int bits, const void* w, uint32_t* wq, void* s, void* b,
                            int64_t ng, cudaStream_t st) {
  const T* wt = (const T*)w;
  T* sc = (T*)s;
  T* bi = (T*)b;
  if (gs == 32) launch_quantize_bits<T, 32>(bits, wt, wq, sc, bi, ng, st);
  if (gs == 64) launch_quantize_bits<T, 64>(bits, wt, wq, sc, bi, ng, st);
  if (gs == 128) launch_quantize_bits<T, 128>(bits, wt, wq, sc, bi, ng, st);
}

template <typename TS, typename TO>
static void launch_dequantize(int bits, const uint32_t* wq, const void* s, const void* b, void* out,
                              int64_t n_words, int gs, cudaStream_t st) {
  int threads = 256;
  unsigned blocks = (unsigned)((n_words + threads - 1) / threads);
  const TS* sc = (const TS*)s;
  const TS* bi = (const TS*)b;
  TO* o = (TO*)out;
  if (bits == 2) dequantize_kernel<TS, TO, 2><<<blocks, threads, 0, st>>>(wq, sc, bi, o, n_words, gs);
  if (bits == 4) dequantize_kernel<TS, TO, 4><<<blocks, threads, 0, st>>>(wq, sc, bi, o, n_words, gs);
  if (bits == 8) dequantize_kernel<TS, TO, 8><<<blocks, threads, 0, st>>>(wq, sc, bi, o, n_words, gs);
}

}  // namespace vmlx

using namespace vmlx;

extern "C" int vmlx_cuda_quantize(void* wq, void* scales, void* biases, const void* w, int w_dtype,
                                  int64_t rows, int64_t cols, int group_size, int bits,
                                  const char* mode, void* stream) {
  int rc = check_qargs(rows, cols, group_size, bits, mode);
  if (rc) return rc;
  if (!wq || !scales || !biases || !w) return set_error(VMLX_E_INVALID, "null pointer");
  if (w_dtype != VMLX_BF16 && w_dtype != VMLX_F32)
    return set_error(VMLX_E_UNSUPPORTED, "w_dtype=%d not supported", w_dtype);
  int64_t ng = rows * (cols / group_size);
  if (ng == 0) return VMLX_OK;
  if (w_dtype == VMLX_BF16)
    launch_quantize<bf16>(group_size, bits, w, (uint32_t*)wq, scales, biases, ng, as_stream(stream));
  else
    launch_quantize<float>(group_size, bits, w, (uint32_t*)wq, scales, biases, ng, as_stream(stream));
  return check_launch("vmlx_cuda_quantize");
}

extern "C" int vmlx_cuda_dequantize(void* out, int out_dtype, const uint32_t* wq, const void* scales,
                                    const void* biases, int scales_dtype, int64_t rows, int64_t cols,
                                    int group_size, int bits, const char* mode, void* stream) {
  int rc = check_qargs(rows, cols, group_size, bits, mode);
  if (rc) return rc;
  if (!wq || !scales || !biases || !out) return set_error(VMLX_E_INVALID, "null pointer");
  if ((out_dtype != VMLX_BF16 && out_dtype != VMLX_F32) ||
      (scales_dtype != VMLX_BF16 && scales_dtype != VMLX_F32))
    return set_error(VMLX_E_UNSUPPORTED, "dtype not supported");
  int64_t n_words = rows * cols * bits / 32;
  if (n_words == 0) return VMLX_OK;
  cudaStream_t st = as_stream(stream);
  if (scales_dtype == VMLX_BF16 && out_dtype == VMLX_BF16)
    launch_dequantize<bf16, bf16>(bits, wq, scales, biases, out, n_words, group_size, st);
  else if (scales_dtype == VMLX_BF16 && out_dtype == VMLX_F32)
    launch_dequantize<bf16, float>(bits, wq, scales, biases, out, n_words, group_size, st);
  else if (scales_dtype == VMLX_F32 && out_dtype == VMLX_BF16)
    launch_dequantize<float, bf16>(bits, wq, scales, biases, out, n_words, group_size, st);
  else
    launch_dequantize<float, float>(bits, wq, scales, biases, out, n_words, group_size, st);
  return check_launch("vmlx_cuda_dequantize");
}
