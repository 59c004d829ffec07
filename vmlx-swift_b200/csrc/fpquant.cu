// fpquant.cu -- the MXFP4 block-scaled format (MLX mode "mxfp4"): quantize, dequantize and a
// decode GEMV.  Replaces fp_quantize / fp_dequantize / the fp qmv kernels of MLX
// (Source/Cmlx/mlx-generated/metal/fp_quantized.h:20-140, 1749-1820; fp4.h; fp8.h:51-80).
//
// Format: groups of 32 values along K; each value a 4-bit e2m1 code (sign, 2 exponent bits, 1
// mantissa bit: magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6), two codes per byte, low nibble first (so
// eight per little-endian u32 word, as the affine layout); one e8m0 scale byte per group
// (2^(s - 127); s = 0 encodes 2^-127).  No biases.
//   quantize: scale = e8m0(max|w| / 6) (log2 rounded to nearest, clamped to [-127, 127]);
//             code = e2m1(w / scale) with the reference's thresholds (ties to the even mantissa).
//   dequantize: scale * e2m1 value, rounded once to the output type.
//   matmul: per group scale * sum(x * value) in fp32 (MLX's fp qdot).
// Load-time and decode-rate kernels on CUDA cores; not tuned to the HBM roofline.
#include <string>

#include "kernels.cuh"

namespace vmlx {

__device__ __forceinline__ float fq_ld(float v) { return v; }
__device__ __forceinline__ float fq_ld(bf16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T fq_st(float v);
template <> __device__ __forceinline__ float fq_st<float>(float v) { return v; }
template <> __device__ __forceinline__ bf16 fq_st<bf16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ uint32_t e2m1_code(float x) {
  if (isnan(x)) return 0x7;
  const uint32_t sign = signbit(x) ? 0x8u : 0x0u;
  x = fabsf(x);
  uint32_t b;
  if (x > 5.0f) b = 7;
  else if (x >= 3.5f) b = 6;
  else if (x > 2.5f) b = 5;
  else if (x >= 1.75f) b = 4;
  else if (x > 1.25f) b = 3;
  else if (x >= 0.75f) b = 2;
  else if (x > 0.25f) b = 1;
  else b = 0;
  return b | sign;
}

// e2m1 code -> float (exact): 0, 0.5 for codes 0, 1; 2^(e-1) * (1 + m/2) above.
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t v = c & 7u;
  const float mag = v >= 2u ? __uint_as_float((v + 252u) << 22) : 0.5f * (float)v;
  return (c & 8u) ? -mag : mag;
}

__device__ __forceinline__ float e8m0_value(uint32_t s) {
  return __uint_as_float(s == 0 ? 0x400000u : (s << 23));
}

__device__ __forceinline__ uint32_t e8m0_code(float x) {
  if (!isfinite(x)) return 0xFFu;
  if (x < 0.0f) return 0x00u;
  int n;
  if (x == 0.0f) {
    n = -127;
  } else {
    n = (int)roundf(log2f(x));
    n = n < -127 ? -127 : (n > 127 ? 127 : n);
  }
  return (uint32_t)(n + 127);
}

// One thread per group of 32 values: scale byte + 4 packed words.
template <typename T>
__global__ void mxfp4_quantize_kernel(const T* __restrict__ w, uint32_t* __restrict__ wq, uint8_t* __restrict__ sc,
                                      int64_t n_groups) {
  const int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gi >= n_groups) return;
  const T* wg = w + gi * 32;
  float amax = 0.f;
  for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(fq_ld(wg[i])));
  const uint32_t s = e8m0_code(amax / 6.0f);
  const float scale = e8m0_value(s);
  sc[gi] = (uint8_t)s;
  for (int j = 0; j < 4; j++) {
    uint32_t word = 0;
    for (int i = 0; i < 8; i++) {
      const float x = fq_ld(wg[8 * j + i]);
      word |= e2m1_code(scale == 0.f ? 0.f : x / scale) << (4 * i);
    }
    wq[gi * 4 + j] = word;
  }
}

template <typename TO>
__global__ void mxfp4_dequantize_kernel(const uint32_t* __restrict__ wq, const uint8_t* __restrict__ sc,
                                        TO* __restrict__ out, int64_t n_words) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_words) return;
  const float scale = e8m0_value(sc[i / 4]);
  const uint32_t word = wq[i];
#pragma unroll
  for (int j = 0; j < 8; j++) out[i * 8 + j] = fq_st<TO>(scale * e2m1_value((word >> (4 * j)) & 0xFu));
}

// GEMV / skinny GEMM: y[m, n] = sum_g scale[n, g] * sum_{k in g} x[m, k] * v[n, k].  One warp per
// output row n and token set; lane l takes groups l, l + 32, ... (16 bytes of codes + 1 scale each).
constexpr int FQ_ROWS = 8;  // warps (rows) per CTA
template <int MT>
__global__ void __launch_bounds__(32 * FQ_ROWS)
mxfp4_gemv_kernel(const bf16* __restrict__ x, const uint32_t* __restrict__ wq, const uint8_t* __restrict__ sc,
                  bf16* __restrict__ y, int64_t M, int64_t N, int64_t K) {
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)blockIdx.x * FQ_ROWS + (threadIdx.x >> 5);
  const int64_t m0 = (int64_t)blockIdx.y * MT;
  if (n >= N) return;
  const int64_t G = K / 32;
  float acc[MT];
#pragma unroll
  for (int t = 0; t < MT; t++) acc[t] = 0.f;
  const uint4* wr = reinterpret_cast<const uint4*>(wq + n * (K / 8));
  for (int64_t g = lane; g < G; g += 32) {
    const uint4 c = wr[g];
    const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
    const float scale = e8m0_value(sc[n * G + g]);
    float v[32];
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int i = 0; i < 8; i++) v[8 * j + i] = e2m1_value((cw[j] >> (4 * i)) & 0xFu);
#pragma unroll
    for (int t = 0; t < MT; t++) {
      if (m0 + t >= M) break;
      const bf16* xr = x + (m0 + t) * K + g * 32;
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xr + 8 * q);
        const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int h = 0; h < 4; h++) {
          const float2 f = __bfloat1622float2(u32_as_bf162(xu[h]));
          s = fmaf(f.x, v[8 * q + 2 * h], s);
          s = fmaf(f.y, v[8 * q + 2 * h + 1], s);
        }
      }
      acc[t] = fmaf(scale, s, acc[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < MT; t++) {
    float a = acc[t];
    for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0 && m0 + t < M) y[(m0 + t) * N + n] = __float2bfloat16_rn(a);
  }
}

static int fq_check_mode(const char* mode, int group_size, int bits) {
  if (!mode || std::string(mode) != "mxfp4")
    return set_error(VMLX_E_UNSUPPORTED, "fp quantization mode '%s' not supported (mxfp4)", mode ? mode : "(null)");
  if (group_size != 32 || bits != 4)
    return set_error(VMLX_E_UNSUPPORTED, "mxfp4 needs group_size 32 and bits 4 (got %d, %d)", group_size, bits);
  return VMLX_OK;
}

}  // namespace vmlx

using namespace vmlx;

extern "C" int vmlx_cuda_fp_quantize(void* wq, void* scales, const void* w, int w_dtype, int64_t rows, int64_t cols,
                                     int group_size, int bits, const char* mode, void* stream) {
  int rc = fq_check_mode(mode, group_size, bits);
  if (rc) return rc;
  if (rows < 0 || cols <= 0 || cols % 32) return set_error(VMLX_E_INVALID, "fp_quantize: cols must be a multiple of 32");
  if (rows == 0) return VMLX_OK;
  if (!wq || !scales || !w) return set_error(VMLX_E_INVALID, "fp_quantize: null pointer");
  const int64_t ng = rows * cols / 32;
  const unsigned blocks = (unsigned)((ng + 127) / 128);
  if (w_dtype == VMLX_BF16)
    mxfp4_quantize_kernel<bf16><<<blocks, 128, 0, as_stream(stream)>>>((const bf16*)w, (uint32_t*)wq,
                                                                       (uint8_t*)scales, ng);
  else if (w_dtype == VMLX_F32)
    mxfp4_quantize_kernel<float><<<blocks, 128, 0, as_stream(stream)>>>((const float*)w, (uint32_t*)wq,
                                                                        (uint8_t*)scales, ng);
  else
    return set_error(VMLX_E_UNSUPPORTED, "fp_quantize: dtype %d", w_dtype);
  return check_launch("mxfp4_quantize_kernel");
}

extern "C" int vmlx_cuda_fp_dequantize(void* out, int out_dtype, const void* wq, const void* scales, int64_t rows,
                                       int64_t cols, int group_size, int bits, const char* mode, void* stream) {
  int rc = fq_check_mode(mode, group_size, bits);
  if (rc) return rc;
  if (rows < 0 || cols <= 0 || cols % 32) return set_error(VMLX_E_INVALID, "fp_dequantize: cols must be a multiple of 32");
  if (rows == 0) return VMLX_OK;
  if (!out || !wq || !scales) return set_error(VMLX_E_INVALID, "fp_dequantize: null pointer");
  const int64_t nw = rows * cols / 8;
  const unsigned blocks = (unsigned)((nw + 255) / 256);
  if (out_dtype == VMLX_BF16)
    mxfp4_dequantize_kernel<bf16><<<blocks, 256, 0, as_stream(stream)>>>((const uint32_t*)wq, (const uint8_t*)scales,
                                                                         (bf16*)out, nw);
  else if (out_dtype == VMLX_F32)
    mxfp4_dequantize_kernel<float><<<blocks, 256, 0, as_stream(stream)>>>((const uint32_t*)wq, (const uint8_t*)scales,
                                                                          (float*)out, nw);
  else
    return set_error(VMLX_E_UNSUPPORTED, "fp_dequantize: dtype %d", out_dtype);
  return check_launch("mxfp4_dequantize_kernel");
}

extern "C" int vmlx_cuda_fp_quantized_matmul(void* y, const void* x, const void* wq, const void* scales,
                                             int group_size, int bits, const char* mode, int64_t M, int64_t N,
                                             int64_t K, void* stream) {
  int rc = fq_check_mode(mode, group_size, bits);
  if (rc) return rc;
  if (M < 0 || N <= 0 || K <= 0 || K % 32) return set_error(VMLX_E_INVALID, "fp_quantized_matmul: bad shape");
  if (M == 0) return VMLX_OK;
  if (!y || !x || !wq || !scales) return set_error(VMLX_E_INVALID, "fp_quantized_matmul: null pointer");
  if (!aligned(x, 16) || !aligned(wq, 16)) return set_error(VMLX_E_INVALID, "fp_quantized_matmul: 16-byte alignment");
  constexpr int MT = 4;
  if ((M + MT - 1) / MT > 65535) return set_error(VMLX_E_UNSUPPORTED, "fp_quantized_matmul: M=%lld", (long long)M);
  dim3 grid((unsigned)((N + FQ_ROWS - 1) / FQ_ROWS), (unsigned)((M + MT - 1) / MT));
  mxfp4_gemv_kernel<MT><<<grid, 32 * FQ_ROWS, 0, as_stream(stream)>>>((const bf16*)x, (const uint32_t*)wq,
                                                                        (const uint8_t*)scales, (bf16*)y, M, N, K);
  return check_launch("mxfp4_gemv_kernel");
}
