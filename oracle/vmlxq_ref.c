/*
 * vmlxq_ref.c -- CPU oracle for the affine-quantized linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA product
 * path is compared against, and the timed CPU baseline of bench.py.  Nothing in
 * the product library links it or calls it.
 *
 * It restates, in plain C, the arithmetic of MLX's affine quantization as the
 * reference ships it in Metal source form:
 *   Source/Cmlx/mlx-generated/metal/quantized.h
 *     :17-26     pack factor / bytes per pack
 *     :2393-2496 affine_quantize   (edge-exact scale/bias rule, LSB-first pack)
 *     :2498-2558 affine_dequantize (w = scale*q + bias)
 *     :28-114, :209-316, :799-864  qmv_fast_impl accumulation
 *                                  (scale*sum(x*q) + bias*sum(x) per group)
 *     :1438-1491 adjust_matrix_offsets (gather lhs/rhs index semantics)
 * Parity status: quantize and dequantize are bit-exact against the reference's own
 * affine_quantize / affine_dequantize, and the fp64 qmv agrees with its qmv_fast_impl
 * within 1e-2, both compiled for the CPU from quantized.h (make -C oracle ref ->
 * oracle/_ref; tests/test_oracle_ref.py, golden outputs in tests/golden/ref_kernels.npz),
 * and the known-answer fixture of Tests/MLXTests/QuantizationTests.swift:65-111 holds.
 *
 * Conventions
 *   - bf16 values travel as uint16_t bit patterns; bf16 <- f32 is round to
 *     nearest even (the rounding of a Metal/CUDA float->bfloat conversion).
 *   - Packed weights: uint32 words, row-major [rows, cols*bits/32]; element k of
 *     a row lives in word k/(32/bits) at bit offset bits*(k%(32/bits)).
 *   - scales/biases: [rows, cols/group_size], dtype T (f32 or bf16).
 *   - Supported bits: 2, 4, 8 (power-of-two packs into uint32).
 *   - Build WITHOUT fast-math: the quantize rule depends on IEEE division and
 *     on round-half-away-from-zero (C roundf == Metal round).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

uint16_t vq_f32_to_bf16(float f) { return f32_to_bf16(f); }
float vq_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }

static int valid_bits(int bits) { return bits == 2 || bits == 4 || bits == 8; }

/*
 * Quantize one group of `gs` float values (quantized.h:2416-2496).
 * Writes codes[gs] (0..2^bits-1) and the unrounded fp32 scale/bias.
 * Note w_max starts at 0 (quantized.h:2424) while w_min starts at the type's
 * max, so an all-positive group keeps its true minimum but an all-negative
 * group has w_max == 0.
 */
static void quantize_group(const float* v, int gs, int bits, float t_max,
                           uint8_t* codes, float* scale_out, float* bias_out) {
  const float eps = 1e-7f;
  const float n_bins = (float)((1 << bits) - 1);
  float w_min = t_max, w_max = 0.0f;
  for (int i = 0; i < gs; i++) {
    w_min = fminf(w_min, v[i]);
    w_max = fmaxf(w_max, v[i]);
  }
  float scale = fmaxf((w_max - w_min) / n_bins, eps);
  int side = fabsf(w_min) > fabsf(w_max);
  scale = side ? scale : -scale;
  float edge = side ? w_min : w_max;
  float q0 = roundf(edge / scale);
  int at_zero = (q0 == 0.0f);
  scale = at_zero ? scale : edge / q0;
  float bias = at_zero ? 0.0f : edge;
  for (int i = 0; i < gs; i++) {
    float q = fminf(roundf((v[i] - bias) / scale), n_bins);
    /* float -> uint8 conversion: saturate (negative / NaN -> 0). */
    codes[i] = (q > 0.0f) ? (uint8_t)q : 0;
  }
  *scale_out = scale;
  *bias_out = bias;
}

static void pack_row(const uint8_t* codes, int64_t cols, int bits, uint32_t* out) {
  int per = 32 / bits;
  int64_t words = cols / per;
  for (int64_t w = 0; w < words; w++) {
    uint32_t acc = 0;
    for (int j = 0; j < per; j++) acc |= ((uint32_t)codes[w * per + j]) << (bits * j);
    out[w] = acc;
  }
}

/* Quantize with T = float32 (scales/biases stored as f32). Returns 0 / -1. */
int vq_quantize_f32(const float* w, int64_t rows, int64_t cols, int gs, int bits,
                    uint32_t* wq, float* scales, float* biases) {
  if (!valid_bits(bits) || gs <= 0 || cols % gs || (cols * bits) % 32) return -1;
  int64_t ng = cols / gs, wpr = cols * bits / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    uint8_t* codes = (uint8_t*)malloc((size_t)cols);
    for (int64_t g = 0; g < ng; g++) {
      float s, b;
      quantize_group(w + r * cols + g * gs, gs, bits, FLT_MAX, codes + g * gs, &s, &b);
      scales[r * ng + g] = s;
      biases[r * ng + g] = b;
    }
    pack_row(codes, cols, bits, wq + r * wpr);
    free(codes);
  }
  return 0;
}

/* Quantize with T = bfloat16: inputs are bf16 bit patterns; the fp32 math is
 * identical, the stored scale/bias are bf16(scale)/bf16(bias), while the codes
 * use the unrounded fp32 scale (quantized.h:2446-2460). */
int vq_quantize_bf16(const uint16_t* w, int64_t rows, int64_t cols, int gs, int bits,
                     uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  if (!valid_bits(bits) || gs <= 0 || cols % gs || (cols * bits) % 32) return -1;
  int64_t ng = cols / gs, wpr = cols * bits / 32;
  const float bf16_max = bf16_to_f32(0x7f7f);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    uint8_t* codes = (uint8_t*)malloc((size_t)cols);
    float* v = (float*)malloc((size_t)gs * sizeof(float));
    for (int64_t g = 0; g < ng; g++) {
      for (int i = 0; i < gs; i++) v[i] = bf16_to_f32(w[r * cols + g * gs + i]);
      float s, b;
      quantize_group(v, gs, bits, bf16_max, codes + g * gs, &s, &b);
      scales[r * ng + g] = f32_to_bf16(s);
      biases[r * ng + g] = f32_to_bf16(b);
    }
    pack_row(codes, cols, bits, wq + r * wpr);
    free(codes);
    free(v);
  }
  return 0;
}

static inline uint32_t code_at(const uint32_t* row, int64_t k, int bits) {
  int per = 32 / bits;
  return (row[k / per] >> (bits * (k % per))) & ((1u << bits) - 1u);
}

/* Dequantize (quantized.h:2498-2558): out = float(scale)*q + float(bias),
 * computed in fp32 as an unfused multiply then add (built with
 * -ffp-contract=off); for bf16 scales the product is exact, so this also equals
 * the fused form.
 * scales_bf16 != 0 means scales/biases are bf16 bit patterns, else f32. */
int vq_dequantize(const uint32_t* wq, const void* scales, const void* biases, int scales_bf16,
                  int64_t rows, int64_t cols, int gs, int bits, float* out) {
  if (!valid_bits(bits) || cols % gs || (cols * bits) % 32) return -1;
  int64_t ng = cols / gs, wpr = cols * bits / 32;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    for (int64_t k = 0; k < cols; k++) {
      int64_t gi = r * ng + k / gs;
      float s = scales_bf16 ? bf16_to_f32(((const uint16_t*)scales)[gi]) : ((const float*)scales)[gi];
      float b = scales_bf16 ? bf16_to_f32(((const uint16_t*)biases)[gi]) : ((const float*)biases)[gi];
      out[r * cols + k] = s * (float)code_at(wq + r * wpr, k, bits) + b;
    }
  }
  return 0;
}

/*
 * Tolerance reference for quantized_matmul with transpose=true:
 *   y[m, n] = sum_k x[m, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g])
 * accumulated in fp64 over the exact fp32 dequantized weights.  x, scales and
 * biases are bf16.  y is returned in f64 so tests can measure error honestly.
 */
int vq_qmm_f64(const uint16_t* x, int64_t M, int64_t K, const uint32_t* wq,
               const uint16_t* scales, const uint16_t* biases, int64_t N, int gs, int bits,
               double* y) {
  if (!valid_bits(bits) || K % gs || (K * bits) % 32) return -1;
  int64_t ng = K / gs, wpr = K * bits / 32;
  double* xf = (double*)malloc((size_t)(M * K) * sizeof(double));
  for (int64_t i = 0; i < M * K; i++) xf[i] = bf16_to_f32(x[i]);
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; n++) {
    double* wrow = (double*)malloc((size_t)K * sizeof(double));
    for (int64_t k = 0; k < K; k++) {
      float s = bf16_to_f32(scales[n * ng + k / gs]);
      float b = bf16_to_f32(biases[n * ng + k / gs]);
      wrow[k] = (double)(s * (float)code_at(wq + n * wpr, k, bits) + b);
    }
    for (int64_t m = 0; m < M; m++) {
      double acc = 0.0;
      const double* xr = xf + m * K;
      for (int64_t k = 0; k < K; k++) acc += xr[k] * wrow[k];
      y[m * N + n] = acc;
    }
    free(wrow);
  }
  free(xf);
  return 0;
}

/*
 * The reference's factorisation of the decode GEMV, restated on the CPU
 * (qmv_fast_impl, quantized.h:799-864 with qdot :209-316): per group an fp32
 * accumulation of x*q (exact products), then scale*accum + bias*sum(x), summed
 * over groups in fp32; result rounded to bf16.  The summation order across
 * SIMD lanes differs from the Metal kernel (fp32-level differences only).
 * This is the timed CPU baseline (OpenMP over output rows) and a second
 * opinion on the bf16 outputs.
 */
int vq_qmm_fp32(const uint16_t* x, int64_t M, int64_t K, const uint32_t* wq,
                const uint16_t* scales, const uint16_t* biases, int64_t N, int gs, int bits,
                uint16_t* y) {
  if (!valid_bits(bits) || K % gs || (K * bits) % 32) return -1;
  int64_t ng = K / gs, wpr = K * bits / 32;
  int per = 32 / bits;
  uint32_t mask = (1u << bits) - 1u;
  float* xf = (float*)malloc((size_t)(M * K) * sizeof(float));
  float* xs = (float*)malloc((size_t)(M * ng) * sizeof(float));
  for (int64_t i = 0; i < M * K; i++) xf[i] = bf16_to_f32(x[i]);
  for (int64_t m = 0; m < M; m++)
    for (int64_t g = 0; g < ng; g++) {
      float s = 0.f;
      for (int i = 0; i < gs; i++) s += xf[m * K + g * gs + i];
      xs[m * ng + g] = s;
    }
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; n++) {
    const uint32_t* wr = wq + n * wpr;
    for (int64_t m = 0; m < M; m++) {
      const float* xr = xf + m * K;
      float result = 0.f;
      for (int64_t g = 0; g < ng; g++) {
        float accum = 0.f;
        const uint32_t* wg = wr + g * gs / per;
        const float* xg = xr + g * gs;
        for (int w = 0; w < gs / per; w++) {
          uint32_t word = wg[w];
          for (int j = 0; j < per; j++) accum += xg[w * per + j] * (float)((word >> (bits * j)) & mask);
        }
        float s = bf16_to_f32(scales[n * ng + g]);
        float b = bf16_to_f32(biases[n * ng + g]);
        result += s * accum + xs[m * ng + g] * b;
      }
      y[m * N + n] = f32_to_bf16(result);
    }
  }
  free(xf);
  free(xs);
  return 0;
}

/*
 * gather_qmm tolerance reference (quantized.h:1438-1491 + GatherQMM):
 * for each batch element z in [0, nb):
 *   y[z] (M x N) = x[lhs[z]] (M x K) @ deq(W[rhs[z]])^T
 * x: [n_x, M, K] bf16; W: [E, N, K*bits/32]; scales/biases [E, N, K/g];
 * lhs == NULL means x batch z is used directly (x has nb batches).
 */
int vq_gather_qmm_f64(const uint16_t* x, int64_t M, int64_t K, const uint32_t* wq,
                      const uint16_t* scales, const uint16_t* biases, int64_t N, int64_t E,
                      const uint32_t* lhs, const uint32_t* rhs, int64_t nb, int gs, int bits,
                      double* y) {
  if (!valid_bits(bits) || K % gs || (K * bits) % 32) return -1;
  int64_t wstride = N * (K * bits / 32), sstride = N * (K / gs);
  for (int64_t z = 0; z < nb; z++) {
    int64_t xi = lhs ? (int64_t)lhs[z] : z;
    int64_t e = (int64_t)rhs[z];
    if (e < 0 || e >= E) return -2;
    int rc = vq_qmm_f64(x + xi * M * K, M, K, wq + e * wstride, scales + e * sstride,
                        biases + e * sstride, N, gs, bits, y + z * M * N);
    if (rc) return rc;
  }
  return 0;
}

int vq_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
