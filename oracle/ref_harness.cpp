// ref_harness.cpp -- drives the reference's own affine_quantize, affine_dequantize and
// qmv_fast_impl (Metal source text of Source/Cmlx/mlx-generated/metal/quantized.h,
// lines 12-26, 28-114, 209-316, 798-864 and 2392-2560, cut out unchanged by
// oracle/Makefile into oracle/_ref/quantized_subset.h) on the CPU, through the host
// environment of oracle/ref_shim.h.
//
// TEST INFRASTRUCTURE ONLY: it pins the C restatement (oracle/vmlxq_ref.c) to the
// reference's kernels; the product library never links or calls it.
//
// Dispatch follows MLX's host code for these kernels: one thread per
// group_size/32 values for quantize (a SIMD group = one group), one thread per pack
// for dequantize, and for qmv_fast threadgroups of 2 SIMD groups x 4 output rows.
#include "ref_shim.h"
#include "quantized_subset.h"

#include <cstdlib>

namespace {

template <typename T, int GS, int BITS>
void quantize_t(const T* w, int64_t rows, int64_t cols, uint8_t* out, T* scales, T* biases) {
  constexpr int vpr = GS / 32;  // values per thread
  const int64_t threads = rows * cols / vpr;
  const int64_t groups = threads / 32;
#pragma omp parallel for schedule(static)
  for (int64_t sg = 0; sg < groups; sg++) {
    simdemu::run([&](int lane) {
      uint2 index{(uint32_t)(sg * 32 + lane), 0};
      uint2 grid{(uint32_t)threads, 1};
      affine_quantize<T, GS, BITS>(w, out, scales, biases, index, grid);
    });
  }
}

template <typename T, int GS, int BITS>
void dequantize_t(const uint8_t* wq, const T* scales, const T* biases, int64_t rows, int64_t cols, T* out) {
  constexpr int pf = 8 / BITS;  // get_pack_factor<bits, 8>: values per byte
  const int64_t threads = rows * cols / pf;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < threads; i++) {
    uint2 index{(uint32_t)i, 0};
    uint2 grid{(uint32_t)threads, 1};
    affine_dequantize<T, GS, BITS>(wq, scales, biases, out, index, grid);
  }
}

template <int GS, int BITS>
void qmv_t(const bfloat16_t* x, int64_t M, int64_t K, const uint32_t* w, const bfloat16_t* scales,
           const bfloat16_t* biases, int64_t N, bfloat16_t* y) {
  const int in_vec = (int)K, out_vec = (int)N;
  const int64_t tgy = N / 8;  // 2 SIMD groups x 4 rows
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t m = 0; m < M; m++)
    for (int64_t ty = 0; ty < tgy; ty++)
      for (uint32_t sgid = 0; sgid < 2; sgid++) {
        simdemu::run([&](int lane) {
          uint3 tid{(uint32_t)m, (uint32_t)ty, 0};
          qmv_fast_impl<bfloat16_t, GS, BITS>(w, scales, biases, x, y, in_vec, out_vec, tid, sgid, (uint32_t)lane);
        });
      }
}

#define VMLX_DISPATCH_GB(F, ...)                             \
  switch (gs * 100 + bits) {                                 \
    case 3202: F<32, 2>(__VA_ARGS__); return 0;              \
    case 3204: F<32, 4>(__VA_ARGS__); return 0;              \
    case 3208: F<32, 8>(__VA_ARGS__); return 0;              \
    case 6402: F<64, 2>(__VA_ARGS__); return 0;              \
    case 6404: F<64, 4>(__VA_ARGS__); return 0;              \
    case 6408: F<64, 8>(__VA_ARGS__); return 0;              \
    case 12802: F<128, 2>(__VA_ARGS__); return 0;            \
    case 12804: F<128, 4>(__VA_ARGS__); return 0;            \
    case 12808: F<128, 8>(__VA_ARGS__); return 0;            \
    default: return -1;                                      \
  }

template <int GS, int BITS>
void quantize_bf(const void* w, int64_t r, int64_t c, void* o, void* s, void* b) {
  quantize_t<bfloat16_t, GS, BITS>((const bfloat16_t*)w, r, c, (uint8_t*)o, (bfloat16_t*)s, (bfloat16_t*)b);
}
template <int GS, int BITS>
void quantize_f(const void* w, int64_t r, int64_t c, void* o, void* s, void* b) {
  quantize_t<float, GS, BITS>((const float*)w, r, c, (uint8_t*)o, (float*)s, (float*)b);
}
template <int GS, int BITS>
void dequantize_bf(const void* wq, const void* s, const void* b, int64_t r, int64_t c, void* o) {
  dequantize_t<bfloat16_t, GS, BITS>((const uint8_t*)wq, (const bfloat16_t*)s, (const bfloat16_t*)b, r, c,
                                     (bfloat16_t*)o);
}
template <int GS, int BITS>
void dequantize_f(const void* wq, const void* s, const void* b, int64_t r, int64_t c, void* o) {
  dequantize_t<float, GS, BITS>((const uint8_t*)wq, (const float*)s, (const float*)b, r, c, (float*)o);
}
template <int GS, int BITS>
void qmv_bf(const void* x, int64_t M, int64_t K, const uint32_t* w, const void* s, const void* b, int64_t N,
            void* y) {
  qmv_t<GS, BITS>((const bfloat16_t*)x, M, K, w, (const bfloat16_t*)s, (const bfloat16_t*)b, N, (bfloat16_t*)y);
}

}  // namespace

extern "C" {

// w [rows, cols] (bf16 if is_bf16 else f32) -> packed bytes, scales, biases (same dtype as w)
int ref_quantize(const void* w, int is_bf16, int64_t rows, int64_t cols, int gs, int bits, void* wq,
                 void* scales, void* biases) {
  if (cols % gs) return -1;
  if (is_bf16) {
    VMLX_DISPATCH_GB(quantize_bf, w, rows, cols, wq, scales, biases)
  }
  VMLX_DISPATCH_GB(quantize_f, w, rows, cols, wq, scales, biases)
}

int ref_dequantize(const void* wq, const void* scales, const void* biases, int is_bf16, int64_t rows,
                   int64_t cols, int gs, int bits, void* out) {
  if (cols % gs) return -1;
  if (is_bf16) {
    VMLX_DISPATCH_GB(dequantize_bf, wq, scales, biases, rows, cols, out)
  }
  VMLX_DISPATCH_GB(dequantize_f, wq, scales, biases, rows, cols, out)
}

// y [M, N] bf16 = x [M, K] bf16 @ dequantize(w)^T through qmv_fast_impl; needs K % 512 == 0
// (4-bit; 256 for 8-bit) and N % 8 == 0, the shapes MLX routes to the fast kernel.
int ref_qmv_fast(const void* x, int64_t M, int64_t K, const uint32_t* w, const void* scales, const void* biases,
                 int64_t N, int gs, int bits, void* y) {
  const int64_t block = bits == 8 ? 256 : 512;
  if (K % block || N % 8 || bits == 2) return -1;
  VMLX_DISPATCH_GB(qmv_bf, x, M, K, w, scales, biases, N, y)
}

}  // extern "C"
