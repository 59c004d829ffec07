// kernels.cuh -- launchers shared between the C-ABI translation units.
#pragma once
#include "common.cuh"

namespace vmlx {

// Token addressing modes of the decode GEMV kernel.
enum QmvMode : int {
  QMV_DENSE = 0,   // x [M, K] -> y [M, N]
  QMV_GATHER = 1,  // blockIdx.y = batch element b: x[lhs[b]] (M rows), expert rhs[b]
  QMV_SORTED = 2,  // blockIdx.y = expert e: every (b, m) row with rhs[b] == e
};

struct QmvArgs {
  const bf16* x;
  const uint32_t* w;
  const bf16* scales;
  const bf16* biases;
  bf16* y;
  const uint32_t* lhs;  // may be null
  const uint32_t* rhs;  // gather modes
  int64_t M, N, K;
  int64_t batch;      // gather: number of batch elements
  int64_t x_batches;  // gather: number of x matrices
  int64_t n_experts;
  int* status;  // optional device word set to VMLX_E_STATE if a bounded wait ran out
  // optional fusions (decoder block): RMSNorm of x on load, residual add on store
  const bf16* norm_w;   // x <- norm_w * bf16(x * rsqrt(mean(x^2) + eps)) over the full row
  float eps;
  const bf16* residual;  // y <- bf16(residual + bf16(x @ W^T)), residual laid out like y (may alias y)
};

int launch_qmv(const QmvArgs& a, int mode, int bits, int gs, int64_t zcount, int toka, cudaStream_t st);

// tcgen05 GEMM for M > 32; sets *handled = false when the shape is not covered.
int launch_qmm_tc(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases, bf16* y,
                  int64_t M, int64_t N, int64_t K, int bits, int gs, cudaStream_t st, bool* handled);

}  // namespace vmlx
