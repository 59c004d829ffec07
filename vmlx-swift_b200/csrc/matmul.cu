// matmul.cu -- C-ABI entry points quantized_matmul / gather_qmm and their dispatch.
#include "kernels.cuh"

namespace vmlx {

static int check_mm_args(const void* y, const void* x, const void* w, const void* s, const void* b,
                         bool transpose, int gs, int bits, const char* mode, int64_t M, int64_t N,
                         int64_t K) {
  if (!mode_is_affine(mode)) return set_error(VMLX_E_UNSUPPORTED, "mode '%s' not supported", mode ? mode : "");
  if (!transpose) return set_error(VMLX_E_UNSUPPORTED, "transpose=false is not supported");
  if (bits != 4 && bits != 8) return set_error(VMLX_E_UNSUPPORTED, "bits=%d not supported for matmul (4, 8)", bits);
  if (gs != 32 && gs != 64 && gs != 128) return set_error(VMLX_E_UNSUPPORTED, "group_size=%d not supported", gs);
  if (!y || !x || !w || !s) return set_error(VMLX_E_INVALID, "null pointer");
  if (!b) return set_error(VMLX_E_INVALID, "affine mode requires biases");
  if (M < 0 || N <= 0 || K <= 0 || K % gs)
    return set_error(VMLX_E_INVALID, "bad shape M=%lld N=%lld K=%lld (K must be a multiple of %d)",
                     (long long)M, (long long)N, (long long)K, gs);
  if (!aligned(x, 16) || !aligned(w, 16))
    return set_error(VMLX_E_INVALID, "x and w must be 16-byte aligned");
  return VMLX_OK;
}

// Smallest M that runs on the tensor-core GEMM (VMLX_TC_MIN_M overrides; read once).
// From 5 rows up the tcgen05 GEMM is the faster kernel on every Llama-shaped matrix but
// the small ones at 8 rows (the warp-level mma.sync of the GEMV kernel runs far below
// HBM speed at 16-32 rows on B200); one kernel for 5..32 rows keeps them batch-invariant.
static int64_t tc_min_m() {
  static const int64_t v = [] {
    const char* e = getenv("VMLX_TC_MIN_M");
    return (int64_t)(e && *e ? atoll(e) : 5);
  }();
  return v;
}

static int toka_for(int64_t m) { return (int)(m < 1 ? 1 : (m > 32 ? 32 : m)); }

}  // namespace vmlx

using namespace vmlx;

extern "C" int vmlx_cuda_quantized_matmul(void* y, const void* x, const uint32_t* w, const void* scales,
                                          const void* biases, bool transpose, int group_size, int bits,
                                          const char* mode, int64_t M, int64_t N, int64_t K,
                                          void* stream) {
  if (M == 0 && N > 0 && K > 0) return VMLX_OK;  // empty input: nothing to read or write
  int rc = check_mm_args(y, x, w, scales, biases, transpose, group_size, bits, mode, M, N, K);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  if (M >= tc_min_m()) {
    bool handled = false;
    rc = launch_qmm_tc((const bf16*)x, w, (const bf16*)scales, (const bf16*)biases, (bf16*)y, M, N, K,
                       bits, group_size, st, &handled);
    if (rc || handled) return rc;
  }
  QmvArgs a{(const bf16*)x, w, (const bf16*)scales, (const bf16*)biases, (bf16*)y, nullptr, nullptr,
            M, N, K, 0, 1, 1};
  return launch_qmv(a, QMV_DENSE, bits, group_size, 1, toka_for(M), st);
}

extern "C" int vmlx_cuda_gather_qmm(void* y, const void* x, const uint32_t* w, const void* scales,
                                    const void* biases, const uint32_t* lhs_indices,
                                    const uint32_t* rhs_indices, bool transpose, int group_size,
                                    int bits, const char* mode, bool sorted_indices, int64_t batch,
                                    int64_t x_batches, int64_t M, int64_t N, int64_t K,
                                    int64_t n_experts, void* stream) {
  int rc = check_mm_args(y, x, w, scales, biases, transpose, group_size, bits, mode, M, N, K);
  if (rc) return rc;
  if (!rhs_indices && batch % n_experts)
    return set_error(VMLX_E_INVALID, "without rhs_indices, batch=%lld must be a multiple of n_experts=%lld",
                     (long long)batch, (long long)n_experts);
  if (batch < 0 || x_batches <= 0 || n_experts <= 0)
    return set_error(VMLX_E_INVALID, "bad batch=%lld x_batches=%lld n_experts=%lld", (long long)batch,
                     (long long)x_batches, (long long)n_experts);
  if (!lhs_indices && batch % x_batches)
    return set_error(VMLX_E_INVALID, "without lhs_indices, batch=%lld must be a multiple of x_batches=%lld",
                     (long long)batch, (long long)x_batches);
  if (batch == 0 || M == 0) return VMLX_OK;
  QmvArgs a{(const bf16*)x, w, (const bf16*)scales, (const bf16*)biases, (bf16*)y, lhs_indices,
            rhs_indices, M, N, K, batch, x_batches, n_experts};
  cudaStream_t st = as_stream(stream);
  if (sorted_indices && rhs_indices) {
    // rows per expert on average, staged in passes of up to 32 rows
    int64_t avg = (batch * M + n_experts - 1) / n_experts;
    int toka = (int)((avg + avg / 2 + 7) / 8 * 8);
    return launch_qmv(a, QMV_SORTED, bits, group_size, n_experts, toka, st);
  }
  return launch_qmv(a, QMV_GATHER, bits, group_size, batch, toka_for(M), st);
}

extern "C" int vmlx_cuda_quantized_matmul_fused(void* y, const void* x, const uint32_t* w, const void* scales,
                                                const void* biases, int group_size, int bits, int64_t M, int64_t N,
                                                int64_t K, const void* norm_weight, float eps, const void* residual,
                                                void* stream) {
  if (M == 0 && N > 0 && K > 0) return VMLX_OK;
  int rc = check_mm_args(y, x, w, scales, biases, true, group_size, bits, "affine", M, N, K);
  if (rc) return rc;
  if (M > 32) return set_error(VMLX_E_UNSUPPORTED, "quantized_matmul_fused: M=%lld > 32", (long long)M);
  if (norm_weight && (!aligned(norm_weight, 16) || K % 8))
    return set_error(VMLX_E_INVALID, "quantized_matmul_fused: norm_weight must be 16-byte aligned, K a multiple of 8");
  QmvArgs a{(const bf16*)x, w, (const bf16*)scales, (const bf16*)biases, (bf16*)y, nullptr, nullptr,
            M, N, K, 0, 1, 1, nullptr, (const bf16*)norm_weight, eps, (const bf16*)residual};
  return launch_qmv(a, QMV_DENSE, bits, group_size, 1, toka_for(M), as_stream(stream));
}

// Down projection with the MLP's SwiGLU fused into the GEMV's x staging (decode, M <= 32):
//   y = [residual +] bf16(SwiGLU(gate_up) @ dequantize(W)^T),  gate_up bf16 [M, 2K] = gate | up
// -- compiledSwiGLU followed by the down QuantizedLinear (Libraries/MLXLMCommon/SwitchLayers.swift:40-50,
// Libraries/MLXLLM/Models/Llama.swift:96-99) in one kernel.
extern "C" int vmlx_cuda_quantized_matmul_swiglu(void* y, const void* gate_up, const uint32_t* w, const void* scales,
                                                 const void* biases, int group_size, int bits, int64_t M, int64_t N,
                                                 int64_t K, const void* residual, void* stream) {
  if (M == 0 && N > 0 && K > 0) return VMLX_OK;
  int rc = check_mm_args(y, gate_up, w, scales, biases, true, group_size, bits, "affine", M, N, K);
  if (rc) return rc;
  if (M > 32) return set_error(VMLX_E_UNSUPPORTED, "quantized_matmul_swiglu: M=%lld > 32", (long long)M);
  if (K % 8) return set_error(VMLX_E_INVALID, "quantized_matmul_swiglu: K must be a multiple of 8");
  QmvArgs a{(const bf16*)gate_up, w, (const bf16*)scales, (const bf16*)biases, (bf16*)y, nullptr, nullptr,
            M, N, K, 0, 1, 1, nullptr, nullptr, 0.f, (const bf16*)residual};
  a.x_swiglu = 1;
  return launch_qmv(a, QMV_DENSE, bits, group_size, 1, toka_for(M), as_stream(stream));
}


extern "C" size_t vmlx_cuda_gather_qmm_workspace_size(int64_t batch, int64_t M, int64_t K, int64_t n_experts) {
  if (batch <= 0 || M <= 0 || K <= 0 || n_experts <= 0) return 0;
  return gather_tc_workspace(batch, M, K, n_experts);
}

// vmlx_cuda_gather_qmm with a caller-owned workspace: sorted gathers with enough rows per
// expert (on average >= 8) run as an expert-segmented tcgen05 GEMM -- one 64-row tile per
// run of equal experts, each expert's weights dequantized once per tile, the reference's
// affine_gather_qmm_rhs (quantized.h:2197-2391) -- instead of the GEMV kernel.
extern "C" int vmlx_cuda_gather_qmm_ws(void* y, const void* x, const uint32_t* w, const void* scales,
                                       const void* biases, const uint32_t* lhs_indices,
                                       const uint32_t* rhs_indices, bool transpose, int group_size, int bits,
                                       const char* mode, bool sorted_indices, int64_t batch, int64_t x_batches,
                                       int64_t M, int64_t N, int64_t K, int64_t n_experts, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  const bool tc = sorted_indices && rhs_indices && workspace && batch > 0 && M > 0 && n_experts <= 1024 &&
                  workspace_bytes >= gather_tc_workspace(batch, M, K, n_experts) && batch * M >= 8 * n_experts &&
                  K % 64 == 0 && batch * M < (1LL << 30) && aligned(workspace, 256);
  if (!tc)
    return vmlx_cuda_gather_qmm(y, x, w, scales, biases, lhs_indices, rhs_indices, transpose, group_size, bits, mode,
                                sorted_indices, batch, x_batches, M, N, K, n_experts, stream);
  int rc = check_mm_args(y, x, w, scales, biases, transpose, group_size, bits, mode, M, N, K);
  if (rc) return rc;
  if (batch % x_batches && !lhs_indices)
    return set_error(VMLX_E_INVALID, "without lhs_indices, batch=%lld must be a multiple of x_batches=%lld",
                     (long long)batch, (long long)x_batches);
  return launch_gather_tc((const bf16*)x, w, (const bf16*)scales, (const bf16*)biases, lhs_indices, rhs_indices,
                          (bf16*)y, batch, x_batches, M, N, K, n_experts, bits, group_size, workspace,
                          as_stream(stream));
}
