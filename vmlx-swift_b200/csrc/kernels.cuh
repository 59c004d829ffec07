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

constexpr int QMV_TP_MAX_WORLD = 8;  // ranks a fused row-parallel GEMV reduces over

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
  // x_swiglu (dense): x is a [M, 2K] gate||up buffer and the GEMV input is
  // bf16(bf16(silu(gate)) * up), computed while x is staged (the SwiGLU of the MLP fused
  // into the down projection)
  int x_swiglu;
  // Row-parallel tensor parallelism (tp_world > 1, dense mode): the bf16 partial y of
  // this rank goes into slot [parity][tp_rank] of every rank's buffer over P2P; each
  // CTA then waits for the same CTA of every rank and reduces its rows in rank order:
  //   y = bf16(residual + bf16(sum_r partial_r)).
  char* tp_buf[QMV_TP_MAX_WORLD];  // every rank's TP buffer base, as seen from this device
  int tp_rank, tp_world;
  size_t tp_slot_bytes;                             // bytes per rank slot
  size_t tp_slots_off, tp_flags_off, tp_epoch_off;  // regions inside each buffer
  uint64_t tp_timeout_ns;
  int* tp_status;  // set to VMLX_E_PEER_TIMEOUT when a peer wait runs out
  // Loopback group (tp_loop = 1): every rank of the group lives on this device and the
  // ranks run as one grid, rank = blockIdx.y.  x / y / residual hold all ranks' rows
  // stacked along a leading rank axis ([world, M, .]) and the weights all ranks' shards
  // stacked along N ([world * N, .]).
  int tp_loop;
};

constexpr int TP_FUSED_MAXC = 1024;  // CTAs of a fused TP GEMV grid (flag slots per rank)

// Streaming decode GEMV for 1..4 token rows (dense mode, no TP); launch_qmv routes
// the calls it covers to it.
bool qgemv_covers(const QmvArgs& a, int mode, int bits, int gs);
int launch_qgemv(const QmvArgs& a, int bits, int gs, cudaStream_t st);

int launch_qmv(const QmvArgs& a, int mode, int bits, int gs, int64_t zcount, int toka, cudaStream_t st);

// tcgen05 GEMM for M > 32; sets *handled = false when the shape is not covered.
int launch_qmm_tc(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases, bf16* y,
                  int64_t M, int64_t N, int64_t K, int bits, int gs, cudaStream_t st, bool* handled);

// Expert-segmented tcgen05 GEMM (sorted gather_qmm): slots {expert, first row, rows}.
int launch_qmm_tc_grouped(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases, bf16* y,
                          int64_t M, int64_t N, int64_t K, int64_t n_experts, const int4* slots, int64_t n_slots,
                          int bits, int gs, cudaStream_t st);
// Sorted gather_qmm on the tensor cores: row gather + slots + grouped GEMM, in `ws`
// (gather_tc_workspace bytes).
size_t gather_tc_workspace(int64_t batch, int64_t M, int64_t K, int64_t n_experts);
int launch_gather_tc(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases,
                     const uint32_t* lhs, const uint32_t* rhs, bf16* y, int64_t batch, int64_t x_batches,
                     int64_t M, int64_t N, int64_t K, int64_t n_experts, int bits, int gs, void* ws,
                     cudaStream_t st);

}  // namespace vmlx
