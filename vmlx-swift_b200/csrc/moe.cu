// moe.cu -- the MoE routing step around SwitchGLU, on the device.
//
//  * vmlx_cuda_moe_route   Qwen3MoESparseMoeBlock routing (Libraries/MLXLLM/Models/
//    Qwen3MoE.swift:137-148): softmax(gates, precise) in fp32, the top-k experts of the
//    gates, their softmax scores, optional renormalisation.
//  * vmlx_cuda_moe_sort    gatherSort (Libraries/MLXLMCommon/SwitchLayers.swift:64-75):
//    the (token, slot) pairs sorted by expert, stably, as argSort of the flattened
//    indices; emits the sorted expert ids, the x row of every sorted pair (order / k,
//    passed to gather_qmm as lhs_indices instead of copying x) and the inverse order.
//  * vmlx_cuda_moe_combine scatterUnsort + the score-weighted sum of the block
//    (SwitchLayers.swift:77-83, Qwen3MoE.swift:150-151): out[t] = sum_j y[inv[t*k+j]] *
//    scores[t, j]; with bf16 scores each product is rounded to bf16 (the reference's
//    bf16 multiply), with fp32 scores it stays fp32 (MLX promotes the product); the sum
//    over j is fp32 (MLX's sum accumulates in fp32) and the result is rounded to bf16.
//
// All three are latency-sized (a few KB); one warp per token row for routing, one CTA
// for the sort (a counting sort: histogram, scan, then a stable placement pass in
// rounds of CTA-size pairs), one CTA column per token for the combine.
#include "kernels.cuh"

namespace vmlx {

constexpr int MOE_MAX_E = 1024;    // experts per routing row (32 per lane)
constexpr int MOE_MAX_K = 32;
constexpr int SORT_THREADS = 1024;
constexpr int SORT_MAX_E = 1024;   // experts of the sort's histogram (shared memory)

template <typename T>
__device__ __forceinline__ float ld_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_f<bf16>(const bf16* p, int64_t i) { return __bfloat162float(p[i]); }

template <typename T>
__device__ __forceinline__ void st_f(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void st_f<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st_f<bf16>(bf16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }
template <typename T>
__device__ __forceinline__ float round_t(float v);
template <>
__device__ __forceinline__ float round_t<float>(float v) { return v; }
template <>
__device__ __forceinline__ float round_t<bf16>(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// One warp per token row.  Top-k: k rounds of a warp arg-max over the gates (larger
// gate first, the lower expert id on ties), so the ids come out in descending gate
// order -- one valid order of argPartition's unordered top-k.  Scores are the softmax
// probabilities at those ids, in the logits' dtype (softmax(precise) computes in fp32
// and returns the input dtype).
template <typename T>
__global__ void moe_route_kernel(const T* __restrict__ logits, int64_t rows, int E, int k, int norm,
                                 uint32_t* __restrict__ inds, T* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  constexpr int PER = MOE_MAX_E / 32;
  float v[PER];
  const T* lr = logits + row * E;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; i++) {
    const int e = i * 32 + lane;
    v[i] = e < E ? ld_f<T>(lr, e) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER; i++)
    if (i * 32 + lane < E) sum += expf(v[i] - mx);
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  uint32_t taken = 0;  // bit i: this lane's slot i already selected
  float sel_score[MOE_MAX_K];
  uint32_t sel_id[MOE_MAX_K];
  float ssum = 0.f;
  for (int r = 0; r < k; r++) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      const int e = i * 32 + lane;
      if (e < E && !(taken >> i & 1u) && (v[i] > best || (v[i] == best && e < bi))) {
        best = v[i];
        bi = e;
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (bi != 0x7fffffff && (bi & 31) == lane) taken |= 1u << (bi >> 5);
    const float p = round_t<T>(expf(best - mx) / sum);  // softmax output in T
    sel_score[r < MOE_MAX_K ? r : 0] = p;
    sel_id[r < MOE_MAX_K ? r : 0] = (uint32_t)bi;
    ssum += p;
  }
  if (lane == 0) {
    const float denom = round_t<T>(ssum);  // sum(scores) in T (fp32 accumulation)
    for (int r = 0; r < k; r++) {
      inds[row * k + r] = sel_id[r];
      st_f<T>(scores, row * k + r, norm ? sel_score[r] / denom : sel_score[r]);
    }
  }
}

// Counting sort of P expert ids (stable).  Pass 1: histogram; scan -> first sorted
// position of each expert.  Pass 2, in rounds of SORT_THREADS pairs: a pair's rank among
// equal ids of its round is the number of equal ids in earlier warps of the round
// (per-warp counts in shared memory) plus those in earlier lanes (match_any), and the
// expert's cursor advances by the round's count -- so equal ids keep their input order.
__global__ void __launch_bounds__(SORT_THREADS) moe_sort_kernel(const uint32_t* __restrict__ idx, int64_t P, int m,
                                                                int E, uint32_t* __restrict__ sorted_ids,
                                                                uint32_t* __restrict__ lhs, uint32_t* __restrict__ inv,
                                                                int* __restrict__ status) {
  extern __shared__ int sm[];
  int* cursor = sm;                    // [E]
  int* wcnt = sm + E;                  // [32 warps][E] counts of the current round
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += SORT_THREADS) cursor[e] = 0;
  __syncthreads();
  bool bad = false;
  for (int64_t i = tid; i < P; i += SORT_THREADS) {
    const uint32_t e = idx[i];
    if (e < (uint32_t)E) atomicAdd(&cursor[e], 1); else bad = true;
  }
  __syncthreads();
  if (tid == 0) {  // exclusive scan (E <= SORT_MAX_E: a single thread is fast enough at decode sizes)
    int run = 0;
    for (int e = 0; e < E; e++) { const int c = cursor[e]; cursor[e] = run; run += c; }
  }
  __syncthreads();
  for (int64_t base = 0; base < P; base += SORT_THREADS) {
    for (int i = tid; i < 32 * E; i += SORT_THREADS) wcnt[i] = 0;
    __syncthreads();
    const int64_t i = base + tid;
    const bool act = i < P;
    const uint32_t e = act ? idx[i] : 0xffffffffu;
    const bool ok = act && e < (uint32_t)E;
    const unsigned same = __match_any_sync(0xffffffffu, ok ? e : 0xffffffffu);
    const int rank_w = __popc(same & ((1u << lane) - 1u));
    if (ok && rank_w == 0) wcnt[warp * E + e] = __popc(same);
    __syncthreads();
    if (ok) {
      int before = 0;
      for (int w = 0; w < warp; w++) before += wcnt[w * E + e];
      const int pos = cursor[e] + before + rank_w;
      sorted_ids[pos] = e;
      lhs[pos] = (uint32_t)(i / m);
      inv[i] = (uint32_t)pos;
    }
    __syncthreads();
    // advance cursors by this round's counts
    for (int ee = tid; ee < E; ee += SORT_THREADS) {
      int c = 0;
      for (int w = 0; w < 32; w++) c += wcnt[w * E + ee];
      cursor[ee] += c;
    }
    __syncthreads();
  }
  if (bad && status) atomicExch(status, VMLX_E_INVALID);
}

// out[t, d] = bf16( sum_j float(bf16(y[src(t, j), d] * s[t, j])) ), src = inv[t*k + j] or t*k + j.
template <typename TS>
__global__ void moe_combine_kernel(const bf16* __restrict__ y, const uint32_t* __restrict__ inv,
                                   const TS* __restrict__ scores, int64_t T, int k, int64_t D,
                                   bf16* __restrict__ out) {
  const int64_t t = blockIdx.y;
  const int64_t d0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (t >= T || d0 >= D) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < k; j++) {
    const int64_t pair = t * k + j;
    const int64_t src = inv ? (int64_t)inv[pair] : pair;
    const float s = ld_f<TS>(scores, pair);
    const bf16* yr = y + src * D + d0;
    if (d0 + 8 <= D) {
      const uint4 v = *reinterpret_cast<const uint4*>(yr);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 f = __bfloat1622float2(u32_as_bf162(u[q]));
        acc[2 * q] += round_t<TS>(f.x * s);
        acc[2 * q + 1] += round_t<TS>(f.y * s);
      }
    } else {
      for (int q = 0; q < 8 && d0 + q < D; q++) acc[q] += round_t<TS>(__bfloat162float(yr[q]) * s);
    }
  }
  for (int q = 0; q < 8 && d0 + q < D; q++) out[t * D + d0 + q] = __float2bfloat16_rn(acc[q]);
}


// ---- sorted gather_qmm on the tensor cores: slots and row gather ----------------------

// Slots of the expert-segmented GEMM: rows (b, m) of a sorted gather (rhs non-decreasing,
// M rows per batch element) are grouped by expert into tiles of <= QMM_SLOT_ROWS rows:
// slot = {expert, first row, rows}; the first `cap` entries are written, unused ones
// with rows = 0.  One CTA; a thread per expert (binary search of its run in rhs) and a
// shared-memory scan of the per-expert slot counts.
constexpr int QMM_SLOT_ROWS = 64;
__global__ void __launch_bounds__(1024) qmm_slots_kernel(const uint32_t* __restrict__ rhs, int64_t batch, int64_t M,
                                                         int E, int4* __restrict__ slots, int64_t cap) {
  __shared__ int scan[1024];
  const int tid = threadIdx.x;
  int64_t lo = 0, hi = 0;
  int ns = 0;
  if (tid < E) {
    int64_t a = 0, b = batch;
    while (a < b) { const int64_t mid = (a + b) >> 1; if (rhs[mid] < (uint32_t)tid) a = mid + 1; else b = mid; }
    lo = a;
    b = batch;
    while (a < b) { const int64_t mid = (a + b) >> 1; if (rhs[mid] < (uint32_t)tid + 1) a = mid + 1; else b = mid; }
    hi = a;
    ns = (int)(((hi - lo) * M + QMM_SLOT_ROWS - 1) / QMM_SLOT_ROWS);
  }
  scan[tid] = ns;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {  // inclusive Hillis-Steele scan
    const int v = tid >= o ? scan[tid - o] : 0;
    __syncthreads();
    scan[tid] += v;
    __syncthreads();
  }
  const int total = scan[1023];
  const int first = scan[tid] - ns;
  for (int j = 0; j < ns; j++) {
    const int64_t r0 = lo * M + (int64_t)j * QMM_SLOT_ROWS, r1 = hi * M;
    if (first + j < cap)
      slots[first + j] = make_int4(tid, (int)r0, (int)(r1 - r0 < QMM_SLOT_ROWS ? r1 - r0 : QMM_SLOT_ROWS), 0);
  }
  for (int64_t i = total + tid; i < cap; i += 1024) slots[i] = make_int4(0, 0, 0, 0);
}

// xs[b*M + m] = x[(lhs ? lhs[b] : b*x_batches/batch)*M + m] (bf16 rows of K), and y rows of
// batch elements whose expert id is out of range set to zero (no slot covers them).
__global__ void gather_rows_kernel(const bf16* __restrict__ x, const uint32_t* __restrict__ lhs, int64_t x_batches,
                                   int64_t batch, int64_t M, int64_t K, const uint32_t* __restrict__ rhs, int E,
                                   bf16* __restrict__ xs, bf16* __restrict__ y, int64_t N) {
  const int64_t r = blockIdx.x, b = r / M, m = r - b * M;
  if (xs) {
    const int64_t xi = lhs ? (int64_t)lhs[b] : b * x_batches / batch;
    const uint4* src = reinterpret_cast<const uint4*>(x + (xi * M + m) * K);
    uint4* dst = reinterpret_cast<uint4*>(xs + r * K);
    for (int64_t i = threadIdx.x; i < K / 8; i += blockDim.x) dst[i] = src[i];
  }
  if (rhs[b] >= (uint32_t)E)
    for (int64_t i = threadIdx.x; i < N; i += blockDim.x) y[r * N + i] = __float2bfloat16_rn(0.f);
}

size_t gather_tc_workspace(int64_t batch, int64_t M, int64_t K, int64_t n_experts) {
  const int64_t cap = n_experts + (batch * M + QMM_SLOT_ROWS - 1) / QMM_SLOT_ROWS;
  return (size_t)((cap * 16 + 255) / 256 * 256) + (size_t)batch * M * K * 2;
}

int launch_gather_tc(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases,
                     const uint32_t* lhs, const uint32_t* rhs, bf16* y, int64_t batch, int64_t x_batches,
                     int64_t M, int64_t N, int64_t K, int64_t n_experts, int bits, int gs, void* ws,
                     cudaStream_t st) {
  const int64_t rows = batch * M;
  const int64_t cap = n_experts + (rows + QMM_SLOT_ROWS - 1) / QMM_SLOT_ROWS;
  int4* slots = reinterpret_cast<int4*>(ws);
  bf16* xs = reinterpret_cast<bf16*>(reinterpret_cast<char*>(ws) + (cap * 16 + 255) / 256 * 256);
  // x already in sorted row order when every batch element reads its own x matrix
  const bool copy = lhs != nullptr || x_batches != batch;
  gather_rows_kernel<<<(unsigned)rows, 128, 0, st>>>(x, lhs, x_batches, batch, M, K, rhs, (int)n_experts,
                                                     copy ? xs : nullptr, y, N);
  int rc = check_launch("gather_rows_kernel");
  if (rc) return rc;
  qmm_slots_kernel<<<1, 1024, 0, st>>>(rhs, batch, M, (int)n_experts, slots, cap);
  rc = check_launch("qmm_slots_kernel");
  if (rc) return rc;
  return launch_qmm_tc_grouped(copy ? xs : x, w, scales, biases, y, rows, N, K, n_experts, slots, cap, bits, gs, st);
}

}  // namespace vmlx

using namespace vmlx;

extern "C" int vmlx_cuda_moe_route(const void* logits, int dtype, int64_t rows, int n_experts, int k,
                                   bool norm_topk_prob, uint32_t* indices, void* scores, void* stream) {
  if (rows < 0 || n_experts < 1 || n_experts > MOE_MAX_E || k < 1 || k > MOE_MAX_K || k > n_experts)
    return set_error(VMLX_E_INVALID, "moe_route: rows=%lld experts=%d k=%d (experts <= %d, k <= %d)",
                     (long long)rows, n_experts, k, MOE_MAX_E, MOE_MAX_K);
  if (rows == 0) return VMLX_OK;
  if (!logits || !indices || !scores) return set_error(VMLX_E_INVALID, "moe_route: null pointer");
  const int wpb = 4;
  const dim3 grid((unsigned)((rows + wpb - 1) / wpb));
  cudaStream_t st = as_stream(stream);
  if (dtype == VMLX_F32)
    moe_route_kernel<float><<<grid, 32 * wpb, 0, st>>>((const float*)logits, rows, n_experts, k, norm_topk_prob,
                                                        indices, (float*)scores);
  else if (dtype == VMLX_BF16)
    moe_route_kernel<bf16><<<grid, 32 * wpb, 0, st>>>((const bf16*)logits, rows, n_experts, k, norm_topk_prob,
                                                       indices, (bf16*)scores);
  else
    return set_error(VMLX_E_UNSUPPORTED, "moe_route: logits dtype %d (float32 or bfloat16)", dtype);
  return check_launch("moe_route_kernel");
}

extern "C" int vmlx_cuda_moe_sort(const uint32_t* indices, int64_t pairs, int k, int n_experts,
                                  uint32_t* sorted_indices, uint32_t* lhs_indices, uint32_t* inverse_order,
                                  int* status, void* stream) {
  if (pairs < 0 || k < 1 || n_experts < 1 || n_experts > SORT_MAX_E || pairs >= (1LL << 31))
    return set_error(VMLX_E_INVALID, "moe_sort: pairs=%lld k=%d experts=%d (experts <= %d)", (long long)pairs, k,
                     n_experts, SORT_MAX_E);
  if (pairs == 0) return VMLX_OK;
  if (!indices || !sorted_indices || !lhs_indices || !inverse_order)
    return set_error(VMLX_E_INVALID, "moe_sort: null pointer");
  const size_t smem = (size_t)33 * n_experts * sizeof(int);
  if (smem > 200 * 1024) return set_error(VMLX_E_UNSUPPORTED, "moe_sort: %d experts need too much shared memory",
                                          n_experts);
  {
    const int rc = ensure_max_dynamic_smem((const void*)moe_sort_kernel, 200 * 1024);
    if (rc) return rc;
  }
  moe_sort_kernel<<<1, SORT_THREADS, smem, as_stream(stream)>>>(indices, pairs, k, n_experts, sorted_indices,
                                                                lhs_indices, inverse_order, status);
  return check_launch("moe_sort_kernel");
}

extern "C" int vmlx_cuda_moe_combine(const void* y, const uint32_t* inverse_order, const void* scores,
                                     int scores_dtype, int64_t rows, int k, int64_t dims, void* out, void* stream) {
  if (rows < 0 || k < 1 || dims < 1) return set_error(VMLX_E_INVALID, "moe_combine: bad shape");
  if (rows == 0) return VMLX_OK;
  if (!y || !scores || !out) return set_error(VMLX_E_INVALID, "moe_combine: null pointer");
  if (dims % 8 || !aligned(y, 16)) return set_error(VMLX_E_INVALID, "moe_combine: dims must be a multiple of 8");
  if (rows > 65535) return set_error(VMLX_E_UNSUPPORTED, "moe_combine: rows=%lld > 65535", (long long)rows);
  const int thr = 128;
  const dim3 grid((unsigned)((dims / 8 + thr - 1) / thr), (unsigned)rows);
  cudaStream_t st = as_stream(stream);
  if (scores_dtype == VMLX_F32)
    moe_combine_kernel<float><<<grid, thr, 0, st>>>((const bf16*)y, inverse_order, (const float*)scores, rows, k,
                                                    dims, (bf16*)out);
  else if (scores_dtype == VMLX_BF16)
    moe_combine_kernel<bf16><<<grid, thr, 0, st>>>((const bf16*)y, inverse_order, (const bf16*)scores, rows, k,
                                                   dims, (bf16*)out);
  else
    return set_error(VMLX_E_UNSUPPORTED, "moe_combine: scores dtype %d", scores_dtype);
  return check_launch("moe_combine_kernel");
}
