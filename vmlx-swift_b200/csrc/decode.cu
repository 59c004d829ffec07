// decode.cu -- the pieces of a full decode step around the quantized linears: quantized
// embedding lookup, RoPE with the per-head q/k RMSNorm of Qwen3 and a cache position read
// from device memory, greedy sampling, and the device-side position counter.
//
// Replaces, for the token loop of Libraries/MLXLMCommon/Evaluate.swift:2505-2578:
//   * QuantizedEmbedding.callAsFunction (Source/MLXNN/Quantized.swift:229-236):
//     dequantized(weight[ids], scales[ids], biases[ids]) -- one output row per token id;
//   * Qwen3Attention's qNorm / kNorm + RoPE + KVCacheSimple.update
//     (Libraries/MLXLLM/Models/Qwen3.swift:75-80, Libraries/MLXLMCommon/KVCache.swift:452-470);
//   * ArgMaxSampler (Libraries/MLXLMCommon/Evaluate.swift:515-521): argMax(logits, axis: -1),
//     the first index of the maximum.
// The position lives in device memory so that one captured CUDA graph serves every step:
// the step's kernels read it, and vmlx_cuda_advance moves it at the end of the step.
#include "kernels.cuh"

namespace vmlx {

// ---- quantized embedding: one CTA per token row ----
template <int BITS>
__global__ void embed_kernel(const int32_t* __restrict__ ids, const uint32_t* __restrict__ wq,
                             const bf16* __restrict__ scales, const bf16* __restrict__ biases,
                             bf16* __restrict__ out, int64_t n, int vocab, int dims, int gs, int* status) {
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
  const int id = ids[r];
  bf16* orow = out + r * dims;
  if (id < 0 || id >= vocab) {  // out of range: zeros and a status, never an out-of-bounds read
    for (int k = threadIdx.x; k < dims; k += blockDim.x) orow[k] = __float2bfloat16_rn(0.f);
    if (threadIdx.x == 0 && status) atomicExch(status, VMLX_E_INVALID);
    continue;
  }
  constexpr int PER = 32 / BITS;
  const int words = dims / PER;
  const uint32_t* wrow = wq + (int64_t)id * words;
  const bf16* srow = scales + (int64_t)id * (dims / gs);
  const bf16* brow = biases + (int64_t)id * (dims / gs);
  for (int i = threadIdx.x; i < words; i += blockDim.x) {
    const int k0 = i * PER, g = k0 / gs;
    const float s = __bfloat162float(srow[g]), b = __bfloat162float(brow[g]);
    const uint32_t w = wrow[i];
#pragma unroll
    for (int j = 0; j < PER; j++) {
      // affine_dequantize in bfloat: the product rounds to bf16 before the add
      const float q = (float)((w >> (BITS * j)) & ((1u << BITS) - 1u));
      const float prod = __bfloat162float(__float2bfloat16_rn(__fmul_rn(s, q)));
      orow[k0 + j] = __float2bfloat16_rn(__fadd_rn(prod, b));
    }
  }
  }
}

// ---- RoPE (+ per-head RMSNorm of q and k) + KV-cache append at a device position ----
// One warp per (row, head) of q | k | v; head_dim 64..256 in steps of 64 (lane holds the
// pairs (d, d + D/2) for d = lane + 32 j).  tokens_per_seq = 0: row r is sequence r at the
// base position (decode); T > 0: row r is token r % T of sequence r / T at base + r % T
// (prefill).  base = *pos_dev when pos_dev is given, else pos.
template <int D>
__global__ void rope_norm_kernel(const bf16* __restrict__ qkv, bf16* __restrict__ q_out, bf16* __restrict__ kc,
                                 bf16* __restrict__ vc, int Hq, int Hkv, const int32_t* __restrict__ pos_dev,
                                 int pos, int tokens_per_seq, int max_len, const bf16* __restrict__ qn,
                                 const bf16* __restrict__ kn, float eps, float log2_base, float scale,
                                 int* status) {
  constexpr int HALF = D / 2, PL = HALF / 32;  // pairs per lane
  const int H = Hq + 2 * Hkv;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.y;
  if (warp >= H) return;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the position and qkv come from earlier kernels
  const int base = pos_dev ? pos_dev[0] : pos;
  const int p = tokens_per_seq ? base + r % tokens_per_seq : base;
  const int seq = tokens_per_seq ? r / tokens_per_seq : r;
  if (p < 0 || p >= max_len) {
    if (lane == 0 && status) atomicExch(status, VMLX_E_INVALID);
    return;
  }
  const bf16* src = qkv + ((int64_t)r * H + warp) * D;
  if (warp >= Hq + Hkv) {  // v: copy into the cache
    bf16* dst = vc + (((int64_t)seq * Hkv + (warp - Hq - Hkv)) * max_len + p) * D;
    for (int d = lane; d < D; d += 32) dst[d] = src[d];
    return;
  }
  const bool is_q = warp < Hq;
  float x1[PL], x2[PL];
#pragma unroll
  for (int j = 0; j < PL; j++) {
    x1[j] = __bfloat162float(src[lane + 32 * j]);
    x2[j] = __bfloat162float(src[lane + 32 * j + HALF]);
  }
  const bf16* nw = is_q ? qn : kn;
  if (nw) {  // RMSNorm over the head: n = bf16(x * rsqrt(mean(x^2) + eps)), out = bf16(w * n)
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PL; j++) ss = fmaf(x1[j], x1[j], fmaf(x2[j], x2[j], ss));
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int j = 0; j < PL; j++) {
      const int d = lane + 32 * j;
      const float n1 = __bfloat162float(__float2bfloat16_rn(x1[j] * inv));
      const float n2 = __bfloat162float(__float2bfloat16_rn(x2[j] * inv));
      x1[j] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(nw[d]) * n1));
      x2[j] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(nw[d + HALF]) * n2));
    }
  }
  bf16* dst = is_q ? q_out + ((int64_t)r * Hq + warp) * D
                   : kc + (((int64_t)seq * Hkv + (warp - Hq)) * max_len + p) * D;
#pragma unroll
  for (int j = 0; j < PL; j++) {
    const int d = lane + 32 * j;
    const float inv_freq = exp2f(-((float)d / (float)HALF) * log2_base);
    float sn, cs;
    sincosf(scale * (float)p * inv_freq, &sn, &cs);
    dst[d] = __float2bfloat16_rn(x1[j] * cs - x2[j] * sn);
    dst[d + HALF] = __float2bfloat16_rn(x1[j] * sn + x2[j] * cs);
  }
}

// ---- greedy sampling: the first index of the row maximum (NaN never wins) ----
constexpr int AM_THREADS = 1024;
__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(const bf16* __restrict__ logits, int32_t* __restrict__ out,
                                                            int64_t V) {
  const bf16* row = logits + (int64_t)blockIdx.x * V;
  float best = -INFINITY;
  int64_t bi = V;  // "none yet": larger than every index
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int64_t i = threadIdx.x; i < V; i += AM_THREADS) {
    const float v = __bfloat162float(row[i]);
    if (v > best) { best = v; bi = i; }  // strictly greater: the first index wins within a thread
  }
  // (value, index) reduction: larger value, then smaller index
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  __shared__ float sv[AM_THREADS / 32];
  __shared__ int64_t si[AM_THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = lane < AM_THREADS / 32 ? sv[lane] : -INFINITY;
    bi = lane < AM_THREADS / 32 ? si[lane] : V;
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) out[blockIdx.x] = (int32_t)(bi < V ? bi : 0);  // an all-NaN row samples token 0
  }
}

__global__ void advance_kernel(int32_t* counter, int32_t delta) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  counter[0] += delta;
}

}  // namespace vmlx

using namespace vmlx;

extern "C" int vmlx_cuda_quantized_embedding(void* out, const int32_t* ids, const uint32_t* w, const void* scales,
                                             const void* biases, int group_size, int bits, int64_t n, int64_t vocab,
                                             int64_t dims, int* status, void* stream) {
  if (n == 0) return VMLX_OK;
  if (!out || !ids || !w || !scales || !biases) return set_error(VMLX_E_INVALID, "quantized_embedding: null pointer");
  if (bits != 2 && bits != 4 && bits != 8) return set_error(VMLX_E_UNSUPPORTED, "bits=%d not supported", bits);
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return set_error(VMLX_E_UNSUPPORTED, "group_size=%d not supported", group_size);
  if (n < 0 || n >= (1LL << 31) || vocab <= 0 || vocab >= (1LL << 31) || dims <= 0 || dims % group_size)
    return set_error(VMLX_E_INVALID, "quantized_embedding: n=%lld vocab=%lld dims=%lld", (long long)n,
                     (long long)vocab, (long long)dims);
  const cudaStream_t st = as_stream(stream);
  const unsigned grid = (unsigned)(n < 65535 ? n : 65535);
  if (bits == 2)
    embed_kernel<2><<<grid, 256, 0, st>>>(ids, w, (const bf16*)scales, (const bf16*)biases, (bf16*)out, n,
                                                 (int)vocab, (int)dims, group_size, status);
  else if (bits == 4)
    embed_kernel<4><<<grid, 256, 0, st>>>(ids, w, (const bf16*)scales, (const bf16*)biases, (bf16*)out, n,
                                                 (int)vocab, (int)dims, group_size, status);
  else
    embed_kernel<8><<<grid, 256, 0, st>>>(ids, w, (const bf16*)scales, (const bf16*)biases, (bf16*)out, n,
                                                 (int)vocab, (int)dims, group_size, status);
  return check_launch("embed_kernel");
}

extern "C" int vmlx_cuda_rope_qk_norm(void* q_out, void* k_cache, void* v_cache, const void* qkv, int64_t rows,
                                      int n_heads, int n_kv_heads, int head_dim, const int32_t* pos_dev, int64_t pos,
                                      int tokens_per_seq, int64_t max_len, const void* q_norm, const void* k_norm,
                                      float eps, float base, float scale, int* status, void* stream) {
  if (rows == 0) return VMLX_OK;
  if (!q_out || !k_cache || !v_cache || !qkv) return set_error(VMLX_E_INVALID, "rope_qk_norm: null pointer");
  if (head_dim != 64 && head_dim != 128 && head_dim != 256)
    return set_error(VMLX_E_UNSUPPORTED, "rope_qk_norm: head_dim=%d (64, 128, 256)", head_dim);
  if (n_heads <= 0 || n_kv_heads <= 0 || rows < 0 || rows > 65535 || max_len <= 0 || max_len >= (1LL << 31) ||
      tokens_per_seq < 0 || (tokens_per_seq && rows % tokens_per_seq) ||
      (!pos_dev && (pos < 0 || pos + (tokens_per_seq ? tokens_per_seq : 1) > max_len)))
    return set_error(VMLX_E_INVALID, "rope_qk_norm: rows=%lld pos=%lld max_len=%lld", (long long)rows,
                     (long long)pos, (long long)max_len);
  const int H = n_heads + 2 * n_kv_heads;
  dim3 grid((unsigned)((H + 7) / 8), (unsigned)rows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  const float lb = log2f(base);
  cudaError_t e;
#define VMLX_ROPE(DD)                                                                                          \
  e = cudaLaunchKernelEx(&cfg, rope_norm_kernel<DD>, (const bf16*)qkv, (bf16*)q_out, (bf16*)k_cache,          \
                         (bf16*)v_cache, n_heads, n_kv_heads, pos_dev, (int)pos, tokens_per_seq, (int)max_len, \
                         (const bf16*)q_norm, (const bf16*)k_norm, eps, lb, scale, status)
  if (head_dim == 64) VMLX_ROPE(64);
  else if (head_dim == 128) VMLX_ROPE(128);
  else VMLX_ROPE(256);
#undef VMLX_ROPE
  return check_cuda(e, "rope_norm_kernel launch");
}

extern "C" int vmlx_cuda_argmax(int32_t* out, const void* logits, int64_t rows, int64_t vocab, void* stream) {
  if (rows == 0) return VMLX_OK;
  if (!out || !logits) return set_error(VMLX_E_INVALID, "argmax: null pointer");
  if (rows < 0 || rows > 65535 || vocab <= 0 || vocab >= (1LL << 31))
    return set_error(VMLX_E_INVALID, "argmax: rows=%lld vocab=%lld", (long long)rows, (long long)vocab);
  argmax_kernel<<<(unsigned)rows, AM_THREADS, 0, as_stream(stream)>>>((const bf16*)logits, out, vocab);
  return check_launch("argmax_kernel");
}

extern "C" int vmlx_cuda_advance(int32_t* counter, int32_t delta, void* stream) {
  if (!counter) return set_error(VMLX_E_INVALID, "advance: null pointer");
  advance_kernel<<<1, 1, 0, as_stream(stream)>>>(counter, delta);
  return check_launch("advance_kernel");
}
