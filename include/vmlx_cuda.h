/*
 * vmlx_cuda.h -- C ABI of the B200 (sm_100a) affine-quantized linear path.
 *
 * Drop-in device-side replacement for the entry points that vmlx-swift's
 * QuantizedLinear / SwitchGLU / MLXDistributedTP layers reach through mlx-c
 * and CmlxDistributedShim.  Every function:
 *   - takes plain device pointers and sizes (no framework types);
 *   - is stream ordered on the `stream` argument (a cudaStream_t passed as
 *     void*, NULL = legacy default stream) and never synchronises the host,
 *     so calls can be captured into a CUDA graph;
 *   - allocates nothing on the hot path: outputs are caller-allocated;
 *   - returns VMLX_OK (0) or a VMLX_E_* code and leaves a description in the
 *     calling thread's vmlx_last_error() (the mlx-c convention of returning a
 *     nonzero int plus an error handler, Source/Cmlx/include/mlx/c/error.h:15-33);
 *   - never aborts the process and never waits without a bound.
 *
 * Tensor conventions (MLX affine layout, Source/MLX/Ops.swift:2368-2388):
 *   x        bf16  [M, K]                (activations, row major)
 *   w        u32   [N, K*bits/32]        (element k of row n at word k/(32/bits),
 *                                          bit offset bits*(k%(32/bits)))
 *   scales   bf16  [N, K/group_size]
 *   biases   bf16  [N, K/group_size]
 *   y        bf16  [M, N]                y = x @ dequantize(w)^T  (transpose=true)
 * Supported: mode "affine" (or NULL), bits in {2,4,8}, group_size in {32,64,128},
 * transpose = true (the only orientation the quantized layers use,
 * Source/MLXNN/Quantized.swift:367, Libraries/MLXLMCommon/SwitchLayers.swift:500).
 */
#ifndef VMLX_CUDA_H
#define VMLX_CUDA_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VMLX_API __attribute__((visibility("default")))
#else
#define VMLX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define VMLX_OK 0
#define VMLX_E_INVALID 1      /* bad pointer, shape or argument */
#define VMLX_E_UNSUPPORTED 2  /* bits / group_size / mode / transpose not supported */
#define VMLX_E_CUDA 3         /* a CUDA runtime call failed */
#define VMLX_E_PEER_TIMEOUT 4 /* a bounded wait on a peer GPU ran out */
#define VMLX_E_STATE 5        /* handle used in the wrong state */

/* Element types for the dtype arguments. */
#define VMLX_BF16 0
#define VMLX_F32 1

/* Text of the last error raised on the calling thread ("" if none). */
VMLX_API const char* vmlx_last_error(void);

/* ABI version: major*10000 + minor*100 + patch. */
VMLX_API int vmlx_version(void);

/*
 * Launch overlap (programmatic dependent launch) for the streaming kernels:
 * when enabled, a quantized_matmul / gather_qmm grid may start streaming its
 * weights, scales and biases while the previous kernel in the same stream is
 * still running; it waits for that kernel before reading x or writing y.
 * Enable it only when the weights, scales and biases of a call are never
 * written by the kernel launched just before it in the same stream (true for
 * inference with loaded weights).  Off by default.  Process-wide; returns the
 * previous setting.  No counterpart in the reference (MLX schedules its own
 * command buffers).
 */
VMLX_API int vmlx_set_launch_overlap(int enable);

/*
 * Affine quantization of a row-major matrix w [rows, cols].
 * Replaces mlx_quantize (Source/Cmlx/include/mlx/c/ops.h:801-808) for
 * mode "affine"; arithmetic of affine_quantize
 * (Source/Cmlx/mlx-generated/metal/quantized.h:2393-2496).
 * w_dtype = VMLX_BF16 or VMLX_F32; scales/biases are written in the same dtype
 * (MLX returns scales in the input dtype).
 */
VMLX_API int vmlx_cuda_quantize(void* wq, void* scales, void* biases, const void* w, int w_dtype,
                       int64_t rows, int64_t cols, int group_size, int bits, const char* mode,
                       void* stream);

/*
 * Affine dequantization: out[r, k] = scale*q + bias as affine_dequantize computes it
 * (quantized.h:2498-2560): with out_dtype VMLX_F32 an unfused fp32 multiply and add
 * (exact); with out_dtype VMLX_BF16 from bf16 scales the reference's bfloat
 * arithmetic, bf16(bf16(scale*q) + bias), each step rounded to nearest even.
 * Replaces mlx_dequantize (Source/Cmlx/include/mlx/c/ops.h:359-369).
 * scales_dtype gives the dtype of scales/biases.
 */
VMLX_API int vmlx_cuda_dequantize(void* out, int out_dtype, const uint32_t* wq, const void* scales,
                         const void* biases, int scales_dtype, int64_t rows, int64_t cols,
                         int group_size, int bits, const char* mode, void* stream);

/*
 * y [M, N] = x [M, K] @ dequantize(w [N, K])^T, bf16 in/out, fp32 accumulation.
 * Replaces mlx_quantized_matmul (Source/Cmlx/include/mlx/c/ops.h:809-819), the
 * op behind QuantizedLinear.callAsFunction (Source/MLXNN/Quantized.swift:361-376).
 * biases may not be NULL for mode "affine".  M <= 4 runs a decode GEMV kernel
 * (fp32 accumulation over exact codes); M >= 5 runs the tensor-core (tcgen05) GEMM,
 * which, like the reference's affine_qmm_t, multiplies bf16-dequantized weights.
 */
VMLX_API int vmlx_cuda_quantized_matmul(void* y, const void* x, const uint32_t* w, const void* scales,
                               const void* biases, bool transpose, int group_size, int bits,
                               const char* mode, int64_t M, int64_t N, int64_t K, void* stream);

/*
 * Decoder-block fusion of vmlx_cuda_quantized_matmul for decode (M <= 32):
 *   x' = norm_weight * bf16(x * rsqrt(mean(x^2) + eps))   if norm_weight != NULL
 *        (MLXFast.rmsNorm on the input, Llama.swift:118-127 `attention(norm(x))`)
 *   y  = bf16(residual + bf16(x' @ dequantize(w)^T))     if residual != NULL
 *        (the block's residual add; residual may alias y for an in-place update)
 * Same rounding points as the separate kernels.  No counterpart as one call in
 * the reference (MLX runs these as separate ops).
 */
VMLX_API int vmlx_cuda_quantized_matmul_fused(void* y, const void* x, const uint32_t* w, const void* scales,
                                              const void* biases, int group_size, int bits, int64_t M, int64_t N,
                                              int64_t K, const void* norm_weight, float eps, const void* residual,
                                              void* stream);

/*
 * Down projection with the MLP's SwiGLU fused into the GEMV (decode, M <= 32):
 *   y = [residual +] bf16(x @ dequantize(W)^T),  x = bf16(bf16(silu(gate)) * up)
 * with gate_up bf16 [M, 2K] = gate | up; the SwiGLU is computed while x is staged,
 * exactly as vmlx_cuda_silu_mul rounds it (compiledSwiGLU,
 * Libraries/MLXLMCommon/SwitchLayers.swift:40-50, then the down QuantizedLinear of
 * Libraries/MLXLLM/Models/Llama.swift:96-99).  residual may be NULL or alias y.
 */
VMLX_API int vmlx_cuda_quantized_matmul_swiglu(void* y, const void* gate_up, const uint32_t* w, const void* scales,
                                               const void* biases, int group_size, int bits, int64_t M, int64_t N,
                                               int64_t K, const void* residual, void* stream);

/*
 * Gathered quantized matmul over a stack of E expert matrices.
 * Replaces mlx_gather_qmm (Source/Cmlx/include/mlx/c/ops.h:475-488), the op
 * behind QuantizedSwitchLinear.callAsFunction
 * (Libraries/MLXLMCommon/SwitchLayers.swift:491-512).
 *   x        bf16 [x_batches, M, K]
 *   w        u32  [E, N, K*bits/32];  scales/biases bf16 [E, N, K/group_size]
 *   lhs_indices u32 [batch] or NULL.  NULL means each x matrix serves
 *               batch/x_batches consecutive batch elements (b reads x batch
 *               b*x_batches/batch), the row-major broadcast of x [T,1,..]
 *               against indices [T,k] that SwitchGLU relies on
 *               (quantized.h:1438-1491); batch must be a multiple of x_batches.
 *   rhs_indices u32 [batch]  expert of each batch element, or NULL: batch element b
 *                 uses expert b * n_experts / batch (batch a multiple of n_experts),
 *                 MLX's broadcast of the weight stack when no indices are given
 *   y        bf16 [batch, M, N];  y[b] = x[lhs[b]] @ dequantize(w[rhs[b]])^T
 * sorted_indices = true promises rhs_indices is non-decreasing (the
 * gatherSort'ed order, SwitchLayers.swift:64-75); the kernel then streams each
 * expert's weights once for the whole run of batch elements routed to it.
 * Out-of-range expert ids (>= n_experts) produce zero rows.
 */
VMLX_API int vmlx_cuda_gather_qmm(void* y, const void* x, const uint32_t* w, const void* scales,
                         const void* biases, const uint32_t* lhs_indices,
                         const uint32_t* rhs_indices, bool transpose, int group_size, int bits,
                         const char* mode, bool sorted_indices, int64_t batch, int64_t x_batches,
                         int64_t M, int64_t N, int64_t K, int64_t n_experts, void* stream);


/*
 * vmlx_cuda_gather_qmm with a caller-owned device workspace (256-byte aligned, at least
 * vmlx_cuda_gather_qmm_workspace_size(batch, M, K, n_experts) bytes).  A sorted gather
 * (sorted_indices, rhs_indices given, n_experts <= 1024, K a multiple of 64) with on
 * average >= 8 rows per expert runs as an expert-segmented tcgen05 GEMM: one 64-row tile per
 * run of equal experts, bf16-dequantized weights, as affine_gather_qmm_rhs
 * (quantized.h:2197-2391).  Anything else, or a too-small workspace, runs
 * vmlx_cuda_gather_qmm unchanged.  Same argument order as mlx_gather_qmm (ops.h:475-488)
 * plus the workspace.
 */
VMLX_API size_t vmlx_cuda_gather_qmm_workspace_size(int64_t batch, int64_t M, int64_t K, int64_t n_experts);
VMLX_API int vmlx_cuda_gather_qmm_ws(void* y, const void* x, const uint32_t* w, const void* scales,
                                     const void* biases, const uint32_t* lhs_indices,
                                     const uint32_t* rhs_indices, bool transpose, int group_size, int bits,
                                     const char* mode, bool sorted_indices, int64_t batch, int64_t x_batches,
                                     int64_t M, int64_t N, int64_t K, int64_t n_experts, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* ---- MoE routing around SwitchGLU ---- */

/*
 * Top-k routing of a sparse MoE block (Qwen3MoESparseMoeBlock.callAsFunction,
 * Libraries/MLXLLM/Models/Qwen3MoE.swift:137-148):
 *   soft = softmax(logits, precise)  (fp32 math, stored in the logits' dtype)
 *   indices[r, :] = the k experts with the largest logits (descending logit, lower
 *                   id first on ties -- argPartition leaves the order open)
 *   scores[r, :]  = soft at those experts, divided by their sum if norm_topk_prob
 * logits [rows, n_experts] of dtype VMLX_F32 or VMLX_BF16; scores have the same dtype.
 * n_experts <= 1024, k <= 32.
 */
VMLX_API int vmlx_cuda_moe_route(const void* logits, int dtype, int64_t rows, int n_experts, int k,
                                 bool norm_topk_prob, uint32_t* indices, void* scores, void* stream);

/*
 * gatherSort (Libraries/MLXLMCommon/SwitchLayers.swift:64-75) of the flattened
 * routing indices [pairs] (pairs = tokens * k): a stable sort by expert id.
 *   sorted_indices[p] = expert id of sorted pair p           (indices[order])
 *   lhs_indices[p]    = token row of sorted pair p            (order / k) -- pass to
 *                       vmlx_cuda_gather_qmm as lhs_indices instead of gathering x
 *   inverse_order[i]  = sorted position of input pair i       (argSort(order))
 * n_experts <= 1024.  An id >= n_experts sets *status (if given) to VMLX_E_INVALID.
 */
VMLX_API int vmlx_cuda_moe_sort(const uint32_t* indices, int64_t pairs, int k, int n_experts,
                                uint32_t* sorted_indices, uint32_t* lhs_indices, uint32_t* inverse_order,
                                int* status, void* stream);

/*
 * scatterUnsort + the weighted sum of the MoE block (SwitchLayers.swift:77-83,
 * Qwen3MoE.swift:150-151):
 *   out[t, :] = sum_j y[src(t, j), :] * scores[t, j],  src = inverse_order[t*k + j]
 *               (or t*k + j when inverse_order is NULL: y not sorted)
 * y bf16 [rows*k, dims]; scores [rows, k] VMLX_BF16 (each product rounded to bf16, as
 * the reference's bf16 multiply) or VMLX_F32 (products kept in fp32); the sum over j
 * is fp32 and out bf16 [rows, dims].  dims a multiple of 8, rows <= 65535.
 */
VMLX_API int vmlx_cuda_moe_combine(const void* y, const uint32_t* inverse_order, const void* scores,
                                   int scores_dtype, int64_t rows, int k, int64_t dims, void* out, void* stream);


/* ---- decoder-block support kernels (bf16) ---- */

/*
 * out[r, :] = weight * bf16(x[r, :] * rsqrt(mean(x[r, :]^2) + eps)), fp32 sums.
 * Replaces MLXFast.rmsNorm (Source/MLX/MLXFast.swift:230; kernel
 * mlx-generated/metal/rms_norm.metal:13-81).  dims a multiple of 8.
 */
VMLX_API int vmlx_cuda_rms_norm(void* out, const void* x, const void* weight, float eps, int64_t rows,
                                int64_t dims, void* stream);

/*
 * Decode-step RoPE + KV-cache append for a fused qkv projection.
 *   qkv     bf16 [batch, (n_heads + 2*n_kv_heads) * head_dim]   (q | k | v)
 *   q_out   bf16 [batch, n_heads, head_dim]   rotated q
 *   k_cache, v_cache bf16 [batch, n_kv_heads, max_len, head_dim]; the rotated
 *           k and the v of this step are written at position `pos`.
 * Non-traditional rotation of pairs (i, i + head_dim/2) by
 * theta = scale * pos * base^(-2i/head_dim) (mlx-generated/metal/rope.metal:55-229,
 * Libraries/MLXLLM/Models/Llama.swift:66-67; KVCacheSimple.update,
 * Libraries/MLXLMCommon/KVCache.swift:452-470).
 */
VMLX_API int vmlx_cuda_rope_qkv(void* q_out, void* k_cache, void* v_cache, const void* qkv, int64_t batch,
                                int n_heads, int n_kv_heads, int head_dim, int64_t pos, int64_t max_len,
                                float base, float scale, void* stream);

/* Bytes of workspace vmlx_cuda_sdpa_decode needs for these sizes. */
VMLX_API size_t vmlx_cuda_sdpa_decode_workspace(int64_t batch, int n_heads, int64_t kv_len, int head_dim);

/*
 * Decode attention (one query token per sequence) over a bf16 KV cache:
 *   out[b, h, :] = softmax(scale * q[b, h] . K[b, h/G, :kv_len]^T) V[b, h/G, :kv_len]
 * q bf16 [batch, n_heads, 128]; caches as for vmlx_cuda_rope_qkv; G =
 * n_heads / n_kv_heads in 1..8 (grouped-query attention).  fp32 softmax and
 * accumulation.  The cache is split over CTAs of 256 positions; one kernel
 * computes the splits and the last split of each (sequence, kv head) combines
 * them.  `workspace` (caller-owned, vmlx_cuda_sdpa_decode_workspace bytes for
 * the largest kv_len used) holds split counters followed by the per-split
 * partials: it must be zero-filled once before its first use, every call
 * leaves the counters zero again, and a workspace serves one (batch, n_heads)
 * at a time.
 * Replaces MLXFast.scaledDotProductAttention for decode
 * (Source/MLX/MLXFast.swift:118; kernels mlx-generated/metal/sdpa_vector.h:15-394).
 */
VMLX_API int vmlx_cuda_sdpa_decode(void* out, const void* q, const void* k_cache, const void* v_cache,
                                   int64_t batch, int n_heads, int n_kv_heads, int head_dim, int64_t kv_len,
                                   int64_t max_len, float scale, void* workspace, size_t workspace_bytes,
                                   void* stream);

/*
 * Allocation-free variant of vmlx_cuda_sdpa_decode, for callers that cannot
 * allocate device memory where they run attention (a fixed memory pool owned
 * by the engine, a host that forbids allocation on its inference thread, or
 * code that must not risk a cudaMalloc mid-decode).  The per-split partials
 * live in an 8 MiB array inside the library's device image (held on every GPU
 * that loads the library until the process exits), after 64 KiB of split
 * counters; calls needing more (batch * n_heads * ceil(kv_len/256) *
 * (head_dim + 2) * 4 bytes of partials) are rejected with VMLX_E_INVALID.  The first call on a device looks up the
 * array's address with that device current, so make it before any stream
 * capture.  All calls on a device share the array: calls that may overlap on
 * the GPU race.  Nothing needs clearing between calls.  No counterpart in the
 * reference.
 */
VMLX_API int vmlx_cuda_sdpa_decode_noalloc(void* out, const void* q, const void* k_cache, const void* v_cache,
                                           int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                           int64_t kv_len, int64_t max_len, float scale, void* stream);

/*
 * out[r, j] = bf16(bf16(silu(g)) * u) with gate_up bf16 [rows, 2*ffn] = g | u
 * (compiledSwiGLU, Libraries/MLXLMCommon/SwitchLayers.swift:40-50).
 */
VMLX_API int vmlx_cuda_silu_mul(void* out, const void* gate_up, int64_t rows, int64_t ffn, void* stream);

/* out = bf16(a + b), n elements (the residual adds of a decoder block). */
VMLX_API int vmlx_cuda_add(void* out, const void* a, const void* b, int64_t n, void* stream);
/* out[r, c] = bf16(y[r, c] + bias[c]), rows x cols bf16: the optional bias of QuantizedLinear
 * (Source/MLXNN/Quantized.swift:361-376).  out may alias y. */
VMLX_API int vmlx_cuda_bias_add(void* out, const void* y, const void* bias, int64_t rows, int64_t cols, void* stream);

/* ---- MXFP4 block-scaled weights (mode "mxfp4": group_size 32, bits 4) ---- */

/*
 * Quantize w [rows, cols] (VMLX_BF16 / VMLX_F32, cols a multiple of 32) to e2m1 codes wq
 * (u32 [rows, cols/8], eight codes per word, low nibble first) and e8m0 scales (u8 [rows,
 * cols/32]): scale = e8m0(max|w| / 6), code = e2m1(w / scale).  Replaces fp_quantize
 * (Source/Cmlx/mlx-generated/metal/fp_quantized.h:1749-1789) behind mlx_quantize with mode "mxfp4".
 */
VMLX_API int vmlx_cuda_fp_quantize(void* wq, void* scales, const void* w, int w_dtype, int64_t rows, int64_t cols,
                                   int group_size, int bits, const char* mode, void* stream);
/* out [rows, cols] (VMLX_BF16 / VMLX_F32) = scale * e2m1 value, rounded once (fp_quantized.h:1791-1821). */
VMLX_API int vmlx_cuda_fp_dequantize(void* out, int out_dtype, const void* wq, const void* scales, int64_t rows,
                                     int64_t cols, int group_size, int bits, const char* mode, void* stream);
/*
 * y [M, N] bf16 = x [M, K] bf16 @ dequantize(wq [N, K/8], scales [N, K/32])^T with fp32 sums per
 * group scaled by the group's e8m0 scale (MLX's fp qdot, fp_quantized.h:81-100) -- the
 * mlx_quantized_matmul call of a QuantizedLinear in mode "mxfp4".
 */
VMLX_API int vmlx_cuda_fp_quantized_matmul(void* y, const void* x, const void* wq, const void* scales,
                                           int group_size, int bits, const char* mode, int64_t M, int64_t N,
                                           int64_t K, void* stream);

/* ---- the decode loop around the linears (one CUDA graph per token) ---- */

/*
 * Quantized embedding lookup: out[i, :] = dequantize(w[ids[i]], scales[ids[i]], biases[ids[i]])
 * (bf16 arithmetic of affine_dequantize), i < n.  Replaces QuantizedEmbedding.callAsFunction
 * (Source/MLXNN/Quantized.swift:229-236).  w [vocab, dims*bits/32] u32, scales / biases bf16
 * [vocab, dims/group_size].  An id outside [0, vocab) gives a zero row and sets *status (when
 * given) to VMLX_E_INVALID.
 */
VMLX_API int vmlx_cuda_quantized_embedding(void* out, const int32_t* ids, const uint32_t* w, const void* scales,
                                           const void* biases, int group_size, int bits, int64_t n, int64_t vocab,
                                           int64_t dims, int* status, void* stream);

/*
 * RoPE (non-traditional, pairs (i, i + D/2)) of the q and k heads of qkv [rows, (Hq + 2*Hkv) * D],
 * each head first RMS-normalised over D with q_norm / k_norm [D] when given (Qwen3Attention's
 * qNorm / kNorm, Libraries/MLXLLM/Models/Qwen3.swift:75-80; NULL skips the norm), then q to
 * q_out [rows, Hq, D] and k, v appended to the caches [seqs, Hkv, max_len, D]
 * (KVCacheSimple.update, Libraries/MLXLMCommon/KVCache.swift:452-470).  The base position is
 * *pos_dev when pos_dev is not NULL (read on the device: one captured graph serves every
 * step), else pos.  tokens_per_seq = 0: row r is sequence r at the base position (decode);
 * T > 0: row r is token r % T of sequence r / T at base + r % T (prefill of T tokens per sequence).  head_dim 64, 128 or 256.  A position
 * outside the cache skips the row and sets *status (when given) to VMLX_E_INVALID.
 */
VMLX_API int vmlx_cuda_rope_qk_norm(void* q_out, void* k_cache, void* v_cache, const void* qkv, int64_t rows,
                                    int n_heads, int n_kv_heads, int head_dim, const int32_t* pos_dev, int64_t pos,
                                    int tokens_per_seq, int64_t max_len, const void* q_norm, const void* k_norm,
                                    float eps, float base, float scale, int* status, void* stream);

/*
 * vmlx_cuda_sdpa_decode with the cache length read on the device: kv_len = *pos_dev + 1.  The
 * workspace is sized for max_len (vmlx_cuda_sdpa_decode_workspace(batch, n_heads, max_len, 128)).
 */
VMLX_API int vmlx_cuda_sdpa_decode_at(void* out, const void* q, const void* k_cache, const void* v_cache,
                                      int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                      const int32_t* pos_dev, int64_t max_len, float scale, void* workspace,
                                      size_t workspace_bytes, void* stream);

/*
 * Greedy sampling: out[r] = the first index of the maximum of logits[r, :vocab] (bf16), the
 * ArgMaxSampler of Libraries/MLXLMCommon/Evaluate.swift:515-521.
 */
VMLX_API int vmlx_cuda_argmax(int32_t* out, const void* logits, int64_t rows, int64_t vocab, void* stream);

/* *counter += delta on the device (the token loop's position, advanced inside the graph). */
VMLX_API int vmlx_cuda_advance(int32_t* counter, int32_t delta, void* stream);

/* ---- tensor parallelism (one rank per GPU) ---- */

/*
 * A tensor-parallel group member on the current device: the counterpart of
 * vmlx_group_init / vmlx_group_rank / vmlx_group_size
 * (Libraries/CmlxDistributedShim/include/CmlxDistributedShim.h:21-42) for
 * one rank.  Allocates this rank's receive buffer (2 x world x max_bytes
 * slots plus flags); max_bytes bounds the bytes of one all-reduce (multiple
 * of 16).  The handle owns the buffer; vmlx_tp_destroy frees it.
 * Bootstrap: every rank exports vmlx_tp_ipc_handle (64 bytes, a CUDA IPC
 * handle), the handles are exchanged out of band (the Python Group uses
 * torch.distributed), and every rank calls vmlx_tp_open_peers with the
 * world's handles in rank order.  A process driving several GPUs can instead
 * pass peer buffers (vmlx_tp_buffer of the other handles) to vmlx_tp_set_peer.
 */
VMLX_API int vmlx_tp_create(int rank, int world, size_t max_bytes, void** out);
/*
 * A whole group of `world` ranks (2..8) on the current device, run as one grid per
 * call: the single-GPU form of the group, for testing the collective protocol
 * (the same kernels, word formats, epochs and rank-order sums as a group with one
 * GPU per rank) and for hosts with fewer GPUs than ranks.  No reference
 * counterpart (the reference has one process per rank).  On such a handle every
 * data pointer of vmlx_tp_all_sum / vmlx_tp_quantized_matmul_*_all_sum holds all
 * ranks' data stacked along a leading rank axis: in / out [world, n]; x [world, M, K]
 * (gate_up [world, M, 2K]); y and residual [world, M, N]; w / scales / biases the
 * ranks' shards stacked along N ([world * N, ...]).  Each call is one cooperative
 * launch (all ranks' CTAs resident together, else the call fails).
 */
VMLX_API int vmlx_tp_create_loopback(int world, size_t max_bytes, void** out);
VMLX_API int vmlx_tp_rank(void* tp);
VMLX_API int vmlx_tp_size(void* tp);
VMLX_API int vmlx_tp_ipc_handle(void* tp, void* handle_out);
VMLX_API int vmlx_tp_open_peers(void* tp, const void* handles);
VMLX_API int vmlx_tp_set_peer(void* tp, int peer, void* device_ptr);
VMLX_API void* vmlx_tp_buffer(void* tp);
/* Bound of every wait on a peer (default 2 s); after it the call gives up. */
VMLX_API int vmlx_tp_set_timeout_us(void* tp, uint64_t us);

/*
 * out = sum over the group's ranks of `in` (n bf16 elements, n*2 <= max_bytes,
 * 16-byte aligned), identical bits on every rank (fixed rank order, fp32
 * sums).  Replaces vmlx_all_sum (Libraries/CmlxDistributedShim/CmlxDistributedShim.c:54-60)
 * behind Collectives.allSum (Libraries/MLXDistributedTP/Collectives.swift:27-32).
 * One kernel: P2P stores of this rank's data into every rank's buffer; small
 * vectors (n*8 <= max_bytes) as 8-byte {value, epoch} words that the reader
 * polls, larger ones with release/acquire flags at system scope; bounded waits.  Every rank must make
 * the same sequence of calls.  Size 1: a copy.  Stream ordered; graph-capturable.
 */
VMLX_API int vmlx_tp_all_sum(void* tp, void* out, const void* in, int64_t n, void* stream);

/*
 * Row-parallel quantized linear fused with its all-reduce and the residual add
 * (decode, 1 <= M <= 32, M*N*8 <= max_bytes):
 *   y[M, N] = bf16(residual + bf16(sum_r x_r[M, K] @ dequantize(w_r[N, K])^T))
 * where rank r holds the K-shard x_r / w_r (scales / biases [N, K/group_size]).
 * Replaces QuantizedShardedToAllLinear.callAsFunction -> Collectives.allSum
 * (Libraries/MLXDistributedTP/LinearLayers.swift:198-205, Collectives.swift:27-32)
 * plus the decoder residual add (Libraries/MLXLLM/Models/Llama.swift:110-114).
 * One kernel per rank: the GEMV pushes its bf16 partial rows into every rank's
 * slot over NVLink P2P as 8-byte {value, epoch} words; each CTA then polls
 * (bounded) the words of the rows it computed and sums them in rank order, so y has the same bits on
 * every rank.  The partial rows come from the TP instance of the GEMV kernel for the shape; the separate
 * quantized_matmul -> vmlx_tp_all_sum -> add chain may pick another GEMV kernel for the partials and
 * then agrees within the GEMV tolerance, not bitwise.  residual may be NULL or alias y.
 * Every rank must make the same sequence of calls.  Size 1: the local fused GEMV.
 */
VMLX_API int vmlx_tp_quantized_matmul_all_sum(void* tp, void* y, const void* x, const uint32_t* w,
                                              const void* scales, const void* biases, int group_size, int bits,
                                              int64_t M, int64_t N, int64_t K, const void* residual, void* stream);

/*
 * As vmlx_tp_quantized_matmul_all_sum with the MLP's SwiGLU fused into the
 * GEMV's staging of x: gate_up bf16 [M, 2K] = gate | up (this rank's shard), the
 * GEMV input is bf16(bf16(silu(gate)) * up) as vmlx_cuda_silu_mul computes it.
 */
VMLX_API int vmlx_tp_quantized_matmul_swiglu_all_sum(void* tp, void* y, const void* gate_up, const uint32_t* w,
                                                     const void* scales, const void* biases, int group_size,
                                                     int bits, int64_t M, int64_t N, int64_t K, const void* residual,
                                                     void* stream);

/*
 * The MoE block output under expert-intermediate tensor parallelism, in one kernel per rank:
 *   out[t, :] = bf16([residual +] bf16(sum_r bf16(sum_j y_r[inverse_order[t*k + j], :] * scores[t, j])))
 * i.e. vmlx_cuda_moe_combine on this rank's partial expert outputs y_r ([rows*k, dims], each rank
 * holding its slice of every expert's intermediate dimension), all-reduced over the group with the
 * low-latency word protocol of vmlx_tp_all_sum (counts as one all_sum call in the group's
 * sequence; rows*dims*8 <= max_bytes).  Replaces scatterUnsort + the weighted sum
 * (Libraries/MLXLMCommon/SwitchLayers.swift:77-83, Libraries/MLXLLM/Models/Qwen3MoE.swift:150-151)
 * followed by Collectives.allSum (Libraries/MLXDistributedTP/Collectives.swift:27-32).  Size 1:
 * the combine (+ residual).  residual may be NULL or alias out.
 */
VMLX_API int vmlx_tp_moe_combine_all_sum(void* tp, void* out, const void* y, const uint32_t* inverse_order,
                                         const void* scores, int scores_dtype, int64_t rows, int k, int64_t dims,
                                         const void* residual, void* stream);

/*
 * Reads (synchronously) and clears the group's device status word:
 * *code = 0, or VMLX_E_PEER_TIMEOUT if some wait on a peer ran out since the
 * last read.
 */
VMLX_API int vmlx_tp_status(void* tp, int* code);
VMLX_API int vmlx_tp_destroy(void* tp);

#ifdef __cplusplus
}
#endif
#endif /* VMLX_CUDA_H */
