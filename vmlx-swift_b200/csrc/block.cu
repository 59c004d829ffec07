// block.cu -- support kernels of a decoder block in decode: RMSNorm, RoPE with
// KV-cache append, decode attention (split over the cache), SwiGLU, residual add.
//
// They sit on either side of the quantized linears in the reference's decode
// step (Libraries/MLXLLM/Models/Llama.swift:10-127):
//   rms_norm     MLXFast.rmsNorm -> rms_single_row (mlx-generated/metal/rms_norm.metal:13-81)
//   rope_qkv     RoPE non-traditional (rope.metal:55-229) + KVCacheSimple.update (KVCache.swift:452-470)
//   sdpa_decode  scaledDotProductAttention decode -> sdpa_vector(_2pass) (sdpa_vector.h:15-394)
//   silu_mul     compiledSwiGLU: silu(gate) * up (SwitchLayers.swift:40-50, Llama.swift:96-99)
//   add          residual h = x + f(x) in bf16
// All are HBM- or latency-bound; the attention kernel streams the bf16 cache
// with bulk copies (TMA engine) into shared memory and splits the cache over
// CTAs, writing fp32 partials (m, l, o) that a second kernel combines.
#include "kernels.cuh"
#include "sm100_util.cuh"

#include <mutex>

namespace vmlx {

// ---------------------------------------------------------------- RMSNorm --
// out = w * bf16(x * rsqrt(mean(x^2) + eps)), fp32 accumulation (rms_norm.metal:13-81).
__global__ void rms_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, bf16* __restrict__ out,
                                float eps, int dims) {
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * dims;
  bf16* orow = out + row * dims;
  float acc = 0.f;
  for (int i = threadIdx.x * 8; i < dims; i += blockDim.x * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
      acc = fmaf(f.x, f.x, acc);
      acc = fmaf(f.y, f.y, acc);
    }
  }
  __shared__ float part[32];
  __shared__ float inv_s;
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float a = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (threadIdx.x == 0) inv_s = rsqrtf(a / (float)dims + eps);
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x * 8; i < dims; i += blockDim.x * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(xr + i);
    uint4 ww = *reinterpret_cast<const uint4*>(w + i);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    const uint32_t wu[4] = {ww.x, ww.y, ww.z, ww.w};
    uint32_t o4[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
      bf162 n = __floats2bfloat162_rn(f.x * inv, f.y * inv);  // T(x * inv)
      float2 nf = __bfloat1622float2(n), wf = __bfloat1622float2(u32_as_bf162(wu[j]));
      o4[j] = bf162_as_u32(__floats2bfloat162_rn(wf.x * nf.x, wf.y * nf.y));
    }
    *reinterpret_cast<uint4*>(orow + i) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

// --------------------------------------------------- RoPE + KV-cache append --
// qkv [B, (Hq + 2*Hkv) * D] (q | k | v heads).  Rotates q and k at position
// `pos` (pairs (i, i + D/2), theta = pos * base^(-2i/D)), writes q_out
// [B, Hq, D] and k, v into the caches [B, Hkv, max_len, D] at `pos`.
__global__ void rope_qkv_kernel(const bf16* __restrict__ qkv, bf16* __restrict__ q_out, bf16* __restrict__ kc,
                                bf16* __restrict__ vc, int Hq, int Hkv, int D, int pos, int max_len,
                                float log2_base, float scale) {
  const int b = blockIdx.y;
  const int H = Hq + 2 * Hkv;
  const int half = D / 2;
  const int n_pairs = (Hq + Hkv) * half;
  const bf16* src = qkv + (int64_t)b * H * D;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_pairs + Hkv * D; i += gridDim.x * blockDim.x) {
    if (i < n_pairs) {
      const int h = i / half, d = i - h * half;
      const float inv_freq = exp2f(-((float)d / (float)half) * log2_base);
      const float theta = scale * (float)pos * inv_freq;
      float sn, cs;
      sincosf(theta, &sn, &cs);
      const float x1 = __bfloat162float(src[h * D + d]);
      const float x2 = __bfloat162float(src[h * D + d + half]);
      const bf16 o1 = __float2bfloat16_rn(x1 * cs - x2 * sn);
      const bf16 o2 = __float2bfloat16_rn(x1 * sn + x2 * cs);
      if (h < Hq) {
        bf16* dst = q_out + ((int64_t)b * Hq + h) * D;
        dst[d] = o1;
        dst[d + half] = o2;
      } else {
        bf16* dst = kc + (((int64_t)b * Hkv + (h - Hq)) * max_len + pos) * D;
        dst[d] = o1;
        dst[d + half] = o2;
      }
    } else {
      const int j = i - n_pairs;  // v element
      const int h = j / D, d = j - h * D;
      vc[(((int64_t)b * Hkv + h) * max_len + pos) * D + d] = src[(Hq + Hkv + h) * D + d];
    }
  }
}

// ------------------------------------------------------------ decode SDPA --
// One CTA per (cache split, kv head, batch); warp w serves q head kvh*G + w.
// The CTA streams its [chunk x D] slices of K and V with bulk copies into a
// double-buffered shared-memory ring.  Lane (p = lane/4, part = lane%4) owns
// dims [32*part, 32*part+32) of positions p, p+8, ...: a score is four lanes'
// partial dots joined by two shuffles, and each lane keeps an online softmax
// (m, l) and 32 output dims, merged across the 8 position lanes at the end.
// Partials (m, l, o[D]) of each (batch, q head, split) go to `part`; the
// combine kernel rescales and sums them (flash-decoding).
constexpr int SDPA_D = 128;
constexpr int SDPA_SUB = 32;  // positions per shared-memory stage

constexpr int SDPA_STAGES = 4;  // ring depth: 4 x (K + V) x 32 positions = 64 KB
constexpr size_t SDPA_SMEM = (size_t)SDPA_STAGES * 2 * SDPA_SUB * SDPA_D * sizeof(bf16) + 64;

__global__ void __launch_bounds__(256)
sdpa_decode_kernel(const bf16* __restrict__ q, const bf16* __restrict__ kc, const bf16* __restrict__ vc,
                   float* __restrict__ part, int Hq, int Hkv, int kv_len, int max_len, int chunk, float scale_log2) {
  extern __shared__ __align__(128) uint8_t sdpa_smem[];
  bf16* ring = reinterpret_cast<bf16*>(sdpa_smem);  // [stage][K|V][SUB][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(sdpa_smem + (size_t)SDPA_STAGES * 2 * SDPA_SUB * SDPA_D * sizeof(bf16));
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = lane >> 2, pt = lane & 3;
  const int hq = kvh * G + warp;
  const int t0 = split * chunk;
  const int t1 = min(kv_len, t0 + chunk);
  const int n_splits = gridDim.x;
  const bf16* kbase = kc + ((int64_t)b * Hkv + kvh) * max_len * SDPA_D;
  const bf16* vbase = vc + ((int64_t)b * Hkv + kvh) * max_len * SDPA_D;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SDPA_STAGES; s++) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // the cache and q may come from the previous kernel (launch overlap): wait for it
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int nsub = t1 > t0 ? (t1 - t0 + SDPA_SUB - 1) / SDPA_SUB : 0;
  auto kst = [&](int s) { return ring + ((size_t)(s % SDPA_STAGES) * 2 + 0) * SDPA_SUB * SDPA_D; };
  auto vst = [&](int s) { return ring + ((size_t)(s % SDPA_STAGES) * 2 + 1) * SDPA_SUB * SDPA_D; };
  auto issue = [&](int s) {
    const int a = t0 + s * SDPA_SUB;
    const int n = min(SDPA_SUB, t1 - a);
    const uint32_t bytes = (uint32_t)n * SDPA_D * 2;
    mbar_arrive_expect_tx(&full[s % SDPA_STAGES], 2 * bytes);
    bulk_g2s(kst(s), kbase + (int64_t)a * SDPA_D, bytes, &full[s % SDPA_STAGES]);
    bulk_g2s(vst(s), vbase + (int64_t)a * SDPA_D, bytes, &full[s % SDPA_STAGES]);
  };
  if (threadIdx.x == 0)
    for (int s = 0; s < nsub && s < SDPA_STAGES; s++) issue(s);

  float qf[32];
  if (warp < G) {
    const bf16* qr = q + ((int64_t)b * Hq + hq) * SDPA_D + pt * 32;
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      uint4 v = *reinterpret_cast<const uint4*>(qr + i);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
        qf[i + 2 * j] = f.x * scale_log2;
        qf[i + 2 * j + 1] = f.y * scale_log2;
      }
    }
  }
  float m = -INFINITY, l = 0.f, o[32];
#pragma unroll
  for (int i = 0; i < 32; i++) o[i] = 0.f;

  bool ok = true;
  for (int s = 0; s < nsub; s++) {
    ok &= mbar_wait(&full[s % SDPA_STAGES], (s / SDPA_STAGES) & 1);
    const int n = min(SDPA_SUB, t1 - (t0 + s * SDPA_SUB));
    if (warp < G) {
      const bf16* ks = kst(s);
      const bf16* vs = vst(s);
      for (int pp = p; pp < SDPA_SUB; pp += 8) {
        const bool valid = pp < n;
        float d = 0.f;
        if (valid) {
          const bf16* kr = ks + pp * SDPA_D + pt * 32;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v = *reinterpret_cast<const uint4*>(kr + i);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
              float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
              d = fmaf(qf[i + 2 * j], f.x, d);
              d = fmaf(qf[i + 2 * j + 1], f.y, d);
            }
          }
        }
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        if (valid) {  // online softmax in base 2 (scores carry log2(e) * scale)
          const float mn = fmaxf(m, d);
          const float corr = exp2f(m - mn);
          const float pw = exp2f(d - mn);
          l = l * corr + pw;
          const bf16* vr = vs + pp * SDPA_D + pt * 32;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v = *reinterpret_cast<const uint4*>(vr + i);
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
              float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
              o[i + 2 * j] = fmaf(o[i + 2 * j], corr, pw * f.x);
              o[i + 2 * j + 1] = fmaf(o[i + 2 * j + 1], corr, pw * f.y);
            }
          }
          m = mn;
        }
      }
    }
    __syncthreads();  // stage s is free: refill it with sub s + STAGES
    if (threadIdx.x == 0 && s + SDPA_STAGES < nsub) issue(s + SDPA_STAGES);
  }
  if (warp < G) {
    // merge the 8 position lanes that share `pt`
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
      const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
      const float mn = fmaxf(m, m2);
      const float c1 = (m == -INFINITY) ? 0.f : exp2f(m - mn);
      const float c2 = (m2 == -INFINITY) ? 0.f : exp2f(m2 - mn);
#pragma unroll
      for (int i = 0; i < 32; i++) {
        const float o2 = __shfl_xor_sync(0xffffffffu, o[i], off);
        o[i] = o[i] * c1 + o2 * c2;
      }
      l = l * c1 + l2 * c2;
      m = mn;
    }
    float* dst = part + (((int64_t)b * Hq + hq) * n_splits + split) * (SDPA_D + 2);
    if (p == 0) {
#pragma unroll
      for (int i = 0; i < 32; i++) dst[2 + pt * 32 + i] = o[i];
      if (pt == 0) {
        dst[0] = m;
        dst[1] = l;
      }
    }
  }
  (void)ok;
}

// out[b, hq, :] = sum_s exp2(m_s - M) o_s / sum_s exp2(m_s - M) l_s
__global__ void sdpa_combine_kernel(const float* __restrict__ part, bf16* __restrict__ out, int n_splits) {
  const int64_t bh = blockIdx.x;
  const float* src = part + bh * n_splits * (SDPA_D + 2);
  float M = -INFINITY;
  for (int s = 0; s < n_splits; s++) M = fmaxf(M, src[s * (SDPA_D + 2)]);
  const int d = threadIdx.x;
  float acc = 0.f, L = 0.f;
  for (int s = 0; s < n_splits; s++) {
    const float ms = src[s * (SDPA_D + 2)];
    const float c = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
    L += c * src[s * (SDPA_D + 2) + 1];
    acc += c * src[s * (SDPA_D + 2) + 2 + d];
  }
  out[bh * SDPA_D + d] = __float2bfloat16_rn(L > 0.f ? acc / L : 0.f);
}

// ----------------------------------------------------------- SwiGLU / add --
// out[r, j] = bf16(silu(g) * u) with g = bf16 silu of gate (compiledSwiGLU computes
// silu(gate) in the activation dtype, then multiplies).
__global__ void silu_mul_kernel(const bf16* __restrict__ gu, bf16* __restrict__ out, int64_t rows, int ffn) {
  const int64_t n = rows * ffn;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / ffn, j = i - r * ffn;
    const float g = __bfloat162float(gu[r * 2 * ffn + j]);
    const float u = __bfloat162float(gu[r * 2 * ffn + ffn + j]);
    const float s = __bfloat162float(__float2bfloat16_rn(g / (1.f + __expf(-g))));
    out[i] = __float2bfloat16_rn(s * u);
  }
}

__global__ void add_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b, bf16* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(__bfloat162float(a[i]) + __bfloat162float(b[i]));
}

}  // namespace vmlx

using namespace vmlx;

static unsigned grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  if (g > 148 * 16) g = 148 * 16;
  return (unsigned)(g < 1 ? 1 : g);
}

extern "C" int vmlx_cuda_rms_norm(void* out, const void* x, const void* weight, float eps, int64_t rows,
                                  int64_t dims, void* stream) {
  if (!out || !x || !weight) return set_error(VMLX_E_INVALID, "rms_norm: null pointer");
  if (dims <= 0 || dims % 8 || dims > 65536 || rows < 0)
    return set_error(VMLX_E_INVALID, "rms_norm: dims=%lld must be a positive multiple of 8", (long long)dims);
  if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(out, 16))
    return set_error(VMLX_E_INVALID, "rms_norm: pointers must be 16-byte aligned");
  if (rows == 0) return VMLX_OK;
  int threads = (int)(dims / 8 < 256 ? ((dims / 8 + 31) / 32) * 32 : 256);
  rms_norm_kernel<<<(unsigned)rows, threads, 0, as_stream(stream)>>>((const bf16*)x, (const bf16*)weight, (bf16*)out,
                                                                    eps, (int)dims);
  return check_launch("vmlx_cuda_rms_norm");
}

extern "C" int vmlx_cuda_rope_qkv(void* q_out, void* k_cache, void* v_cache, const void* qkv, int64_t batch,
                                  int n_heads, int n_kv_heads, int head_dim, int64_t pos, int64_t max_len,
                                  float base, float scale, void* stream) {
  if (!q_out || !k_cache || !v_cache || !qkv) return set_error(VMLX_E_INVALID, "rope_qkv: null pointer");
  if (head_dim <= 0 || head_dim % 2 || n_heads <= 0 || n_kv_heads <= 0 || pos < 0 || pos >= max_len)
    return set_error(VMLX_E_INVALID, "rope_qkv: bad shape (head_dim=%d pos=%lld max_len=%lld)", head_dim,
                     (long long)pos, (long long)max_len);
  if (batch == 0) return VMLX_OK;
  const int64_t work = (int64_t)(n_heads + n_kv_heads) * head_dim / 2 + (int64_t)n_kv_heads * head_dim;
  dim3 grid(grid_for(work, 256), (unsigned)batch);
  rope_qkv_kernel<<<grid, 256, 0, as_stream(stream)>>>((const bf16*)qkv, (bf16*)q_out, (bf16*)k_cache,
                                                        (bf16*)v_cache, n_heads, n_kv_heads, head_dim, (int)pos,
                                                        (int)max_len, log2f(base), scale);
  return check_launch("vmlx_cuda_rope_qkv");
}

static int sdpa_splits(int64_t kv_len) {
  int64_t s = (kv_len + 127) / 128;  // ~128 cache positions per CTA
  return (int)(s < 1 ? 1 : (s > 128 ? 128 : s));
}

static int sdpa_launch(const bf16* q, const bf16* kc, const bf16* vc, float* part, bf16* out, int64_t batch,
                       int n_heads, int n_kv_heads, int64_t kv_len, int64_t max_len, float scale, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    int rc = check_cuda(cudaFuncSetAttribute(sdpa_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)SDPA_SMEM), "sdpa_decode: cudaFuncSetAttribute");
    if (rc) return rc;
    attr = true;
  }
  const int splits = sdpa_splits(kv_len);
  const int chunk = (int)((kv_len + splits - 1) / splits);
  const int G = n_heads / n_kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)splits, (unsigned)n_kv_heads, (unsigned)batch);
  cfg.blockDim = dim3(32 * G);
  cfg.dynamicSmemBytes = SDPA_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  int rc = check_cuda(cudaLaunchKernelEx(&cfg, sdpa_decode_kernel, q, kc, vc, part, n_heads, n_kv_heads, (int)kv_len,
                                         (int)max_len, chunk, scale * 1.4426950408889634f),
                      "sdpa_decode_kernel launch");
  if (rc) return rc;
  sdpa_combine_kernel<<<(unsigned)(batch * n_heads), SDPA_D, 0, st>>>(part, out, splits);
  return check_launch("sdpa_combine_kernel");
}

extern "C" size_t vmlx_cuda_sdpa_decode_workspace(int64_t batch, int n_heads, int64_t kv_len, int head_dim) {
  return (size_t)batch * n_heads * sdpa_splits(kv_len) * (head_dim + 2) * sizeof(float);
}

extern "C" int vmlx_cuda_sdpa_decode(void* out, const void* q, const void* k_cache, const void* v_cache,
                                     int64_t batch, int n_heads, int n_kv_heads, int head_dim, int64_t kv_len,
                                     int64_t max_len, float scale, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  if (!out || !q || !k_cache || !v_cache || !workspace) return set_error(VMLX_E_INVALID, "sdpa_decode: null pointer");
  if (head_dim != SDPA_D) return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode: head_dim=%d (only 128)", head_dim);
  if (n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > 8)
    return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode: %d q heads per kv head (1..8 supported)",
                     n_kv_heads > 0 ? n_heads / n_kv_heads : 0);
  if (kv_len <= 0 || kv_len > max_len) return set_error(VMLX_E_INVALID, "sdpa_decode: kv_len=%lld", (long long)kv_len);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 16))
    return set_error(VMLX_E_INVALID, "sdpa_decode: pointers must be 16-byte aligned");
  const size_t need = vmlx_cuda_sdpa_decode_workspace(batch, n_heads, kv_len, head_dim);
  if (workspace_bytes < need)
    return set_error(VMLX_E_INVALID, "sdpa_decode: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if (batch == 0) return VMLX_OK;
  return sdpa_launch((const bf16*)q, (const bf16*)k_cache, (const bf16*)v_cache, (float*)workspace, (bf16*)out,
                     batch, n_heads, n_kv_heads, kv_len, max_len, scale, as_stream(stream));
}

extern "C" int vmlx_cuda_silu_mul(void* out, const void* gate_up, int64_t rows, int64_t ffn, void* stream) {
  if (!out || !gate_up) return set_error(VMLX_E_INVALID, "silu_mul: null pointer");
  if (rows < 0 || ffn <= 0) return set_error(VMLX_E_INVALID, "silu_mul: bad shape");
  if (rows == 0) return VMLX_OK;
  silu_mul_kernel<<<grid_for(rows * ffn, 256), 256, 0, as_stream(stream)>>>((const bf16*)gate_up, (bf16*)out, rows,
                                                                           (int)ffn);
  return check_launch("vmlx_cuda_silu_mul");
}

extern "C" int vmlx_cuda_add(void* out, const void* a, const void* b, int64_t n, void* stream) {
  if (!out || !a || !b) return set_error(VMLX_E_INVALID, "add: null pointer");
  if (n <= 0) return n == 0 ? VMLX_OK : set_error(VMLX_E_INVALID, "add: bad size");
  add_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>((const bf16*)a, (const bf16*)b, (bf16*)out, n);
  return check_launch("vmlx_cuda_add");
}

// ---------------------------------------------------------------------------
// Allocation-free decode attention.
//
// Some callers cannot allocate device memory at the point where they run
// attention: an engine that hands the library only the buffers it already owns
// (a fixed memory pool reserved at start-up, a plug-in host that forbids
// allocation on its inference thread, code that must not call cudaMalloc
// because that call can synchronise the device or fail under memory pressure
// mid-decode).  For them this entry point keeps the per-split partials in a
// fixed array that lives inside the library's device image, so the call needs
// nothing but its inputs and output.
//
// Limits and behaviour:
//  * the array holds SDPA_NOALLOC_BYTES (8 MiB) per GPU, for as long as the
//    process has the library loaded on that GPU; calls whose partials need
//    more (batch * n_heads * ceil(kv_len/128, at most 128) * (head_dim + 2) * 4
//    bytes) are rejected with VMLX_E_INVALID;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture;
//  * every call on a device shares the one array: calls that can overlap on
//    the GPU (different streams without ordering) race and must not be issued;
//  * each call writes every partial it later reads, so nothing needs clearing
//    and stale contents of an earlier call are never used.
// ---------------------------------------------------------------------------
constexpr size_t SDPA_NOALLOC_BYTES = (size_t)8 << 20;
static __device__ __align__(256) float g_sdpa_noalloc_scratch[SDPA_NOALLOC_BYTES / sizeof(float)];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {};

// Device address of the scratch array on the current device (set up once per device).
static int noalloc_scratch(void** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "sdpa_decode_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return set_error(VMLX_E_INVALID, "sdpa_decode_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_sdpa_noalloc_scratch), "sdpa_decode_noalloc: cudaGetSymbolAddress");
    if (rc) return rc;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return VMLX_OK;
}

extern "C" int vmlx_cuda_sdpa_decode_noalloc(void* out, const void* q, const void* k_cache, const void* v_cache,
                                             int64_t batch, int n_heads, int n_kv_heads, int head_dim, int64_t kv_len,
                                             int64_t max_len, float scale, void* stream) {
  if (!out || !q || !k_cache || !v_cache) return set_error(VMLX_E_INVALID, "sdpa_decode_noalloc: null pointer");
  if (head_dim != SDPA_D)
    return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode_noalloc: head_dim=%d (only 128)", head_dim);
  if (n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > 8)
    return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode_noalloc: %d q heads per kv head (1..8 supported)",
                     n_kv_heads > 0 ? n_heads / n_kv_heads : 0);
  if (kv_len <= 0 || kv_len > max_len || batch < 0)
    return set_error(VMLX_E_INVALID, "sdpa_decode_noalloc: kv_len=%lld", (long long)kv_len);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 16))
    return set_error(VMLX_E_INVALID, "sdpa_decode_noalloc: pointers must be 16-byte aligned");
  const size_t need = vmlx_cuda_sdpa_decode_workspace(batch, n_heads, kv_len, head_dim);
  if (need > SDPA_NOALLOC_BYTES)
    return set_error(VMLX_E_INVALID,
                     "sdpa_decode_noalloc: these sizes need %zu bytes of partials, more than the %zu-byte "
                     "built-in scratch; use vmlx_cuda_sdpa_decode with a workspace",
                     need, SDPA_NOALLOC_BYTES);
  if (batch == 0) return VMLX_OK;
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return sdpa_launch((const bf16*)q, (const bf16*)k_cache, (const bf16*)v_cache, (float*)scratch, (bf16*)out,
                     batch, n_heads, n_kv_heads, kv_len, max_len, scale, as_stream(stream));
}
