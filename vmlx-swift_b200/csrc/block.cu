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
#include "tmap.cuh"
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
// One CTA per (cache split of 128 or 256 positions, kv head, sequence), 4 or 8 warps:
// warp w takes the split's 32-position stage w.  K and V arrive as 2-D TMA boxes
// [32 positions x 64 dims] with the 128-byte swizzle (the whole split is in
// flight at once).  The math runs on the tensor cores (mma.sync m16n8k16, bf16
// in, fp32 accumulate): the G q heads of the kv head are the rows of
// S = Q K^T (K fragments read straight from the swizzled tiles, bank-conflict
// free), the softmax of the stage stays in registers, and P (bf16) is the A
// operand of O = P V (V fragments by ldmatrix.trans).  The warps' (m, l, O) are
// merged through shared memory into the split's partial; the last CTA of each
// (sequence, kv head) to finish -- a counter in the workspace, reset by that CTA
// -- combines the splits (flash-decoding) and writes the output.
constexpr int SDPA_D = 128;
constexpr int SDPA_SUB = 32;     // positions per stage (one warp each)
// Stages per split (a template parameter of the kernel): 8 (256 positions, 128 KB of K/V in
// flight, one CTA per SM) while the grid is small, 4 (128 positions, 64 KB, 2-3 CTAs per SM)
// once it covers the SMs twice over, where more resident warps per SM hide the latencies.
constexpr int SDPA_MAX_STAGES = 8;
constexpr int SDPA_MIN_CHUNK = SDPA_SUB * 4;  // the smallest split: workspaces are sized for it
template <int ST> struct SdpaCfg {
  static constexpr int STAGES = ST;
  static constexpr int CHUNK = SDPA_SUB * ST;  // positions per split
  static constexpr int THREADS = 32 * ST;
  static constexpr size_t RING = (size_t)ST * 2 * SDPA_SUB * SDPA_D * sizeof(bf16);
  static constexpr size_t SMEM = RING + 64 + 1024;  // + alignment slack
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <int ST>
__global__ void __launch_bounds__(SdpaCfg<ST>::THREADS)
sdpa_decode_kernel(const bf16* __restrict__ q, const __grid_constant__ CUtensorMap tmk,
                   const __grid_constant__ CUtensorMap tmv, float* __restrict__ part, unsigned* __restrict__ counters,
                   bf16* __restrict__ out, int Hq, int Hkv, int kv_len, int max_len, float scale_log2,
                   const int32_t* __restrict__ kv_dev, int kv_add) {
  constexpr int SDPA_STAGES = SdpaCfg<ST>::STAGES, SDPA_CHUNK = SdpaCfg<ST>::CHUNK, SDPA_THREADS = SdpaCfg<ST>::THREADS;
  constexpr size_t SDPA_RING = SdpaCfg<ST>::RING;
  extern __shared__ __align__(1024) uint8_t sdpa_smem_raw[];
  uint8_t* sdpa_smem = sdpa_smem_raw + ((1024 - (smem_u32(sdpa_smem_raw) & 1023)) & 1023);
  uint8_t* ring = sdpa_smem;  // [stage][K|V][2 boxes][32 positions][128 B], 128-byte swizzle
  uint64_t* full = reinterpret_cast<uint64_t*>(sdpa_smem + SDPA_RING);
  float* mrg = reinterpret_cast<float*>(sdpa_smem);  // [warp][head][D + 2], reuses the ring after the math
  __shared__ int s_last;
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;  // MMA fragment coordinates: head row g, column pair c
  const int row0 = ((int)b * Hkv + kvh) * max_len;  // this head's first cache row in the [rows, D] maps

  if (threadIdx.x == 0) {
    for (int s = 0; s < SDPA_STAGES; s++) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // the cache and q may come from the previous kernel (launch overlap): wait for it
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // a cache length held in device memory (one graph for every decode step): the grid covers
  // the longest cache, and splits past this call's length leave before touching anything
  if (kv_dev) {
    kv_len = kv_dev[0] + kv_add;
    if (kv_len < 1 || kv_len > max_len) return;
  }
  const int n_splits = (kv_len + SDPA_CHUNK - 1) / SDPA_CHUNK;
  if (split >= n_splits) return;
  const int t0 = split * SDPA_CHUNK;
  const int t1 = min(kv_len, t0 + SDPA_CHUNK);

  const int nsub = t1 > t0 ? (t1 - t0 + SDPA_SUB - 1) / SDPA_SUB : 0;  // <= SDPA_STAGES
  auto kst = [&](int s) { return ring + ((size_t)s * 2 + 0) * SDPA_SUB * SDPA_D * 2; };
  auto vst = [&](int s) { return ring + ((size_t)s * 2 + 1) * SDPA_SUB * SDPA_D * 2; };
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
    for (int s = 0; s < nsub; s++) {
      // two [32 x 64] boxes per matrix (dims 0-63, 64-127); rows past the cache read as zeros
      const int row = row0 + t0 + s * SDPA_SUB;
      mbar_arrive_expect_tx(&full[s], 4 * SDPA_SUB * 128);
      tma_load_2d(kst(s), &tmk, 0, row, &full[s]);
      tma_load_2d(kst(s) + SDPA_SUB * 128, &tmk, 64, row, &full[s]);
      tma_load_2d(vst(s), &tmv, 0, row, &full[s]);
      tma_load_2d(vst(s) + SDPA_SUB * 128, &tmv, 64, row, &full[s]);
    }
  }
  // byte offset of (position r, dim d) in a swizzled [32 x 128] stage tile (two [32 x 64] boxes)
  auto tile_off = [](int r, int d) {
    return (uint32_t)((d >> 6) * (SDPA_SUB * 128) + r * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) + (d & 7) * 2);
  };

  // Q as the A operand: rows = the G heads (rows >= G and g + 8 are zero), k = dims
  const bool hv = g < G;
  const bf16* qr = q + ((int64_t)b * Hq + kvh * G + (hv ? g : 0)) * SDPA_D;
  uint32_t qa0[8], qa2[8];
#pragma unroll
  for (int ks = 0; ks < 8; ks++) {
    qa0[ks] = hv ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 2 * c) : 0u;
    qa2[ks] = hv ? *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 2 * c + 8) : 0u;
  }
  float m = -INFINITY, l = 0.f;
  float o[16][4];
#pragma unroll
  for (int nd = 0; nd < 16; nd++) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;

  const int s = warp;
  if (s < nsub) {
    mbar_wait(&full[s], 0);
    const int n = min(SDPA_SUB, t1 - (t0 + s * SDPA_SUB));
    const uint8_t* kt = kst(s);
    const uint32_t vt = smem_u32(vst(s));
    // S = Q K^T: 4 n-tiles of 8 positions x 8 k-steps of 16 dims
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
      const uint32_t a[4] = {qa0[ks], 0u, qa2[ks], 0u};
#pragma unroll
      for (int nt = 0; nt < 4; nt++) {
        const int r = nt * 8 + g;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kt + tile_off(r, 16 * ks + 2 * c));
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kt + tile_off(r, 16 * ks + 2 * c + 8));
        mma_bf16_16816(sc[nt], a, b0, b1);
      }
    }
    // softmax of the stage in base 2: lane holds positions nt*8 + 2c (+1) of head g
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; nt++)
#pragma unroll
      for (int j = 0; j < 2; j++) {
        const float v = (nt * 8 + 2 * c + j < n) ? sc[nt][j] * scale_log2 : -INFINITY;
        sc[nt][j] = v;
        mx = fmaxf(mx, v);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    m = mx;
    // P = P_hi + P_lo, both bf16 (P_lo = the rounding residue), so the tensor-core P V keeps
    // ~16 bits of each probability, as close to the reference's fp32 as the sums need
    uint32_t pa[2][4], pl[2][4];
#pragma unroll
    for (int nt = 0; nt < 4; nt++) {
      const float p0 = exp2f(sc[nt][0] - m), p1 = exp2f(sc[nt][1] - m);
      l += p0 + p1;
      const bf162 hi = __floats2bfloat162_rn(p0, p1);
      const float2 hf = __bfloat1622float2(hi);
      const uint32_t pk = bf162_as_u32(hi), pr = bf162_as_u32(__floats2bfloat162_rn(p0 - hf.x, p1 - hf.y));
      // A fragment of P for k-step nt/2: positions 16*ks2 + 2c (a0) and + 8 (a2); rows g + 8 are zero
      if (nt & 1) { pa[nt >> 1][2] = pk; pl[nt >> 1][2] = pr; } else { pa[nt >> 1][0] = pk; pl[nt >> 1][0] = pr; }
    }
    pa[0][1] = pa[0][3] = pa[1][1] = pa[1][3] = 0u;
    pl[0][1] = pl[0][3] = pl[1][1] = pl[1][3] = 0u;
    // O = P V: 2 k-steps of 16 positions x 16 n-tiles of 8 dims; V fragments by ldmatrix.trans
    // (lanes 0-7 / 8-15 / 16-23 / 24-31 address rows 0-7 / 8-15 of dims nd*8 and nd*8 + 8)
#pragma unroll
    for (int ks2 = 0; ks2 < 2; ks2++) {
      const int r = 16 * ks2 + (lane & 15);
#pragma unroll
      for (int nd = 0; nd < 16; nd += 2) {
        const int d = (nd + (lane >> 4)) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(vt + tile_off(r, d), b0, b1, b2, b3);
        mma_bf16_16816(o[nd], pa[ks2], b0, b1);
        mma_bf16_16816(o[nd + 1], pa[ks2], b2, b3);
        mma_bf16_16816(o[nd], pl[ks2], b0, b1);
        mma_bf16_16816(o[nd + 1], pl[ks2], b2, b3);
      }
    }
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  // the next kernel may start streaming its own inputs while this grid finishes
  asm volatile("griddepcontrol.launch_dependents;");
  __syncthreads();  // every stage consumed: the ring becomes the merge buffer
  if (hv) {
    float* w = mrg + ((size_t)warp * G + g) * (SDPA_D + 2);
#pragma unroll
    for (int nd = 0; nd < 16; nd++) {
      w[2 + nd * 8 + 2 * c] = o[nd][0];
      w[2 + nd * 8 + 2 * c + 1] = o[nd][1];
    }
    if (c == 0) {
      w[0] = m;
      w[1] = l;
    }
  }
  __syncthreads();
  // merge the warps (stages), write this split's partial (m, l, o[D])
  for (int t = threadIdx.x; t < G * SDPA_D; t += SDPA_THREADS) {
    const int gg = t / SDPA_D, dd = t % SDPA_D;
    float mm = -INFINITY;
    for (int s2 = 0; s2 < SDPA_STAGES; s2++) mm = fmaxf(mm, mrg[((size_t)s2 * G + gg) * (SDPA_D + 2)]);
    float ll = 0.f, oo = 0.f;
    for (int s2 = 0; s2 < SDPA_STAGES; s2++) {
      const float* w = mrg + ((size_t)s2 * G + gg) * (SDPA_D + 2);
      const float cw = (w[0] == -INFINITY) ? 0.f : exp2f(w[0] - mm);
      ll += cw * w[1];
      oo += cw * w[2 + dd];
    }
    float* dst = part + (((int64_t)b * Hq + kvh * G + gg) * n_splits + split) * (SDPA_D + 2);
    dst[2 + dd] = oo;
    if (dd == 0) {
      dst[0] = mm;
      dst[1] = ll;
    }
  }
  // last split of this (sequence, kv head) to finish combines: out = sum c_s o_s / sum c_s l_s
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* cnt = counters + (int64_t)b * Hkv + kvh;
    s_last = atomicAdd(cnt, 1u) == (unsigned)(n_splits - 1);
    if (s_last) *cnt = 0u;  // ready for the next call
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // per (head, split): m and l loaded in one parallel pass into shared memory (the ring is
  // free), weights c = exp2(m - M_head) and L = sum c*l per head, then every thread sums c*o
  // for four output dims at once (independent loads in flight)
  float* cw = mrg;                   // [G][n_splits] m, then weights
  float* lw = mrg + G * n_splits;    // [G][n_splits] l
  float* lsum = lw + G * n_splits;   // [G]
  const int64_t bh0 = (int64_t)b * Hq + kvh * G;
  const float* src0 = part + bh0 * n_splits * (SDPA_D + 2);
  for (int t = threadIdx.x; t < G * n_splits; t += SDPA_THREADS) {
    cw[t] = __ldcg(src0 + (int64_t)t * (SDPA_D + 2));
    lw[t] = __ldcg(src0 + (int64_t)t * (SDPA_D + 2) + 1);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int gg = threadIdx.x;
    float M = -INFINITY;
    for (int s2 = 0; s2 < n_splits; s2++) M = fmaxf(M, cw[gg * n_splits + s2]);
    float L = 0.f;
    for (int s2 = 0; s2 < n_splits; s2++) {
      const float ms = cw[gg * n_splits + s2];
      const float c = (ms == -INFINITY) ? 0.f : exp2f(ms - M);
      cw[gg * n_splits + s2] = c;
      L += c * lw[gg * n_splits + s2];
    }
    lsum[gg] = L;
  }
  __syncthreads();
  // thread t sums dims t, t + 128/... of one head: 4 outputs per pass
  for (int t0 = threadIdx.x; t0 < G * SDPA_D; t0 += 4 * SDPA_THREADS) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const float* src[4];
    const float* cws[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int t = min(t0 + j * SDPA_THREADS, G * SDPA_D - 1);
      const int gg = t / SDPA_D, dd = t % SDPA_D;
      src[j] = src0 + (int64_t)gg * n_splits * (SDPA_D + 2) + 2 + dd;
      cws[j] = cw + gg * n_splits;
    }
#pragma unroll 4
    for (int s2 = 0; s2 < n_splits; s2++) {
#pragma unroll
      for (int j = 0; j < 4; j++) acc[j] = fmaf(cws[j][s2], __ldcg(src[j] + (int64_t)s2 * (SDPA_D + 2)), acc[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int t = t0 + j * SDPA_THREADS;
      if (t < G * SDPA_D) {
        const int gg = t / SDPA_D, dd = t % SDPA_D;
        const float L = lsum[gg];
        out[(bh0 + gg) * SDPA_D + dd] = __float2bfloat16_rn(L > 0.f ? acc[j] / L : 0.f);
      }
    }
  }
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

// out[r, c] = bf16(y[r, c] + bias[c]): the bias of a QuantizedLinear (Quantized.swift:361-376).
__global__ void bias_add_kernel(const bf16* __restrict__ y, const bf16* __restrict__ bias, bf16* __restrict__ out,
                                int64_t n, int64_t cols) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16_rn(__bfloat162float(y[i]) + __bfloat162float(bias[i % cols]));
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

static int sdpa_splits(int64_t kv_len, int chunk = SDPA_MIN_CHUNK) {
  const int64_t s = (kv_len + chunk - 1) / chunk;  // chunk cache positions per CTA
  return (int)(s < 1 ? 1 : s);
}

// Workspace: one split counter per (sequence, head) first -- at a fixed place, so that calls
// with a growing kv_len find them zero -- then the per-split partials.
static size_t sdpa_cnt_bytes(int64_t batch, int n_heads) {
  return ((size_t)batch * n_heads * sizeof(unsigned) + 255) / 256 * 256;
}
static size_t sdpa_part_bytes(int64_t batch, int n_heads, int64_t kv_len) {
  return (size_t)batch * n_heads * sdpa_splits(kv_len) * (SDPA_D + 2) * sizeof(float);
}
static size_t sdpa_ws_bytes(int64_t batch, int n_heads, int64_t kv_len) {
  return sdpa_cnt_bytes(batch, n_heads) + sdpa_part_bytes(batch, n_heads, kv_len);
}

template <int ST>
static int sdpa_launch_st(const bf16* q, const bf16* kc, const bf16* vc, unsigned* counters, float* part, bf16* out,
                          int64_t batch, int n_heads, int n_kv_heads, int64_t kv_len, int64_t max_len, float scale,
                          cudaStream_t st, const int32_t* kv_dev, int kv_add) {
  using C = SdpaCfg<ST>;
  auto kern = sdpa_decode_kernel<ST>;
  {
    const int rc = ensure_max_dynamic_smem((const void*)kern, (int)C::SMEM);
    if (rc) return rc;
  }
  const int splits = sdpa_splits(kv_len, C::CHUNK);
  // the combining CTA keeps m and l per (head, split) in the ring
  if (splits > 65535 || (size_t)(2 * splits + 1) * (n_heads / n_kv_heads) * sizeof(float) > C::RING)
    return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode: kv_len=%lld too long", (long long)kv_len);
  const int64_t rows = batch * n_kv_heads * max_len;
  if (rows >= (1LL << 31)) return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode: cache of %lld rows", (long long)rows);
  CUtensorMap tmk, tmv;
  if (!make_tmap_2d(&tmk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kc, SDPA_D, (uint64_t)rows, SDPA_D * 2, 64, SDPA_SUB,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, vc, SDPA_D, (uint64_t)rows, SDPA_D * 2, 64, SDPA_SUB,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return VMLX_E_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)splits, (unsigned)n_kv_heads, (unsigned)batch);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, q, tmk, tmv, part, counters, out, n_heads, n_kv_heads,
                                       (int)kv_len, (int)max_len, scale * 1.4426950408889634f, kv_dev, kv_add),
                    "sdpa_decode_kernel launch");
}

// Split size from the grid it gives (never from the data): 256-position splits while they give
// fewer than two CTAs per SM, 128-position splits (smaller CTAs, 2-3 per SM) beyond.
static int sdpa_launch(const bf16* q, const bf16* kc, const bf16* vc, unsigned* counters, float* part, bf16* out,
                       int64_t batch, int n_heads, int n_kv_heads, int64_t kv_len, int64_t max_len, float scale,
                       cudaStream_t st, const int32_t* kv_dev = nullptr, int kv_add = 0) {
  const int64_t ctas8 = (int64_t)sdpa_splits(kv_len, SdpaCfg<8>::CHUNK) * n_kv_heads * batch;
  if (ctas8 < 2 * (int64_t)sm_count())
    return sdpa_launch_st<8>(q, kc, vc, counters, part, out, batch, n_heads, n_kv_heads, kv_len, max_len, scale, st,
                             kv_dev, kv_add);
  return sdpa_launch_st<4>(q, kc, vc, counters, part, out, batch, n_heads, n_kv_heads, kv_len, max_len, scale, st,
                           kv_dev, kv_add);
}


extern "C" size_t vmlx_cuda_sdpa_decode_workspace(int64_t batch, int n_heads, int64_t kv_len, int head_dim) {
  (void)head_dim;
  return sdpa_ws_bytes(batch, n_heads, kv_len);
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
  return sdpa_launch((const bf16*)q, (const bf16*)k_cache, (const bf16*)v_cache, static_cast<unsigned*>(workspace),
                     reinterpret_cast<float*>(static_cast<char*>(workspace) + sdpa_cnt_bytes(batch, n_heads)),
                     (bf16*)out, batch, n_heads, n_kv_heads, kv_len, max_len, scale, as_stream(stream));
}

// Decode attention with the cache length read from device memory: kv_len = *pos_dev + 1 (the
// token at position *pos_dev was just appended).  The grid and the workspace cover max_len,
// so one captured graph serves every step of a token loop.
extern "C" int vmlx_cuda_sdpa_decode_at(void* out, const void* q, const void* k_cache, const void* v_cache,
                                        int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                        const int32_t* pos_dev, int64_t max_len, float scale, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (!out || !q || !k_cache || !v_cache || !workspace || !pos_dev)
    return set_error(VMLX_E_INVALID, "sdpa_decode_at: null pointer");
  if (head_dim != SDPA_D) return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode_at: head_dim=%d (only 128)", head_dim);
  if (n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > 8)
    return set_error(VMLX_E_UNSUPPORTED, "sdpa_decode_at: %d q heads per kv head (1..8 supported)",
                     n_kv_heads > 0 ? n_heads / n_kv_heads : 0);
  if (max_len <= 0) return set_error(VMLX_E_INVALID, "sdpa_decode_at: max_len=%lld", (long long)max_len);
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 16))
    return set_error(VMLX_E_INVALID, "sdpa_decode_at: pointers must be 16-byte aligned");
  const size_t need = vmlx_cuda_sdpa_decode_workspace(batch, n_heads, max_len, head_dim);
  if (workspace_bytes < need)
    return set_error(VMLX_E_INVALID, "sdpa_decode_at: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if (batch == 0) return VMLX_OK;
  return sdpa_launch((const bf16*)q, (const bf16*)k_cache, (const bf16*)v_cache, static_cast<unsigned*>(workspace),
                     reinterpret_cast<float*>(static_cast<char*>(workspace) + sdpa_cnt_bytes(batch, n_heads)),
                     (bf16*)out, batch, n_heads, n_kv_heads, max_len, max_len, scale, as_stream(stream), pos_dev, 1);
}

extern "C" int vmlx_cuda_silu_mul(void* out, const void* gate_up, int64_t rows, int64_t ffn, void* stream) {
  if (!out || !gate_up) return set_error(VMLX_E_INVALID, "silu_mul: null pointer");
  if (rows < 0 || ffn <= 0) return set_error(VMLX_E_INVALID, "silu_mul: bad shape");
  if (rows == 0) return VMLX_OK;
  silu_mul_kernel<<<grid_for(rows * ffn, 256), 256, 0, as_stream(stream)>>>((const bf16*)gate_up, (bf16*)out, rows,
                                                                           (int)ffn);
  return check_launch("vmlx_cuda_silu_mul");
}

extern "C" int vmlx_cuda_bias_add(void* out, const void* y, const void* bias, int64_t rows, int64_t cols,
                                  void* stream) {
  if (!out || !y || !bias) return set_error(VMLX_E_INVALID, "bias_add: null pointer");
  if (rows < 0 || cols <= 0) return set_error(VMLX_E_INVALID, "bias_add: bad shape");
  if (rows == 0) return VMLX_OK;
  bias_add_kernel<<<grid_for(rows * cols, 256), 256, 0, as_stream(stream)>>>((const bf16*)y, (const bf16*)bias,
                                                                            (bf16*)out, rows * cols, cols);
  return check_launch("vmlx_cuda_bias_add");
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
//    process has the library loaded on that GPU: 64 KiB of split counters
//    (zero when the library loads; every call leaves them zero) and the
//    partials; calls whose partials need more (batch * n_heads *
//    ceil(kv_len/256) * (head_dim + 2) * 4 bytes) than the rest are rejected
//    with VMLX_E_INVALID;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture;
//  * every call on a device shares the one array: calls that can overlap on
//    the GPU (different streams without ordering) race and must not be issued;
//  * each call writes every partial it later reads, so stale partials of an
//    earlier call are never used.
// ---------------------------------------------------------------------------
constexpr size_t SDPA_NOALLOC_BYTES = (size_t)8 << 20;
constexpr size_t SDPA_NOALLOC_CNT_BYTES = (size_t)64 << 10;  // split counters (zero at load; calls leave them zero)
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
  const size_t need = sdpa_part_bytes(batch, n_heads, kv_len);
  if (need > SDPA_NOALLOC_BYTES - SDPA_NOALLOC_CNT_BYTES || (size_t)batch * n_heads * 4 > SDPA_NOALLOC_CNT_BYTES)
    return set_error(VMLX_E_INVALID,
                     "sdpa_decode_noalloc: these sizes need %zu bytes of partials, more than the %zu-byte "
                     "built-in scratch; use vmlx_cuda_sdpa_decode with a workspace",
                     need, SDPA_NOALLOC_BYTES - SDPA_NOALLOC_CNT_BYTES);
  if (batch == 0) return VMLX_OK;
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return sdpa_launch((const bf16*)q, (const bf16*)k_cache, (const bf16*)v_cache, static_cast<unsigned*>(scratch),
                     reinterpret_cast<float*>(static_cast<char*>(scratch) + SDPA_NOALLOC_CNT_BYTES), (bf16*)out,
                     batch, n_heads, n_kv_heads, kv_len, max_len, scale, as_stream(stream));
}
