// qgemv.cu -- decode GEMV for 1..4 token rows (4/8-bit MLX affine weights).
//
// Computes y[t, n] = sum_k x[t, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g]) for the
// single-token decode regime of MLX's affine_qmv_fast / affine_qmv
// (Source/Cmlx/mlx-generated/metal/quantized.h:799-1025), with the decoder-block
// fusions of the other GEMV kernel (RMSNorm of x on load, SwiGLU of a gate||up x on
// load, residual add on store).
//
// B200 design.  At 0.5625 B per 4-bit weight the op is a pure HBM stream; the kernel
// keeps bytes in flight on every SM for the whole call and spends few instructions per
// weight:
//  * Persistent CTAs (as many as are resident), each looping over row tiles of 16*S
//    rows.  Every warp streams its own weights: lane 0 keeps QG_STAGES TMA loads
//    (cp.async.bulk.tensor.2d, 16 rows x 128 bytes, 128-byte swizzle, no multicast) in
//    flight into a warp-private shared-memory ring, each completing on its own
//    mbarrier, and the ring runs ahead across tile boundaries -- no producer warp, no
//    cross-warp handshake, no refill gap between tiles.
//  * A tile's 16*S rows are split over the CTA's 8 warps as S strips x (8/S) group
//    ranges; a thread-block cluster of C CTAs splits K further.  Partial tiles are
//    added in a fixed order (warps through shared memory, cluster CTAs through
//    distributed shared memory): deterministic, no atomics, no global scratch.
//  * The next tile's bf16 scales and biases are copied into shared memory with
//    cp.async while the current tile is computed (double buffer, padded rows so the
//    8 rows a warp reads at once fall in different banks).
//  * The dot products run on mma.sync.m16n8k16 in fp16 with fp32 accumulation:
//    A = the 16 rows' codes as exact fp16 values 1024+q (4-bit odd nibbles 1024+16q),
//    built with one prmt and four lop3 per 8 codes; B = x in the matching k order,
//    tokens as the MMA's N dimension.  x is staged once per CTA, each token scaled by a
//    power of two 2^s (max |x| 2^s < 2^15, so fp16 holds every bf16 value exactly) and
//    the odd-nibble positions by a further 2^-4; per group the fold is
//    scale * (sum(x' code) - 1024 sum(x')) * 2^-s + bias * sum(x), the factorisation of
//    MLX's qdot (quantized.h:209-316).  Power-of-two scaling commutes with rounding, so
//    the result does not depend on s.
// The CTA geometry depends on (N, K, bits, group size) only, never on M, so a row's
// result is the same whether it is computed alone or with up to 3 other rows (batch
// invariance, QuantizedSmallMScalingBenchTests.swift:110-127).
#include "kernels.cuh"
#include "sm100_util.cuh"
#include "qmv_util.cuh"
#include "tmap.cuh"

#include <cuda_fp16.h>

#include <algorithm>

namespace vmlx {

namespace cg = cooperative_groups;

constexpr int QG_WARPS = 8;
constexpr int QG_THREADS = 32 * QG_WARPS;
constexpr int QG_MAXM = 4;        // token rows of this regime
constexpr int QG_MAX_CLUSTER = 8;
constexpr int QG_TOKP = 8;        // token slots of an MMA tile (N dimension)
constexpr int QG_STAGES = 3;      // ring stages per warp
constexpr int QG_STAGE_BYTES = 16 * 128;  // one stage: 16 rows x 128 bytes

template <int BITS, int GS>
struct QGT {
  static constexpr int LB = GS * BITS / 32;          // bytes per lane per row per group
  static constexpr int WL = LB / 4;                  // 32-bit words per lane per row per group
  static constexpr int GB = GS * BITS / 8;           // bytes per row per group
  static constexpr int GC = 128 / GB;                // groups per ring stage
};

struct QgGeom {
  int S;         // 16-row strips per tile
  int C;         // CTAs per cluster (K split)
  int KGC;       // groups per CTA
  int GW;        // groups per warp (a whole number of ring stages)
  int xstr;      // bytes per staged x row
  int sbrow;     // bytes per staged scale (or bias) row: 16-byte multiple + 16 of padding
  int ntiles;    // row tiles of 16*S rows
  int sc_async;  // scales/biases rows are 16-byte aligned: cp.async them
};

struct QgSmem {
  size_t o_ring, o_bar, o_xs, o_xsum, o_sc, o_red, o_ctile, total;
  __host__ __device__ void init(const QgGeom& g, int m) {
    o_ring = 0;  // 1024-byte aligned (the swizzle atom)
    o_bar = o_ring + (size_t)QG_WARPS * QG_STAGES * QG_STAGE_BYTES;
    o_xs = o_bar + (size_t)QG_WARPS * QG_STAGES * 8;
    o_xsum = o_xs + (size_t)m * g.xstr;
    o_sc = o_xsum + (size_t)2 * g.KGC * QG_TOKP * 4;
    o_red = o_sc + (size_t)2 * 2 * 16 * g.S * g.sbrow;  // [buffer][scale | bias][row]
    o_ctile = o_red + (size_t)QG_WARPS * 16 * QG_TOKP * 4;
    total = o_ctile + (g.C > 1 ? (size_t)16 * g.S * QG_TOKP * 4 : 0) + 1024;  // + alignment slack
  }
};

// Byte offset of (row r in 0..15, byte o) in a 128-byte-swizzled [16][128] stage:
// 16-byte chunk j of row r sits at chunk j ^ (r & 7).
__device__ __forceinline__ int swz(int r, int o) { return r * 128 + ((((o >> 4) ^ (r & 7))) << 4) + (o & 15); }

template <int LB>
__device__ __forceinline__ void lds_lane(const uint8_t* a, uint32_t (&w)[LB / 4]) {
  if constexpr (LB == 4) {
    w[0] = *reinterpret_cast<const uint32_t*>(a);
  } else if constexpr (LB == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(a);
    w[0] = v.x; w[1] = v.y;
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(a);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  }
}

// 4-bit word -> four fp16 pairs, exact: p[0] = (n0, n4) + 1024, p[1] = 16 (n1, n5) + 1024,
// p[2] = (n2, n6) + 1024, p[3] = 16 (n3, n7) + 1024 (under the fp16 exponent byte 0x64
// the low 10 bits are an integer mantissa, so a nibble masked at bits 0-3 or 4-7 of a
// half reads as itself or 16x itself).  One prmt and four lop3 per 8 codes.
__device__ __forceinline__ void unpack4h(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t E = 0x64006400u;
  const uint32_t w2 = prmt(w, 0u, 0x3311);  // bytes (b1, b1, b3, b3)
  p[0] = (w & 0x000F000Fu) | E;
  p[1] = (w & 0x00F000F0u) | E;
  p[2] = (w2 & 0x000F000Fu) | E;
  p[3] = (w2 & 0x00F000F0u) | E;
}

// 8-bit word (4 codes) -> (q0, q1) + 1024, (q2, q3) + 1024: the code byte becomes the
// low mantissa byte under an 0x64 exponent byte.
__device__ __forceinline__ void unpack8h(uint32_t w, uint32_t (&p)[2]) {
  p[0] = prmt(w, 0x64646464u, 0x4140);
  p[1] = prmt(w, 0x64646464u, 0x4342);
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Scales and biases of the tile at row0 (the CTA's groups cg0..cg0+ncg) into buffer
// `dst` ([scale | bias][16*S rows][sbrow bytes]).  Asynchronous (cp.async; one commit
// group per call, empty when !valid) when rows are 16-byte aligned, else plain loads.
__device__ __forceinline__ void qg_load_scales(const QmvArgs& p, const QgGeom& g, uint8_t* dst, int64_t row0,
                                               int64_t KG, int64_t cg0, int ncg, bool valid, int tid) {
  const int rows = 16 * g.S;
  if (valid) {
    if (g.sc_async) {
      const int nchunk = (ncg + 7) >> 3;  // 8 groups per 16-byte chunk (KGC is a multiple of 8)
      for (int i = tid; i < 2 * rows * nchunk; i += QG_THREADS) {
        const int kind = i / (rows * nchunk), rem = i - kind * rows * nchunk;
        const int r = rem / nchunk, ch = rem - r * nchunk;
        const int64_t row = row0 + r < p.N ? row0 + r : p.N - 1;
        const bf16* src = (kind ? p.biases : p.scales) + row * KG + cg0 + ch * 8;
        cp_async16(dst + ((size_t)kind * rows + r) * g.sbrow + ch * 16, src);
      }
    } else {
      for (int i = tid; i < 2 * rows * ncg; i += QG_THREADS) {
        const int kind = i / (rows * ncg), rem = i - kind * rows * ncg;
        const int r = rem / ncg, gl = rem - r * ncg;
        const int64_t row = row0 + r < p.N ? row0 + r : p.N - 1;
        reinterpret_cast<bf16*>(dst + ((size_t)kind * rows + r) * g.sbrow)[gl] =
            (kind ? p.biases : p.scales)[row * KG + cg0 + gl];
      }
    }
  }
  cp_async_commit();
}

#ifdef QG_X_TRACE
__device__ unsigned long long qg_trace[8];
extern "C" int vmlx_qg_trace(unsigned long long* out, int reset) {
  cudaMemcpyFromSymbol(out, qg_trace, sizeof(qg_trace));
  if (reset) { unsigned long long z[8] = {0, 0, 0, 0, 0, ~0ull, 0, 0}; cudaMemcpyToSymbol(qg_trace, z, sizeof(z)); }
  return 0;
}
#endif
template <int BITS, int GS>
__global__ void __launch_bounds__(QG_THREADS, 3)
qgemv_kernel(QmvArgs p, QgGeom g, const __grid_constant__ CUtensorMap tmw) {
  using T = QGT<BITS, GS>;
  constexpr int LB = T::LB, WL = T::WL, GB = T::GB, GC = T::GC;
  constexpr int BPG = GS / 8;  // 8-value x blocks per group
  constexpr int NH = (LB + 15) / 16, LBH = LB < 16 ? LB : 16;  // 16-byte pieces of a lane's slice
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  __shared__ float xinv[QG_MAXM];    // fused RMSNorm: 1 / rms per token
  __shared__ uint32_t smax[QG_MAXM];  // max |x| per token (float bits)
  __shared__ float xscale[QG_MAXM];   // 2^-s per token

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, c = lane & 3;
  const int S = g.S, C = g.C;
  const int M = (int)p.M;
  const int crank = C > 1 ? (int)(blockIdx.x % C) : 0;
  const int64_t cluster_id = blockIdx.x / C, nclusters = gridDim.x / C;
  const int64_t KG = p.K / GS;
  const int64_t cg0 = (int64_t)crank * g.KGC;
  const int ncg = (int)(KG - cg0 < g.KGC ? (KG - cg0 > 0 ? KG - cg0 : 0) : g.KGC);
  const int s = warp % S, ksub = warp / S;
  const int wg0 = ksub * g.GW;
  const int nwg = ncg - wg0 < g.GW ? (ncg - wg0 > 0 ? ncg - wg0 : 0) : g.GW;
  const int nch = (nwg + GC - 1) / GC;  // ring stages per tile for this warp
  const int64_t ntl = cluster_id < g.ntiles ? (g.ntiles - 1 - cluster_id) / nclusters + 1 : 0;
  const int total_st = (int)(ntl * nch);
  const int rows = 16 * S;

  QgSmem L;
  L.init(g, M);
  uint8_t* xs = smem + L.o_xs;
  float* xsumb = reinterpret_cast<float*>(smem + L.o_xsum);  // [g][t] sum of x
  float* xsumq = xsumb + (size_t)g.KGC * QG_TOKP;              // [g][t] 1024 * sum of staged x
  float* red = reinterpret_cast<float*>(smem + L.o_red);
  float* ctile = reinterpret_cast<float*>(smem + L.o_ctile);
  uint8_t* ring = smem + L.o_ring + (size_t)warp * QG_STAGES * QG_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.o_bar) + warp * QG_STAGES;
  const size_t scbuf = (size_t)2 * rows * g.sbrow;

  // Weights and scales are static: start streaming them before waiting on the
  // previous kernel (programmatic dependent launch), and let the next kernel launch.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#ifdef QG_X_TRACE
  const uint64_t t_start = globaltimer();
#endif
  if (lane == 0) {
    for (int d = 0; d < QG_STAGES; d++) mbar_init(&bars[d], 1);
    fence_mbar_init();
  }
  __syncwarp();
  // stage j of this warp: tile j / nch, group range (j % nch) * GC of the warp's range
  // The next stage to load: tile iss_row (first row of the warp's strip in it) and group
  // column iss_x; advanced incrementally (lane 0 only), no divisions on the issue path.
  int iss_jj = 0, iss_row = (int)(cluster_id * rows + s * 16);
  const int row_step = (int)(nclusters * rows);
  const int x0 = (int)((cg0 + wg0) * GB);
  auto issue = [&](int st) {
    mbar_arrive_expect_tx(&bars[st], QG_STAGE_BYTES);
    tma_load_2d(ring + st * QG_STAGE_BYTES, &tmw, x0 + iss_jj * (GC * GB), iss_row, &bars[st]);
    if (++iss_jj == nch) {
      iss_jj = 0;
      iss_row += row_step;
    }
  };
  if (lane == 0) {
    tma_prefetch_desc(&tmw);
    for (int j = 0; j < total_st && j < QG_STAGES; j++) issue(j);
  }
  qg_load_scales(p, g, smem + L.o_sc, cluster_id * rows, KG, cg0, ncg, ntl > 0, tid);
  qg_load_scales(p, g, smem + L.o_sc + scbuf, (cluster_id + nclusters) * rows, KG, cg0, ncg, ntl > 1, tid);

  if (tid < QG_MAXM) smax[tid] = 0u;
  // x may be written by the previous kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __syncthreads();
  if (p.norm_w) {
    // fused RMSNorm: 1 / rms over each token's full row (the order of the other GEMV kernel)
    for (int t = warp; t < M; t += QG_WARPS) {
      const bf16* xr = p.x + (int64_t)t * p.K;
      float ss = 0.f;
#pragma unroll 4
      for (int64_t k = lane * 8; k < p.K; k += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const uint32_t u4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 f = __bfloat1622float2(u32_as_bf162(u4[j]));
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
      for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) xinv[t] = rsqrtf(ss / (float)p.K + p.eps);
    }
    __syncthreads();
  }
  // Stage x in two passes.  Pass 1: load (with the optional SwiGLU / RMSNorm), keep the
  // bf16 values, the per-group sums X[g][t] (fp32) and each token's max |x| over the
  // CTA's K range.  Pass 2: scale each token by a power of two 2^s_t (max |x| 2^s_t <
  // 2^15, exact) into fp16 -- for 4-bit, the positions of odd nibbles get 2^(s_t - 4),
  // which matches the 16x-scaled codes the unpack produces -- permute to the unpack's
  // order, and record Q[g][t] = 1024 * sum of the staged values (the codes carry a +1024
  // offset).  The scale only moves exponents, so results do not depend on it.
  {
    const int nkb = ncg * BPG;
    const int total = M * nkb;
    const int64_t xrs = p.x_swiglu ? 2 * p.K : p.K;
    float tmax[QG_MAXM] = {0.f, 0.f, 0.f, 0.f};
    // 4 blocks per thread per pass, all loads issued before any is used
    for (int base = 0; base < total; base += 4 * QG_THREADS) {
      uint4 v[4], u[4];
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i = base + b * QG_THREADS + tid;
        v[b] = u[b] = make_uint4(0, 0, 0, 0);
        if (i < total) {
          const int t = i / nkb, kb = i - t * nkb;
          const bf16* xr = p.x + t * xrs + cg0 * GS + (int64_t)kb * 8;
          v[b] = *reinterpret_cast<const uint4*>(xr);
          if (p.x_swiglu) u[b] = *reinterpret_cast<const uint4*>(xr + p.K);
        }
      }
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i = base + b * QG_THREADS + tid;
        float sum = 0.f;
        int t = 0, kb = 0;
        if (i < total) {
          t = i / nkb;
          kb = i - t * nkb;
          const int64_t k = cg0 * GS + (int64_t)kb * 8;
          uint4 x8 = v[b];
          if (p.x_swiglu)
            x8 = make_uint4(swiglu2(x8.x, u[b].x), swiglu2(x8.y, u[b].y), swiglu2(x8.z, u[b].z),
                            swiglu2(x8.w, u[b].w));
          if (p.norm_w) x8 = norm8(x8, xinv[t], p.norm_w + k);
          const float2 a = __bfloat1622float2(u32_as_bf162(x8.x)), b2 = __bfloat1622float2(u32_as_bf162(x8.y));
          const float2 c2 = __bfloat1622float2(u32_as_bf162(x8.z)), d2 = __bfloat1622float2(u32_as_bf162(x8.w));
          sum = ((a.x + a.y) + (b2.x + b2.y)) + ((c2.x + c2.y) + (d2.x + d2.y));
          const float mx = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b2.x), fabsf(b2.y))),
                                 fmaxf(fmaxf(fabsf(c2.x), fabsf(c2.y)), fmaxf(fabsf(d2.x), fabsf(d2.y))));
#pragma unroll
          for (int q = 0; q < QG_MAXM; q++)
            if (q == t) tmax[q] = fmaxf(tmax[q], mx);
          *reinterpret_cast<uint4*>(xs + (size_t)t * g.xstr + (size_t)kb * 16) = x8;
        }
#pragma unroll
        for (int o = 1; o < BPG; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (i < total && (kb % BPG) == 0) xsumb[(kb / BPG) * QG_TOKP + t] = sum;
      }
    }
#pragma unroll
    for (int q = 0; q < QG_MAXM; q++) {
      float m = tmax[q];
      for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0 && q < M && m > 0.f) atomicMax(&smax[q], __float_as_uint(m));
    }
    for (int i = tid; i < ncg * (QG_TOKP - M); i += QG_THREADS) {
      const int gl = i / (QG_TOKP - M), t = M + (i - gl * (QG_TOKP - M));
      xsumb[gl * QG_TOKP + t] = 0.f;
      xsumq[gl * QG_TOKP + t] = 0.f;
    }
    __syncthreads();
    for (int base = 0; base < total; base += QG_THREADS) {
      const int i = base + tid;
      float sum = 0.f;
      int t = 0, kb = 0;
      if (i < total) {
        t = i / nkb;
        kb = i - t * nkb;
        // 2^s with max |x| 2^s < 2^15 (fp16 max 65504)
        const uint32_t mb = smax[t];
        const int e = mb ? (int)((mb >> 23) & 0xFF) - 127 : 0;
        int sh = 14 - e;
        sh = sh > 100 ? 100 : (sh < -100 ? -100 : sh);
        const float f0 = ldexpf(1.f, sh), f1 = BITS == 4 ? ldexpf(1.f, sh - 4) : f0;
        uint4* px = reinterpret_cast<uint4*>(xs + (size_t)t * g.xstr + (size_t)kb * 16);
        const uint4 x8 = *px;
        float2 v0 = __bfloat1622float2(u32_as_bf162(x8.x)), v1 = __bfloat1622float2(u32_as_bf162(x8.y));
        float2 v2 = __bfloat1622float2(u32_as_bf162(x8.z)), v3 = __bfloat1622float2(u32_as_bf162(x8.w));
        float2 h0, h1, h2, h3;  // fp16 pairs in MMA operand order
        if constexpr (BITS == 4) {
          // (x0,x4)*f0, (x1,x5)*f1, (x2,x6)*f0, (x3,x7)*f1
          h0 = make_float2(v0.x * f0, v2.x * f0);
          h1 = make_float2(v0.y * f1, v2.y * f1);
          h2 = make_float2(v1.x * f0, v3.x * f0);
          h3 = make_float2(v1.y * f1, v3.y * f1);
        } else {
          h0 = make_float2(v0.x * f0, v0.y * f0);
          h1 = make_float2(v1.x * f0, v1.y * f0);
          h2 = make_float2(v2.x * f0, v2.y * f0);
          h3 = make_float2(v3.x * f0, v3.y * f0);
        }
        const __half2 q0 = __float22half2_rn(h0), q1 = __float22half2_rn(h1);
        const __half2 q2 = __float22half2_rn(h2), q3 = __float22half2_rn(h3);
        const float2 r0 = __half22float2(q0), r1 = __half22float2(q1);
        const float2 r2 = __half22float2(q2), r3 = __half22float2(q3);
        sum = ((r0.x + r0.y) + (r1.x + r1.y)) + ((r2.x + r2.y) + (r3.x + r3.y));
        uint4 o;
        o.x = *reinterpret_cast<const uint32_t*>(&q0);
        o.y = *reinterpret_cast<const uint32_t*>(&q1);
        o.z = *reinterpret_cast<const uint32_t*>(&q2);
        o.w = *reinterpret_cast<const uint32_t*>(&q3);
        *px = o;
        if (kb == 0) xscale[t] = ldexpf(1.f, -sh);
      }
#pragma unroll
      for (int o = 1; o < BPG; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (i < total && (kb % BPG) == 0) xsumq[(kb / BPG) * QG_TOKP + t] = 1024.f * sum;
    }
  }
  __syncthreads();

#ifdef QG_X_TRACE
  if (lane == 0) atomicAdd(&qg_trace[6], globaltimer() - t_start);
#endif
  // ---- stream the warp's stages, tile after tile ----
  const bool tv = gq < M;
  const uint8_t* xlane = xs + (size_t)(tv ? gq : 0) * g.xstr + (size_t)c * (GS / 4) * 2;
  int off0[GC][NH], off1[GC][NH];  // lane-constant swizzled offsets of rows gq, gq + 8
#pragma unroll
  for (int gi = 0; gi < GC; gi++)
#pragma unroll
    for (int h = 0; h < NH; h++) {
      off0[gi][h] = swz(gq, gi * GB + c * LB + 16 * h);
      off1[gi][h] = swz(gq + 8, gi * GB + c * LB + 16 * h);
    }
  const float e0 = 2 * c < M ? xscale[2 * c] : 0.f, e1 = 2 * c + 1 < M ? xscale[2 * c + 1] : 0.f;
  bool ok = true;
  int j = 0, st = 0;
  uint32_t phase = 0;
  for (int64_t ti = 0; ti < ntl; ti++) {
    const int64_t row0 = (cluster_id + ti * nclusters) * rows;
    uint8_t* scb = smem + L.o_sc + (size_t)(ti & 1) * scbuf;
    cp_async_wait1();  // this tile's scales (all but the newest copy group)
    __syncthreads();   // ... visible to every thread; the previous tile's reduction is done
    const bf16* sc0 = reinterpret_cast<const bf16*>(scb + (size_t)(s * 16 + gq) * g.sbrow);
    const bf16* sc1 = reinterpret_cast<const bf16*>(scb + (size_t)(s * 16 + gq + 8) * g.sbrow);
    const bf16* bi0 = reinterpret_cast<const bf16*>(scb + (size_t)(rows + s * 16 + gq) * g.sbrow);
    const bf16* bi1 = reinterpret_cast<const bf16*>(scb + (size_t)(rows + s * 16 + gq + 8) * g.sbrow);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};   // scale * (sum(x' code) - Q), x' domain
    float accb[4] = {0.f, 0.f, 0.f, 0.f};  // bias * X
    for (int jj = 0; jj < nch; jj++, j++) {  // j: this warp's stage counter

#ifdef QG_X_TRACE
      const uint64_t t_a = globaltimer();
#endif
      ok &= mbar_wait(&bars[st], phase);
#ifdef QG_X_TRACE
      const uint64_t t_b = globaltimer();
      if (lane == 0) { atomicAdd(&qg_trace[0], t_b - t_a); atomicAdd(&qg_trace[1], 1ull); }
#endif
      const uint8_t* stg = ring + st * QG_STAGE_BYTES;
#pragma unroll
      for (int gi = 0; gi < GC; gi++) {
        if (jj * GC + gi < nwg) {
          const int gl = wg0 + jj * GC + gi;
          uint32_t w0[WL], w1[WL];
#pragma unroll
          for (int h = 0; h < NH; h++) {
            lds_lane<LBH>(stg + off0[gi][h], *reinterpret_cast<uint32_t(*)[LBH / 4]>(w0 + h * 4));
            lds_lane<LBH>(stg + off1[gi][h], *reinterpret_cast<uint32_t(*)[LBH / 4]>(w1 + h * 4));
          }
          float ag[4] = {0.f, 0.f, 0.f, 0.f};
          const uint8_t* xp = xlane + (size_t)gl * GS * 2;
          if constexpr (BITS == 4) {
#pragma unroll
            for (int wi = 0; wi < WL; wi++) {
              uint32_t pa[4], pb[4];
              unpack4h(w0[wi], pa);
              unpack4h(w1[wi], pb);
              uint4 xv = make_uint4(0, 0, 0, 0);
              if (tv) xv = *reinterpret_cast<const uint4*>(xp + wi * 16);
              const uint32_t a0[4] = {pa[0], pb[0], pa[1], pb[1]};
              const uint32_t a1[4] = {pa[2], pb[2], pa[3], pb[3]};
              mma_f16_16816(ag, a0, xv.x, xv.y);
              mma_f16_16816(ag, a1, xv.z, xv.w);
            }
          } else {
#pragma unroll
            for (int wi = 0; wi < WL; wi++) {
              uint32_t pa[2], pb[2];
              unpack8h(w0[wi], pa);
              unpack8h(w1[wi], pb);
              uint2 xv = make_uint2(0, 0);
              if (tv) xv = *reinterpret_cast<const uint2*>(xp + wi * 8);
              const uint32_t a[4] = {pa[0], pb[0], pa[1], pb[1]};
              mma_f16_16816(ag, a, xv.x, xv.y);
            }
          }
          const float s0 = __bfloat162float(sc0[gl]), s1 = __bfloat162float(sc1[gl]);
          const float b0 = __bfloat162float(bi0[gl]), b1 = __bfloat162float(bi1[gl]);
          const float2 xq = *reinterpret_cast<const float2*>(xsumq + gl * QG_TOKP + 2 * c);
          const float2 xb = *reinterpret_cast<const float2*>(xsumb + gl * QG_TOKP + 2 * c);
          acc[0] = fmaf(s0, ag[0] - xq.x, acc[0]);
          acc[1] = fmaf(s0, ag[1] - xq.y, acc[1]);
          acc[2] = fmaf(s1, ag[2] - xq.x, acc[2]);
          acc[3] = fmaf(s1, ag[3] - xq.y, acc[3]);
          accb[0] = fmaf(b0, xb.x, accb[0]);
          accb[1] = fmaf(b0, xb.y, accb[1]);
          accb[2] = fmaf(b1, xb.x, accb[2]);
          accb[3] = fmaf(b1, xb.y, accb[3]);
        }
      }
      // refill this stage once every lane has read it (generic reads before the async write)
      __syncwarp();
      if (lane == 0 && j + QG_STAGES < total_st) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(st);
      }
      if (++st == QG_STAGES) {
        st = 0;
        phase ^= 1u;
      }
    }

    // ---- fixed-order reduction: warps of the CTA, then the CTAs of the cluster ----
    // back from the x' domain (y = 2^-s acc + accb): (row gq / gq+8, tokens 2c, 2c+1)
    {
      float* rw = red + (size_t)warp * 16 * QG_TOKP;
      *reinterpret_cast<float2*>(rw + gq * QG_TOKP + 2 * c) =
          make_float2(fmaf(acc[0], e0, accb[0]), fmaf(acc[1], e1, accb[1]));
      *reinterpret_cast<float2*>(rw + (gq + 8) * QG_TOKP + 2 * c) =
          make_float2(fmaf(acc[2], e0, accb[2]), fmaf(acc[3], e1, accb[3]));
    }
    __syncthreads();
    // the buffer of this tile's scales is free: start copying the scales two tiles ahead
    qg_load_scales(p, g, scb, (cluster_id + (ti + 2) * nclusters) * rows, KG, cg0, ncg, ti + 2 < ntl, tid);
    const int KSPLIT = QG_WARPS / S;
    for (int i = tid; i < rows * M; i += QG_THREADS) {
      const int r = i / M, t = i - r * M;
      const int ss_ = r >> 4, rr = r & 15;
      float v = 0.f;
      for (int q = 0; q < KSPLIT; q++) v += red[((size_t)(q * S + ss_) * 16 + rr) * QG_TOKP + t];
      if (C == 1) {
        const int64_t n = row0 + r;
        if (n < p.N) {
          const int64_t idx = (int64_t)t * p.N + n;
          if (p.residual) {
            const float sv = __bfloat162float(__float2bfloat16_rn(v));
            p.y[idx] = __float2bfloat16_rn(__bfloat162float(p.residual[idx]) + sv);
          } else {
            p.y[idx] = __float2bfloat16_rn(v);
          }
        }
      } else {
        ctile[r * QG_TOKP + t] = v;
      }
    }
    if (C > 1) {
      cluster_arrive();
      cluster_wait();
      cg::cluster_group cluster = cg::this_cluster();
      const int rlo = crank * rows / C, rhi = (crank + 1) * rows / C;
      for (int i = tid; i < (rhi - rlo) * M; i += QG_THREADS) {
        const int r = rlo + i / M, t = i % M;
        float v = 0.f;
        for (int q = 0; q < C; q++) v += cluster.map_shared_rank(ctile, q)[r * QG_TOKP + t];
        const int64_t n = row0 + r;
        if (n < p.N) {
          const int64_t idx = (int64_t)t * p.N + n;
          if (p.residual) {
            const float sv = __bfloat162float(__float2bfloat16_rn(v));
            p.y[idx] = __float2bfloat16_rn(__bfloat162float(p.residual[idx]) + sv);
          } else {
            p.y[idx] = __float2bfloat16_rn(v);
          }
        }
      }
      cluster_arrive();  // peers have read this CTA's tile before it is overwritten or freed
      cluster_wait();
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
#ifdef QG_X_TRACE
  if (lane == 0) { atomicAdd(&qg_trace[2], globaltimer() - t_start); atomicAdd(&qg_trace[3], 1ull); }
  if (tid == 0) atomicMax(&qg_trace[4], globaltimer());
  if (tid == 0) atomicMin(&qg_trace[5], t_start);
#endif
  if (!ok && p.status) atomicExch(p.status, VMLX_E_STATE);
}

// ---- host side -------------------------------------------------------------

static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

static int qg_per_sm(const QgSmem& L) {
  int per = (int)((228 * 1024) / (L.total + 1024));
  return per > 3 ? 3 : per;  // 80 registers x 256 threads: 3 CTAs per SM
}

static void qg_fill(QgGeom& gm, int64_t N, int64_t K, int gs, int S, int C) {
  const int64_t KG = K / gs;
  gm.S = S;
  gm.C = C;
  int KGC = (int)((KG + C - 1) / C);
  KGC = (KGC + 7) / 8 * 8;  // whole 16-byte scale chunks per CTA
  gm.KGC = KGC;
  gm.xstr = KGC * gs * 2 + 16;
  gm.sbrow = KGC * 2 + 16;
  gm.ntiles = (int)((N + 16 * S - 1) / (16 * S));
}

// Geometry from (N, K, bits, group size) only.  The busiest CTA's work (tiles x ring
// stages per warp, plus a fixed cost per tile and per cluster reduction) against the
// bandwidth share of the resident CTAs; shared memory is sized for the regime's largest
// M so that the geometry never depends on M.
static bool qg_choose(int64_t N, int64_t K, int bits, int gs, QgGeom& best) {
  const int64_t KG = K / gs;
  const int GC = 128 / (gs * bits / 8);
  const int sms = sm_count();
  const int forceS = env_int("VMLX_QG_S", 0), forceC = env_int("VMLX_QG_C", 0);
  double best_cost = 1e30;
  bool found = false;
  for (int C = 1; C <= QG_MAX_CLUSTER; C++) {
    if (forceC && C != forceC) continue;
    if (C > 1 && (int64_t)(C - 1) * (((KG + C - 1) / C + 7) / 8 * 8) >= KG) continue;  // an empty CTA
    for (int S = 1; S <= QG_WARPS; S *= 2) {
      if (forceS && S != forceS) continue;
      QgGeom gm;
      qg_fill(gm, N, K, gs, S, C);
      const int KSPLIT = QG_WARPS / S;
      gm.GW = ((gm.KGC + KSPLIT - 1) / KSPLIT + GC - 1) / GC * GC;
      if (KSPLIT > 1 && (int64_t)(KSPLIT - 1) * gm.GW >= gm.KGC && !forceS) continue;  // an idle warp
      QgSmem L;
      L.init(gm, QG_MAXM);
      if (L.total > 200 * 1024) continue;
      const int per_sm = qg_per_sm(L);
      if (per_sm < 1) continue;
      const int64_t nclu = std::min<int64_t>(gm.ntiles, (int64_t)sms * per_sm / C);
      if (nclu < 1) continue;
      const int64_t tiles_per = (gm.ntiles + nclu - 1) / nclu;
      const double stages = (double)tiles_per * (gm.GW / GC);           // per warp, serial
      const double bw = (double)(N / 16) * KG / GC / ((double)sms * 24);  // stages per warp slot if BW-bound
      const double cost = std::max(stages, bw) + 1.5 * tiles_per + (C > 1 ? 2.0 * tiles_per : 0.0);
      if (cost < best_cost) {
        best_cost = cost;
        best = gm;
        found = true;
      }
    }
  }
  return found;
}

template <int BITS, int GS>
static int launch_qg(const QmvArgs& a, cudaStream_t st) {
  QgGeom g;
  if (!qg_choose(a.N, a.K, BITS, GS, g))
    return set_error(VMLX_E_UNSUPPORTED, "qgemv: no launch geometry for N=%lld K=%lld", (long long)a.N,
                     (long long)a.K);
  g.sc_async = (a.K / GS) % 8 == 0 && aligned(a.scales, 16) && aligned(a.biases, 16);
  QgSmem L;
  L.init(g, (int)a.M);
  auto kern = qgemv_kernel<BITS, GS>;
  {
    const int rc = ensure_max_dynamic_smem((const void*)kern, 220 * 1024);
    if (rc) return rc;
  }
  QgSmem Lmax;
  Lmax.init(g, QG_MAXM);
  const int64_t nclu = std::min<int64_t>(g.ntiles, (int64_t)sm_count() * qg_per_sm(Lmax) / g.C);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nclu * g.C), 1, 1);
  cfg.blockDim = dim3(QG_THREADS);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = (unsigned)g.C;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  na++;
  if (launch_overlap()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  CUtensorMap tmw;
  const uint64_t rowb = (uint64_t)a.K * BITS / 8;
  if (!make_tmap_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, rowb, (uint64_t)a.N, rowb, 128, 16,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return VMLX_E_CUDA;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, a, g, tmw), "qgemv_kernel launch");
}

bool qgemv_covers(const QmvArgs& a, int mode, int bits, int gs) {
  if (mode != QMV_DENSE || a.tp_world > 1) return false;
  if (a.M < 1 || a.M > QG_MAXM) return false;
  if (a.K % 8 || a.N >= (1LL << 31)) return false;
  if (!aligned(a.x, 16) || (a.norm_w && !aligned(a.norm_w, 16))) return false;
  if (!env_int("VMLX_QG", 0) || env_int("VMLX_QG_DISABLE", 0)) return false;
  (void)bits;
  (void)gs;
  return true;
}

int launch_qgemv(const QmvArgs& a, int bits, int gs, cudaStream_t st) {
  if (bits == 4 && gs == 32) return launch_qg<4, 32>(a, st);
  if (bits == 4 && gs == 64) return launch_qg<4, 64>(a, st);
  if (bits == 4 && gs == 128) return launch_qg<4, 128>(a, st);
  if (bits == 8 && gs == 32) return launch_qg<8, 32>(a, st);
  if (bits == 8 && gs == 64) return launch_qg<8, 64>(a, st);
  if (bits == 8 && gs == 128) return launch_qg<8, 128>(a, st);
  return set_error(VMLX_E_UNSUPPORTED, "matmul: bits=%d group_size=%d not supported", bits, gs);
}

}  // namespace vmlx
