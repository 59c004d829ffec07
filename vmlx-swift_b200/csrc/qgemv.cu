// qgemv.cu -- decode GEMV for 1..4 token rows (4/8-bit MLX affine weights).
//
// Computes y[t, n] = sum_k x[t, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g]) for the
// single-token decode regime of MLX's affine_qmv_fast / affine_qmv
// (Source/Cmlx/mlx-generated/metal/quantized.h:799-1025), with the decoder-block
// fusions of the other GEMV kernel (RMSNorm of x on load, SwiGLU of a gate||up x on
// load, residual add on store).
//
// B200 design.  At 0.5625 B per 4-bit weight the op is a pure HBM stream, so the
// kernel is organised around keeping many bytes in flight on every SM with as few
// instructions per weight as possible:
//  * Every warp streams its own weights: lane 0 keeps QG_STAGES TMA loads
//    (cp.async.bulk.tensor.2d, 16 rows x 128 bytes, 128-byte swizzle, no multicast)
//    in flight into a warp-private shared-memory ring, each completing on its own
//    mbarrier.  The bytes in flight per SM are set by the ring, not by registers
//    (3 stages x 2 KB x 24 warps), which is what an HBM stream with microsecond
//    latency needs; there is no producer warp and no cross-warp handshake.
//  * A warp owns a 16-row strip and a contiguous range of groups; the CTA's 8 warps
//    are S strips x (8/S) group ranges; a thread-block cluster of C CTAs splits K
//    further.  Partial tiles are added in a fixed order (warps through shared memory,
//    cluster CTAs through distributed shared memory): deterministic, no atomics, no
//    global scratch.
//  * The dot products run on mma.sync.m16n8k16: A = the 16 rows' codes as exact bf16
//    128+q (one shift and one lop3 per two 4-bit codes, no rounding), B = x in the
//    matching k order, tokens as the MMA's N dimension.  Per group the fold is
//    scale*sum(x*(128+q)) + (bias - 128*scale)*sum(x), the factorisation of MLX's qdot
//    (quantized.h:209-316); the per-group sums of x are computed once per CTA.
//  * x (after the optional RMSNorm / SwiGLU) is staged once per CTA in shared memory,
//    permuted inside each 8-value block to the order the unpack produces codes in.
// The CTA geometry depends on (N, K, bits, group size) only, never on M, so a row's
// result is the same whether it is computed alone or with up to 3 other rows (batch
// invariance, QuantizedSmallMScalingBenchTests.swift:110-127).
#include "kernels.cuh"
#include "sm100_util.cuh"
#include "qmv_util.cuh"
#include "tmap.cuh"

#include <cuda_fp16.h>

namespace vmlx {

namespace cg = cooperative_groups;

constexpr int QG_WARPS = 8;
constexpr int QG_THREADS = 32 * QG_WARPS;
constexpr int QG_MAXM = 4;        // token rows of this regime
constexpr int QG_MAX_CLUSTER = 8;
constexpr int QG_TOKP = 8;        // token slots of an MMA tile (N dimension)
constexpr int QG_STAGES = 3;      // default ring stages per warp
constexpr int QG_STAGE_BYTES = 16 * 128;  // one stage: 16 rows x 128 bytes

template <int BITS, int GS>
struct QGT {
  static constexpr int LB = GS * BITS / 32;          // bytes per lane per row per group
  static constexpr int WL = LB / 4;                  // 32-bit words per lane per row per group
  static constexpr int GB = GS * BITS / 8;           // bytes per row per group
  static constexpr int GC = 128 / GB;                // groups per ring stage
};

struct QgGeom {
  int S;      // 16-row strips per CTA
  int C;      // CTAs per cluster (K split)
  int KGC;    // groups per CTA
  int GW;     // groups per warp
  int xstr;   // bytes per staged x row
  int sbstr;  // 32-bit words per staged (scale, bias) row
  int sc_vec;  // scales/biases rows load as 16-byte vectors
  int D;       // ring stages per warp
  int dbg;
};

struct QgSmem {
  size_t o_ring, o_bar, o_xs, o_xsum, o_sb, o_red, o_ctile, total;
  __host__ __device__ void init(const QgGeom& g, int m) {
    o_ring = 0;  // 1024-byte aligned (the swizzle atom)
    o_bar = o_ring + (size_t)QG_WARPS * g.D * QG_STAGE_BYTES;
    o_xs = o_bar + (size_t)QG_WARPS * g.D * 8;
    o_xsum = o_xs + (size_t)m * g.xstr;
    o_sb = o_xsum + (size_t)2 * g.KGC * QG_TOKP * 4;
    o_red = o_sb + (size_t)16 * g.S * g.sbstr * 4;
    o_ctile = o_red + (size_t)QG_WARPS * 16 * QG_TOKP * 4;
    total = o_ctile + (g.C > 1 ? (size_t)16 * g.S * QG_TOKP * 4 : 0) + 1024;  // + alignment slack
  }
};

// LB bytes of row r (0..15) at byte o of a 128-byte-swizzled [16][128] stage:
// 16-byte chunk j of row r sits at chunk j ^ (r & 7).
template <int LB>
__device__ __forceinline__ void lds_lane(const uint8_t* stg, int r, int o, uint32_t (&w)[LB / 4]) {
#pragma unroll
  for (int h = 0; h < (LB + 15) / 16; h++) {
    const int oo = o + 16 * h;
    const uint8_t* a = stg + r * 128 + ((((oo >> 4) ^ (r & 7))) << 4) + (oo & 15);
    if constexpr (LB == 4) {
      w[0] = *reinterpret_cast<const uint32_t*>(a);
    } else if constexpr (LB == 8) {
      const uint2 v = *reinterpret_cast<const uint2*>(a);
      w[0] = v.x; w[1] = v.y;
    } else {
      const uint4 v = *reinterpret_cast<const uint4*>(a);
      w[4 * h] = v.x; w[4 * h + 1] = v.y; w[4 * h + 2] = v.z; w[4 * h + 3] = v.w;
    }
  }
}

// 4-bit word -> four fp16 pairs, exact: p[0] = (n0, n4) + 1024, p[1] = 16 (n1, n5) + 1024,
// p[2] = (n2, n6) + 1024, p[3] = 16 (n3, n7) + 1024 (the fp16 exponent 0x64 makes the
// low 10 bits integer mantissa, so a masked nibble at bits 0-3 or 4-7 of each half is
// read as itself or 16x itself).  Four lop3 and one prmt per 8 codes, no shifts.
__device__ __forceinline__ void unpack4h(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t E = 0x64006400u;
  const uint32_t w2 = prmt(w, 0u, 0x3311);  // bytes (b1, b1, b3, b3)
  p[0] = (w & 0x000F000Fu) | E;
  p[1] = (w & 0x00F000F0u) | E;
  p[2] = (w2 & 0x000F000Fu) | E;
  p[3] = (w2 & 0x00F000F0u) | E;
}

// 8-bit word (4 codes) -> two fp16 pairs (q0, q1) + 1024, (q2, q3) + 1024: the code byte
// becomes the low mantissa byte under an 0x64 exponent byte.
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

template <int BITS, int GS>
__global__ void __launch_bounds__(QG_THREADS, 3)
qgemv_kernel(QmvArgs p, QgGeom g, const __grid_constant__ CUtensorMap tmw) {
  using T = QGT<BITS, GS>;
  constexpr int LB = T::LB, WL = T::WL, GB = T::GB, GC = T::GC;
  constexpr int BPG = GS / 8;  // 8-value x blocks per group
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
  const int64_t row_base = (int64_t)(blockIdx.x / C) * 16 * S;
  const int64_t KG = p.K / GS;
  const int64_t cg0 = (int64_t)crank * g.KGC;
  const int ncg = (int)(KG - cg0 < g.KGC ? (KG - cg0 > 0 ? KG - cg0 : 0) : g.KGC);
  const int s = warp % S, ksub = warp / S;
  const int wg0 = ksub * g.GW;
  const int nwg = ncg - wg0 < g.GW ? (ncg - wg0 > 0 ? ncg - wg0 : 0) : g.GW;

  QgSmem L;
  L.init(g, M);
  uint8_t* xs = smem + L.o_xs;
  float* xsumb = reinterpret_cast<float*>(smem + L.o_xsum);       // [g][t] sum of x
  float* xsumq = xsumb + (size_t)g.KGC * QG_TOKP;                 // [g][t] 1024 * sum of staged x
  uint32_t* sb = reinterpret_cast<uint32_t*>(smem + L.o_sb);
  float* red = reinterpret_cast<float*>(smem + L.o_red);
  float* ctile = reinterpret_cast<float*>(smem + L.o_ctile);
  const int D = g.D;
  uint8_t* ring = smem + L.o_ring + (size_t)warp * D * QG_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.o_bar) + warp * D;

  // Weights and scales are static: start streaming them before waiting on the
  // previous kernel (programmatic dependent launch), and let the next kernel launch.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int nch = (nwg + GC - 1) / GC;  // ring stages of this warp
  const int wrow = (int)(row_base + s * 16);
  const int wx0 = (int)((cg0 + wg0) * GB);
  if (lane == 0) {
    for (int d = 0; d < D; d++) mbar_init(&bars[d], 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (lane == 0) {
    tma_prefetch_desc(&tmw);
    for (int j = 0; j < nch && j < D; j++) {
      mbar_arrive_expect_tx(&bars[j], QG_STAGE_BYTES);
      tma_load_2d(ring + j * QG_STAGE_BYTES, &tmw, wx0 + j * GC * GB, wrow, &bars[j]);
    }
  }

  // (scale, bias) of the CTA's rows and groups as bf16 pairs.  Items are (row, octet of
  // 8 groups); each thread issues the loads of up to 4 items before storing any, so the
  // staging costs one memory latency rather than one per item.
  {
    const int noct = (ncg + 7) >> 3;
    const int items = 16 * S * noct;
    const bool vec = g.sc_vec;
    for (int base = 0; base < items; base += 4 * QG_THREADS) {
      uint4 sv[4], bv[4];
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i = base + b * QG_THREADS + tid;
        sv[b] = bv[b] = make_uint4(0, 0, 0, 0);
        if (i < items) {
          const int r = i / noct, o8 = (i - r * noct) * 8;
          const int64_t row = row_base + r < p.N ? row_base + r : p.N - 1;
          const bf16* sp = p.scales + row * KG + cg0 + o8;
          const bf16* bp = p.biases + row * KG + cg0 + o8;
          if (vec) {
            sv[b] = *reinterpret_cast<const uint4*>(sp);
            bv[b] = *reinterpret_cast<const uint4*>(bp);
          } else {
            uint16_t ts[8], tb[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
              ts[e] = o8 + e < ncg ? __bfloat16_as_ushort(sp[e]) : 0;
              tb[e] = o8 + e < ncg ? __bfloat16_as_ushort(bp[e]) : 0;
            }
            sv[b] = make_uint4(ts[0] | (uint32_t)ts[1] << 16, ts[2] | (uint32_t)ts[3] << 16,
                               ts[4] | (uint32_t)ts[5] << 16, ts[6] | (uint32_t)ts[7] << 16);
            bv[b] = make_uint4(tb[0] | (uint32_t)tb[1] << 16, tb[2] | (uint32_t)tb[3] << 16,
                               tb[4] | (uint32_t)tb[5] << 16, tb[6] | (uint32_t)tb[7] << 16);
          }
        }
      }
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i = base + b * QG_THREADS + tid;
        if (i < items) {
          const int r = i / noct, o8 = (i - r * noct) * 8;
          const uint32_t su[4] = {sv[b].x, sv[b].y, sv[b].z, sv[b].w};
          const uint32_t bu[4] = {bv[b].x, bv[b].y, bv[b].z, bv[b].w};
          uint32_t* dst = sb + r * g.sbstr + o8;
#pragma unroll
          for (int e = 0; e < 4; e++) {
            if (o8 + 2 * e < ncg) dst[2 * e] = prmt(su[e], bu[e], 0x5410);
            if (o8 + 2 * e + 1 < ncg) dst[2 * e + 1] = prmt(su[e], bu[e], 0x7632);
          }
        }
      }
    }
  }

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

  // ---- stream the warp's groups ----
  float acc[4] = {0.f, 0.f, 0.f, 0.f};   // scale * sum(x'(code)) - scale * Q, x' domain
  float accb[4] = {0.f, 0.f, 0.f, 0.f};  // bias * X
  const bool tv = gq < M;
  const uint8_t* xlane = xs + (size_t)(tv ? gq : 0) * g.xstr + (size_t)c * (GS / 4) * 2;
  const uint32_t* sb0p = sb + (s * 16 + gq) * g.sbstr;
  const uint32_t* sb1p = sb0p + 8 * g.sbstr;
  bool ok = true;
  for (int j = 0; j < nch; j++) {
    const int st = j % D;
    ok &= mbar_wait(&bars[st], (uint32_t)(j / D) & 1u);
    const uint8_t* stg = ring + st * QG_STAGE_BYTES;
#pragma unroll
    for (int gi = 0; gi < GC; gi++) {
      if (j * GC + gi < nwg) {
        const int gl = wg0 + j * GC + gi;
        uint32_t w0[WL], w1[WL];
        lds_lane<LB>(stg, gq, gi * GB + c * LB, w0);
        lds_lane<LB>(stg, gq + 8, gi * GB + c * LB, w1);
        float ag[4] = {0.f, 0.f, 0.f, 0.f};
        const uint8_t* xp = xlane + (size_t)gl * GS * 2;
#if defined(QG_X_NOMMA)
        ag[0] = __uint_as_float(w0[0] ^ w1[WL - 1]); ag[1] = ag[0]; ag[2] = ag[0]; ag[3] = ag[0];
        if (false) {
#else
        if constexpr (BITS == 4) {
#endif
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
#if defined(QG_X_NOFOLD)
        acc[0] += ag[0]; acc[1] += ag[1]; acc[2] += ag[2]; acc[3] += ag[3];
        if (false) {
#else
        {
#endif
        const uint32_t q0 = sb0p[gl], q1 = sb1p[gl];
        const float s0 = __uint_as_float(q0 << 16), s1 = __uint_as_float(q1 << 16);
        const float b0 = __uint_as_float(q0 & 0xFFFF0000u), b1 = __uint_as_float(q1 & 0xFFFF0000u);
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
    }
    // refill this stage once every lane has read it (generic reads before the async write)
    __syncwarp();
    if (lane == 0 && j + D < nch) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(&bars[st], QG_STAGE_BYTES);
      tma_load_2d(ring + st * QG_STAGE_BYTES, &tmw, wx0 + (j + D) * GC * GB, wrow, &bars[st]);
    }
  }
  if (!ok && p.status) atomicExch(p.status, VMLX_E_STATE);

  // ---- fixed-order reduction: warps of the CTA, then the CTAs of the cluster ----
  // accumulator (row gq / gq+8, tokens 2c, 2c+1) -> red[warp][row][token]
  {
    // back from the x' domain: y = 2^-s * acc + accb
    const float e0 = 2 * c < M ? xscale[2 * c] : 0.f, e1 = 2 * c + 1 < M ? xscale[2 * c + 1] : 0.f;
    float* rw = red + (size_t)warp * 16 * QG_TOKP;
    *reinterpret_cast<float2*>(rw + gq * QG_TOKP + 2 * c) =
        make_float2(fmaf(acc[0], e0, accb[0]), fmaf(acc[1], e1, accb[1]));
    *reinterpret_cast<float2*>(rw + (gq + 8) * QG_TOKP + 2 * c) =
        make_float2(fmaf(acc[2], e0, accb[2]), fmaf(acc[3], e1, accb[3]));
  }
  __syncthreads();
  const int KSPLIT = QG_WARPS / S;
  for (int i = tid; i < 16 * S * M; i += QG_THREADS) {
    const int r = i / M, t = i - r * M;
    const int ss_ = r >> 4, rr = r & 15;
    float v = 0.f;
    for (int q = 0; q < KSPLIT; q++) v += red[((size_t)(q * S + ss_) * 16 + rr) * QG_TOKP + t];
    if (C == 1) {
      const int64_t n = row_base + r;
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
    const int rlo = crank * 16 * S / C, rhi = (crank + 1) * 16 * S / C;
    for (int i = tid; i < (rhi - rlo) * M; i += QG_THREADS) {
      const int r = rlo + i / M, t = i % M;
      float v = 0.f;
      for (int q = 0; q < C; q++) v += cluster.map_shared_rank(ctile, q)[r * QG_TOKP + t];
      const int64_t n = row_base + r;
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
    cluster_arrive();  // keep this CTA's shared memory alive until every peer has read it
    cluster_wait();
  }
}

// ---- host side -------------------------------------------------------------

static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

// Geometry from (N, K, bits, group size) only.  Cost, in units of one warp streaming one
// 16-row group: the busiest SM's share of whole CTAs, plus a fixed cost per CTA wave
// (prologue, DRAM latency) and per cluster reduction.  Shared memory is sized for the
// largest M of the regime so that the geometry never depends on M.
static bool qg_choose(int64_t N, int64_t K, int bits, int gs, QgGeom& best) {
  const int64_t KG = K / gs;
  const int64_t strips = (N + 15) / 16;
  const int sms = sm_count();
  double best_cost = 1e30;
  bool found = false;
  const int forceS = env_int("VMLX_QG_S", 0), forceC = env_int("VMLX_QG_C", 0);
  for (int C = 1; C <= QG_MAX_CLUSTER && C <= KG; C++) {
    if (forceC && C != forceC) continue;
    const int KGC = (int)((KG + C - 1) / C);
    if ((int64_t)(C - 1) * KGC >= KG) continue;  // an empty CTA
    for (int S = 1; S <= QG_WARPS; S *= 2) {
      if (forceS && S != forceS) continue;
      const int KSPLIT = QG_WARPS / S;
      QgGeom gm;
      gm.S = S;
      gm.C = C;
      gm.KGC = KGC;
      const int GC = 128 / (gs * bits / 8);
      gm.GW = ((KGC + KSPLIT - 1) / KSPLIT + GC - 1) / GC * GC;  // whole ring stages per warp
      if ((int64_t)(KSPLIT - 1) * gm.GW >= KGC && KSPLIT > 1) continue;  // an idle warp
      gm.xstr = KGC * gs * 2 + 16;
      gm.sbstr = (KGC + 7) / 8 * 8 + 1;
      gm.D = env_int("VMLX_QG_D", QG_STAGES);
      gm.dbg = env_int("VMLX_QG_DBG", 0);
      QgSmem L;
      L.init(gm, QG_MAXM);
      if (L.total > 200 * 1024) continue;
      const int64_t ctas = (strips + S - 1) / S * C;
      const int per_sm = (int)((220 * 1024) / (L.total + 2048)) < 3 ? (int)((220 * 1024) / (L.total + 2048)) : 3;
      if (per_sm < 1) continue;
      const double waves = (double)((ctas + (int64_t)sms * per_sm - 1) / ((int64_t)sms * per_sm));
      const double stream = (double)((ctas + sms - 1) / sms) * QG_WARPS * gm.GW;
      const double cost = stream + 120.0 * waves + (C > 1 ? 80.0 : 0.0) + 0.01 * S;
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
  g.sc_vec = (a.K / GS) % 8 == 0 && g.KGC % 8 == 0 && aligned(a.scales, 16) && aligned(a.biases, 16);
  QgSmem L;
  L.init(g, (int)a.M);
  auto kern = qgemv_kernel<BITS, GS>;
  {
    const int rc = ensure_max_dynamic_smem((const void*)kern, 220 * 1024);
    if (rc) return rc;
  }
  const int64_t ctas = (a.N + 16 * g.S - 1) / (16 * g.S) * g.C;
  if (ctas >= (1LL << 31)) return set_error(VMLX_E_UNSUPPORTED, "qgemv: N=%lld too large", (long long)a.N);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas, 1, 1);
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
  if (a.K % 8) return false;
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
