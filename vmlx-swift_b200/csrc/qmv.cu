// qmv.cu -- decode GEMV / skinny GEMM (M <= 32) for MLX affine-quantized weights.
//
// Computes y[tok, n] = sum_k x[tok, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g])
// for the decode regime, replacing MLX's affine_qmv_fast / affine_qmv
// (Source/Cmlx/mlx-generated/metal/quantized.h:799-1025) and the gathered
// variants affine_gather_qmv(_fast) (:1875-1997) / sorted affine_gather_qmm_rhs
// (:2197-2391) for small runs.
//
// B200 design.  The op is HBM-bound: 0.5625 B/weight (4-bit, g64, bf16
// scale+bias).  Each CTA owns 16 output rows (one m16 tile of the tensor-core
// MMA) and its 8 warps split K into contiguous ranges.  Per group of g weights
// every lane streams g*bits/128 words of two rows (row r and r+8) with
// L1-bypassing vector loads -- the four lanes of a quad cover one group of one
// row, i.e. whole 32-byte sectors -- and unpacks the codes in registers into
// bf16 A fragments holding q exactly (4-bit: prmt with a 0x43 exponent byte
// gives 128+q; 8-bit: the 2^23 float trick).  mma.m16n8k16 (bf16 in, fp32
// accumulate) forms sum(x*q) per group with exact products, a second MMA
// against an all-ones tile forms sum(x), and the group is folded as
// scale*sum(x*q) + bias*sum(x) -- the factorisation of MLX's qdot
// (quantized.h:209-316), so no rounded bf16 weight is ever formed.
// Because a dot product does not care about the order of k, the nibbles are
// used in the order the unpack produces them and x is permuted to match
// (four prmt per eight x values), so no shifts by position are needed.
// Tokens are the MMA's N dimension (8 per tile, up to 4 tiles = 32 rows).
// The 8 warps' partial tiles are summed through shared memory and written
// once as bf16: no global scratch, no atomics, deterministic, and each row's
// result does not depend on M (batch invariance, as the reference's
// QuantizedSmallMScalingBenchTests.swift:110-127 requires).
#include "kernels.cuh"

namespace vmlx {

constexpr int QMV_WARPS = 8;
constexpr int QMV_ROWS = 16;

template <int BITS, int GS>
struct QT {
  static constexpr int WPL = GS * BITS / 128;  // words per lane per row per group
  static constexpr int VPL = GS / 4;           // k values per lane per group
  static constexpr int WPG = GS * BITS / 32;   // words per row per group
  static constexpr int U = (16 / WPL) < 1 ? 1 : (16 / WPL);  // groups in flight per warp
};

// Lower bound of `e` in the non-decreasing array a[0, n).
__device__ __forceinline__ int64_t lower_bound_u32(const uint32_t* a, int64_t n, uint32_t e) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (a[mid] < e) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Row pointers of token `tok` of the CTA's token list (tok < ntok).
__device__ __forceinline__ void token_rows(const QmvArgs& p, int mode, int64_t b_or_r0, int64_t tok,
                                           const bf16*& xr, bf16*& yr) {
  if (mode == QMV_DENSE) {
    xr = p.x + tok * p.K;
    yr = p.y + tok * p.N;
  } else if (mode == QMV_GATHER) {
    int64_t b = b_or_r0;
    int64_t xi = p.lhs ? (int64_t)p.lhs[b] : (b * p.x_batches / p.batch);
    xr = p.x + (xi * p.M + tok) * p.K;
    yr = p.y + (b * p.M + tok) * p.N;
  } else {
    int64_t r = b_or_r0 + tok;  // flattened (b, m) row
    int64_t b = r / p.M, m = r - b * p.M;
    int64_t xi = p.lhs ? (int64_t)p.lhs[b] : (b * p.x_batches / p.batch);
    xr = p.x + (xi * p.M + m) * p.K;
    yr = p.y + r * p.N;
  }
}

// Unpack one 4-bit word into bf16 pairs holding 128+q exactly (prmt with a
// 0x43 exponent byte).  p[0] = nibbles (0,2), p[1] = (4,6), p[2] = (1,3),
// p[3] = (5,7): the order the two masks produce, matched by the x permutation.
__device__ __forceinline__ void unpack4(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t C43 = 0x43434343u;
  uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  p[0] = prmt(lo, C43, 0x4140);
  p[1] = prmt(lo, C43, 0x4342);
  p[2] = prmt(hi, C43, 0x4140);
  p[3] = prmt(hi, C43, 0x4342);
}

// Unpack one 8-bit word (4 consecutive k) into two bf16 pairs holding q exactly
// (the 2^23 float trick, then a packed convert; q <= 255 is exact in bf16).
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t (&p)[2]) {
  const float MAGIC = 8388608.0f;
  const uint32_t K4B = 0x4B000000u;
  float f0 = __uint_as_float(prmt(w, K4B, 0x7540)) - MAGIC;
  float f1 = __uint_as_float(prmt(w, K4B, 0x7541)) - MAGIC;
  float f2 = __uint_as_float(prmt(w, K4B, 0x7542)) - MAGIC;
  float f3 = __uint_as_float(prmt(w, K4B, 0x7543)) - MAGIC;
  p[0] = bf162_as_u32(__floats2bfloat162_rn(f0, f1));
  p[1] = bf162_as_u32(__floats2bfloat162_rn(f2, f3));
}

template <int BITS, int GS, int NT>
__global__ void __launch_bounds__(QMV_WARPS * 32)
qmv_kernel(QmvArgs p, int mode) {
  using T = QT<BITS, GS>;
  constexpr int WPL = T::WPL, VPL = T::VPL, WPG = T::WPG, U = T::U;
  __shared__ float red[QMV_WARPS][NT * 8][QMV_ROWS + 1];

  // A fragment of an all-ones 16x16 bf16 tile (1.0 = 0x3F80)
  const uint32_t kOnes[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, c = lane & 3;
  const int64_t n0 = (int64_t)blockIdx.x * QMV_ROWS;
  const int64_t KG = p.K / GS;
  const int64_t wrow = p.K * BITS / 32;  // words per weight row

  // ---- which weight matrix and which tokens this CTA serves ----
  const uint32_t* W = p.w;
  const bf16* S = p.scales;
  const bf16* B = p.biases;
  int64_t ntok_total = p.M, base = 0;
  bool zero_rows = false;
  if (mode == QMV_GATHER) {
    base = blockIdx.y;
    uint32_t e = p.rhs[base];
    if ((int64_t)e >= p.n_experts) zero_rows = true;
    else {
      W += (int64_t)e * p.N * wrow;
      S += (int64_t)e * p.N * KG;
      B += (int64_t)e * p.N * KG;
    }
  } else if (mode == QMV_SORTED) {
    uint32_t e = blockIdx.y;
    int64_t lo = lower_bound_u32(p.rhs, p.batch, e);
    int64_t hi = lower_bound_u32(p.rhs, p.batch, e + 1);
    if (lo >= hi) return;  // no rows routed to this expert
    base = lo * p.M;
    ntok_total = (hi - lo) * p.M;
    W += (int64_t)e * p.N * wrow;
    S += (int64_t)e * p.N * KG;
    B += (int64_t)e * p.N * KG;
  }

  // rows owned by this lane (clamped for loads; results past N are dropped)
  const int64_t r0 = n0 + gq, r1 = n0 + gq + 8;
  const int64_t r0c = r0 < p.N ? r0 : p.N - 1, r1c = r1 < p.N ? r1 : p.N - 1;
  const uint32_t* w0p = W + r0c * wrow + c * WPL;
  const uint32_t* w1p = W + r1c * wrow + c * WPL;
  const bf16* s0p = S + r0c * KG;
  const bf16* s1p = S + r1c * KG;
  const bf16* b0p = B + r0c * KG;
  const bf16* b1p = B + r1c * KG;

  // contiguous K split over warps (in groups)
  const int64_t gper = (KG + QMV_WARPS - 1) / QMV_WARPS;
  const int64_t g0 = warp * gper;
  const int64_t g1 = (g0 + gper < KG) ? g0 + gper : KG;

  for (int64_t chunk = 0; chunk < ntok_total; chunk += NT * 8) {
    const int64_t ntok = (ntok_total - chunk) < NT * 8 ? (ntok_total - chunk) : NT * 8;
    // x row of this lane's B-fragment token in each tile
    const bf16* xr[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) {
      int64_t tok = t * 8 + gq;
      bf16* yr_unused;
      xr[t] = nullptr;
      if (tok < ntok && !zero_rows) token_rows(p, mode, base, chunk + tok, xr[t], yr_unused);
    }

    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

    if (!zero_rows) {
      for (int64_t g = g0; g < g1; g += U) {
        uint32_t wv0[U][WPL], wv1[U][WPL];
        bf16 sv0[U], bv0[U], sv1[U], bv1[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
          if (g + u < g1) {
            const int64_t gg = g + u;
            if constexpr (WPL == 1) {
              wv0[u][0] = ldg_stream(w0p + gg * WPG);
              wv1[u][0] = ldg_stream(w1p + gg * WPG);
            } else if constexpr (WPL == 2) {
              uint2 a0 = ldg_stream(reinterpret_cast<const uint2*>(w0p + gg * WPG));
              uint2 a1 = ldg_stream(reinterpret_cast<const uint2*>(w1p + gg * WPG));
              wv0[u][0] = a0.x; wv0[u][1] = a0.y;
              wv1[u][0] = a1.x; wv1[u][1] = a1.y;
            } else {
#pragma unroll
              for (int q = 0; q < WPL; q += 4) {
                uint4 a0 = ldg_stream(reinterpret_cast<const uint4*>(w0p + gg * WPG + q));
                uint4 a1 = ldg_stream(reinterpret_cast<const uint4*>(w1p + gg * WPG + q));
                wv0[u][q] = a0.x; wv0[u][q + 1] = a0.y; wv0[u][q + 2] = a0.z; wv0[u][q + 3] = a0.w;
                wv1[u][q] = a1.x; wv1[u][q + 1] = a1.y; wv1[u][q + 2] = a1.z; wv1[u][q + 3] = a1.w;
              }
            }
            sv0[u] = s0p[gg];
            bv0[u] = b0p[gg];
            sv1[u] = s1p[gg];
            bv1[u] = b1p[gg];
          }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
          if (g + u < g1) {
            const int64_t kbase = (g + u) * GS + c * VPL;
            // Per group: ag = sum_k x*code (exact products, fp32 accumulate),
            // xg = sum_k x (an MMA against an all-ones A tile), then
            // y += scale*ag + bias*xg as MLX's qdot does (quantized.h:209-316).
            float ag[NT][4], xg[NT][4];
#pragma unroll
            for (int t = 0; t < NT; t++)
#pragma unroll
              for (int i = 0; i < 4; i++) ag[t][i] = xg[t][i] = 0.f;
#pragma unroll
            for (int wi = 0; wi < WPL; wi++) {
              if constexpr (BITS == 4) {
                uint32_t p0[4], p1[4];
                unpack4(wv0[u][wi], p0);
                unpack4(wv1[u][wi], p1);
                const uint32_t a0[4] = {p0[0], p1[0], p0[1], p1[1]};
                const uint32_t a1[4] = {p0[2], p1[2], p0[3], p1[3]};
#pragma unroll
                for (int t = 0; t < NT; t++) {
                  uint32_t x02 = 0, x46 = 0, x13 = 0, x57 = 0;
                  if (xr[t]) {
                    uint4 xv = *reinterpret_cast<const uint4*>(xr[t] + kbase + wi * 8);
                    x02 = prmt(xv.x, xv.y, 0x5410);
                    x46 = prmt(xv.z, xv.w, 0x5410);
                    x13 = prmt(xv.x, xv.y, 0x7632);
                    x57 = prmt(xv.z, xv.w, 0x7632);
                  }
                  mma_bf16_16816(ag[t], a0, x02, x46);
                  mma_bf16_16816(ag[t], a1, x13, x57);
                  mma_bf16_16816(xg[t], kOnes, x02, x46);
                  mma_bf16_16816(xg[t], kOnes, x13, x57);
                }
              } else {
                uint32_t p0[2], p1[2];
                unpack8(wv0[u][wi], p0);
                unpack8(wv1[u][wi], p1);
                const uint32_t a[4] = {p0[0], p1[0], p0[1], p1[1]};
#pragma unroll
                for (int t = 0; t < NT; t++) {
                  uint32_t x01 = 0, x23 = 0;
                  if (xr[t]) {
                    uint2 xv = *reinterpret_cast<const uint2*>(xr[t] + kbase + wi * 4);
                    x01 = xv.x;
                    x23 = xv.y;
                  }
                  mma_bf16_16816(ag[t], a, x01, x23);
                  mma_bf16_16816(xg[t], kOnes, x01, x23);
                }
              }
            }
            const float s0 = __bfloat162float(sv0[u]), s1 = __bfloat162float(sv1[u]);
            // 4-bit codes carry +128: fold -128*scale*sum(x) into the bias term
            const float c0 = BITS == 4 ? fmaf(-128.f, s0, __bfloat162float(bv0[u])) : __bfloat162float(bv0[u]);
            const float c1 = BITS == 4 ? fmaf(-128.f, s1, __bfloat162float(bv1[u])) : __bfloat162float(bv1[u]);
#pragma unroll
            for (int t = 0; t < NT; t++) {
              acc[t][0] = fmaf(s0, ag[t][0], fmaf(c0, xg[t][0], acc[t][0]));
              acc[t][1] = fmaf(s0, ag[t][1], fmaf(c0, xg[t][1], acc[t][1]));
              acc[t][2] = fmaf(s1, ag[t][2], fmaf(c1, xg[t][2], acc[t][2]));
              acc[t][3] = fmaf(s1, ag[t][3], fmaf(c1, xg[t][3], acc[t][3]));
            }
          }
        }
      }
    }

    // ---- reduce the 8 warps' partial tiles and store bf16 ----
#pragma unroll
    for (int t = 0; t < NT; t++) {
      red[warp][t * 8 + 2 * c][gq] = acc[t][0];
      red[warp][t * 8 + 2 * c + 1][gq] = acc[t][1];
      red[warp][t * 8 + 2 * c][gq + 8] = acc[t][2];
      red[warp][t * 8 + 2 * c + 1][gq + 8] = acc[t][3];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < NT * 8 * QMV_ROWS; i += QMV_WARPS * 32) {
      int tok = i / QMV_ROWS, r = i % QMV_ROWS;
      if (tok < ntok && n0 + r < p.N) {
        float s = 0.f;
#pragma unroll
        for (int wv = 0; wv < QMV_WARPS; wv++) s += red[wv][tok][r];
        const bf16* xr_unused;
        bf16* yr;
        token_rows(p, mode, base, chunk + tok, xr_unused, yr);
        yr[n0 + r] = __float2bfloat16_rn(s);
      }
    }
    __syncthreads();
  }
}

template <int BITS, int GS>
static void launch_qmv_nt(int nt, const QmvArgs& a, int mode, dim3 grid, cudaStream_t st) {
  dim3 block(QMV_WARPS * 32);
  switch (nt) {
    case 1: qmv_kernel<BITS, GS, 1><<<grid, block, 0, st>>>(a, mode); break;
    case 2: qmv_kernel<BITS, GS, 2><<<grid, block, 0, st>>>(a, mode); break;
    case 3: qmv_kernel<BITS, GS, 3><<<grid, block, 0, st>>>(a, mode); break;
    default: qmv_kernel<BITS, GS, 4><<<grid, block, 0, st>>>(a, mode); break;
  }
}

// Host launcher shared by the dense and gathered entry points.
int launch_qmv(const QmvArgs& a, int mode, int bits, int gs, int64_t grid_y, int nt,
               cudaStream_t st) {
  dim3 grid((unsigned)((a.N + QMV_ROWS - 1) / QMV_ROWS), (unsigned)grid_y);
  if (grid.y > 65535) return set_error(VMLX_E_INVALID, "too many batch elements (%lld)", (long long)grid_y);
  if (bits == 4 && gs == 32) launch_qmv_nt<4, 32>(nt, a, mode, grid, st);
  else if (bits == 4 && gs == 64) launch_qmv_nt<4, 64>(nt, a, mode, grid, st);
  else if (bits == 4 && gs == 128) launch_qmv_nt<4, 128>(nt, a, mode, grid, st);
  else if (bits == 8 && gs == 32) launch_qmv_nt<8, 32>(nt, a, mode, grid, st);
  else if (bits == 8 && gs == 64) launch_qmv_nt<8, 64>(nt, a, mode, grid, st);
  else if (bits == 8 && gs == 128) launch_qmv_nt<8, 128>(nt, a, mode, grid, st);
  else return set_error(VMLX_E_UNSUPPORTED, "matmul: bits=%d group_size=%d not supported", bits, gs);
  return check_launch("qmv_kernel");
}

}  // namespace vmlx
