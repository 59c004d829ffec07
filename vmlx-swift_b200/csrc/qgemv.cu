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
#include <map>
#include <mutex>
#include <tuple>

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
  int cpg;       // 16-byte chunks of packed codes per group
};

struct QgSmem {
  size_t o_ring, o_bar, o_xs, o_xsum, o_sc, o_red, o_ctile, total;
  __host__ __device__ void init(const QgGeom& g, int m) {
    o_ring = 0;  // 1024-byte aligned (the swizzle atom)
    o_bar = o_ring + (size_t)QG_WARPS * QG_STAGES * QG_STAGE_BYTES;
    o_xs = o_bar + (size_t)QG_WARPS * QG_STAGES * 8;
    o_xsum = o_xs + (size_t)m * g.xstr;
    o_sc = o_xsum + (size_t)g.KGC * g.cpg * QG_TOKP * 4;
    o_red = o_sc + (size_t)2 * 2 * 16 * g.S * g.sbrow;  // [buffer][scale | bias][row]
    o_ctile = o_red + (size_t)QG_WARPS * 16 * QG_TOKP * 4;
    total = o_ctile + (g.C > 1 ? (size_t)16 * g.S * QG_TOKP * 4 : 0) + 1024;  // + alignment slack
  }
};

// Byte offset of (row r in 0..15, byte o) in a 128-byte-swizzled [16][128] stage:
// 16-byte chunk j of row r sits at chunk j ^ (r & 7).
__device__ __forceinline__ int swz(int r, int o) { return r * 128 + ((((o >> 4) ^ (r & 7))) << 4) + (o & 15); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Scales and biases of the tile at row0 (the CTA's groups cg0..cg0+ncg) into buffer
// `dst` ([scale | bias][16*S rows][sbrow bytes]).  Asynchronous (cp.async; one commit
// group per call, empty when !valid) when rows are 16-byte aligned, else plain loads.
__device__ __forceinline__ void qg_load_scales(const QmvArgs& p, const QgGeom& g, uint8_t* dst, int64_t row0,
                                               int64_t KG, int64_t cg0, int ncg, bool valid, int tid,
                                               int64_t roff) {
  const int rows = 16 * g.S;
  if (valid) {
    if (g.sc_async) {
      const int nchunk = (ncg + 7) >> 3;  // 8 groups per 16-byte chunk (KGC is a multiple of 8)
      for (int i = tid; i < 2 * rows * nchunk; i += QG_THREADS) {
        const int kind = i / (rows * nchunk), rem = i - kind * rows * nchunk;
        const int r = rem / nchunk, ch = rem - r * nchunk;
        const int64_t row = roff + (row0 + r < p.N ? row0 + r : p.N - 1);
        const bf16* src = (kind ? p.biases : p.scales) + row * KG + cg0 + ch * 8;
        cp_async16(dst + ((size_t)kind * rows + r) * g.sbrow + ch * 16, src);
      }
    } else {
      for (int i = tid; i < 2 * rows * ncg; i += QG_THREADS) {
        const int kind = i / (rows * ncg), rem = i - kind * rows * ncg;
        const int r = rem / ncg, gl = rem - r * ncg;
        const int64_t row = roff + (row0 + r < p.N ? row0 + r : p.N - 1);
        reinterpret_cast<bf16*>(dst + ((size_t)kind * rows + r) * g.sbrow)[gl] =
            (kind ? p.biases : p.scales)[row * KG + cg0 + gl];
      }
    }
  }
  cp_async_commit();
}

// One output element: y = bf16([residual +] bf16(v)); under row-parallel TP the bf16 partial
// goes instead to slot [parity][rank] of every rank's buffer as a {value, epoch} word (P2P
// stores; the reduction over the ranks runs after the tile loop).
__device__ __forceinline__ void qg_store(const QmvArgs& p, int64_t idx, float v, bool tp, int trank, int64_t ybias,
                                         uint32_t tp_e) {
  if (tp) {
    const uint32_t hv = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
    const size_t off = p.tp_slots_off + ((size_t)(tp_e & 1) * p.tp_world + trank) * p.tp_slot_bytes +
                       (size_t)idx * sizeof(uint64_t);
    for (int r = 0; r < p.tp_world; r++) st_ll(reinterpret_cast<uint64_t*>(p.tp_buf[r] + off), hv, tp_e);
    return;
  }
  idx += ybias;
  if (p.residual) {
    const float sv = __bfloat162float(__float2bfloat16_rn(v));
    p.y[idx] = __float2bfloat16_rn(__bfloat162float(p.residual[idx]) + sv);
  } else {
    p.y[idx] = __float2bfloat16_rn(v);
  }
}

template <int GS, int MT>
__global__ void __launch_bounds__(QG_THREADS, 2)
qgemv_kernel(QmvArgs p, QgGeom g, const __grid_constant__ CUtensorMap tmw) {
  constexpr int BITS = 4;
  using T = QGT<BITS, GS>;
  constexpr int GB = T::GB, GC = T::GC;
  constexpr int BPG = GS / 8;  // 8-value x blocks per group
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  __shared__ float xinv[QG_MAXM];    // fused RMSNorm: 1 / rms per token

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  const int S = g.S, C = g.C;
  const int M = MT;
  // Row-parallel TP (tp_world > 1): trank = this CTA's rank; lr = the same for a loopback group
  // (all ranks in one grid, rank = blockIdx.y, operands stacked along a rank axis), else 0.
  const bool tp = p.tp_world > 1;
  const int lr = (tp && p.tp_loop) ? (int)blockIdx.y : 0;
  const int trank = tp ? (p.tp_loop ? lr : p.tp_rank) : 0;
  const int64_t wroff = (int64_t)lr * p.N;     // first weight / scale row of this rank's shard
  const int64_t xrow0 = (int64_t)lr * M;       // first x row of this rank
  const int64_t ybias = (int64_t)lr * M * p.N;  // offset of this rank's y / residual
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
  float* xsum = reinterpret_cast<float*>(smem + L.o_xsum);  // [chunk][t] sum of the chunk's 32 x
  float* red = reinterpret_cast<float*>(smem + L.o_red);
  float* ctile = reinterpret_cast<float*>(smem + L.o_ctile);
  uint8_t* ring = smem + L.o_ring + (size_t)warp * QG_STAGES * QG_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.o_bar) + warp * QG_STAGES;
  const size_t scbuf = (size_t)2 * rows * g.sbrow;

  // Weights and scales are static: start streaming them before waiting on the
  // previous kernel (programmatic dependent launch), and let the next kernel launch.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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
    tma_load_2d(ring + st * QG_STAGE_BYTES, &tmw, x0 + iss_jj * (GC * GB), iss_row + (int)wroff, &bars[st]);
    if (++iss_jj == nch) {
      iss_jj = 0;
      iss_row += row_step;
    }
  };
  if (lane == 0) {
    tma_prefetch_desc(&tmw);
    for (int j = 0; j < total_st && j < QG_STAGES; j++) issue(j);
  }
  qg_load_scales(p, g, smem + L.o_sc, cluster_id * rows, KG, cg0, ncg, ntl > 0, tid, wroff);
  qg_load_scales(p, g, smem + L.o_sc + scbuf, (cluster_id + nclusters) * rows, KG, cg0, ncg, ntl > 1, tid, wroff);

  // x may be written by the previous kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // TP: this call's epoch (advanced by the previous call's last CTA) picks the slot parity
  __shared__ uint32_t s_tp_e;
  if (tp && tid == 0) s_tp_e = *reinterpret_cast<const uint32_t*>(p.tp_buf[trank] + p.tp_epoch_off) + 1;
  if (p.norm_w) {
    // fused RMSNorm: 1 / rms over each token's full row (the order of the other GEMV kernel)
    for (int t = warp; t < M; t += QG_WARPS) {
      const bf16* xr = p.x + (xrow0 + t) * p.K;
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
  // Stage x as bf16 (after the optional SwiGLU / RMSNorm) and the sum of every 32-value
  // chunk (one 16-byte chunk of packed 4-bit codes) per token, in fp32.
  {
    const int nkb = ncg * BPG;  // 8-value blocks per token
    const int total = M * nkb;
    const int64_t xrs = p.x_swiglu ? 2 * p.K : p.K;
    for (int base = 0; base < total; base += 4 * QG_THREADS) {
      uint4 v[4], u[4];  // 4 blocks per thread per pass, all loads issued first
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i = base + b * QG_THREADS + tid;
        v[b] = u[b] = make_uint4(0, 0, 0, 0);
        if (i < total) {
          const int t = i / nkb, kb = i - t * nkb;
          const bf16* xr = p.x + (xrow0 + t) * xrs + cg0 * GS + (int64_t)kb * 8;
          v[b] = *reinterpret_cast<const uint4*>(xr);
          if (p.x_swiglu) u[b] = *reinterpret_cast<const uint4*>(xr + p.K);
        }
      }
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int i = base + b * QG_THREADS + tid;
        const bool in = i < total;
        const int t = in ? i / nkb : 0, kb = in ? i - t * nkb : 0;
        uint4 x8 = v[b];
        if (in && p.x_swiglu)
          x8 = make_uint4(swiglu2(x8.x, u[b].x), swiglu2(x8.y, u[b].y), swiglu2(x8.z, u[b].z), swiglu2(x8.w, u[b].w));
        if (in && p.norm_w) x8 = norm8(x8, xinv[t], p.norm_w + cg0 * GS + (int64_t)kb * 8);
        const float2 v0 = __bfloat1622float2(u32_as_bf162(x8.x)), v1 = __bfloat1622float2(u32_as_bf162(x8.y));
        const float2 v2 = __bfloat1622float2(u32_as_bf162(x8.z)), v3 = __bfloat1622float2(u32_as_bf162(x8.w));
        float sum = ((v0.x + v0.y) + (v1.x + v1.y)) + ((v2.x + v2.y) + (v3.x + v3.y));
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // 4 blocks = one 32-value chunk
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (in) {
          *reinterpret_cast<uint4*>(xs + (size_t)t * g.xstr + (size_t)kb * 16) = x8;
          if ((kb & 3) == 0) xsum[(kb >> 2) * QG_TOKP + t] = sum;
        }
      }
    }
  }
  __syncthreads();

  // ---- stream the warp's stages, tile after tile ----
  // lane = (rs, kc): 16-byte chunk kc of each 128-byte stage row, rows rs + 4j of the strip
  const int rs = lane >> 3, kc = lane & 7;
  int soff[4];
#pragma unroll
  for (int jr = 0; jr < 4; jr++) soff[jr] = swz(rs + 4 * jr, kc * 16);
  constexpr int CPG = GB / 16;  // 16-byte chunks per group
  bool ok = true;
  int j = 0, st = 0;
  uint32_t phase = 0;
  for (int64_t ti = 0; ti < ntl; ti++) {
    const int64_t row0 = (cluster_id + ti * nclusters) * rows;
    uint8_t* scb = smem + L.o_sc + (size_t)(ti & 1) * scbuf;
    cp_async_wait1();  // this tile's scales (all but the newest copy group)
    __syncthreads();   // ... visible to every thread; the previous tile's reduction is done
    float res[4][MT];
#pragma unroll
    for (int jr = 0; jr < 4; jr++)
#pragma unroll
      for (int t = 0; t < MT; t++) res[jr][t] = 0.f;
    for (int jj = 0; jj < nch; jj++, j++) {  // j: this warp's stage counter
      ok &= mbar_wait(&bars[st], phase);
      const uint8_t* stg = ring + st * QG_STAGE_BYTES;
      uint4 wv[4];
#pragma unroll
      for (int jr = 0; jr < 4; jr++) wv[jr] = *reinterpret_cast<const uint4*>(stg + soff[jr]);
      // refill this stage now that every lane has read it (generic reads before the async write)
      __syncwarp();
      if (lane == 0 && j + QG_STAGES < total_st) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        issue(st);
      }
      if (++st == QG_STAGES) {
        st = 0;
        phase ^= 1u;
      }
      const int cw = jj * GC * CPG + kc;  // chunk index inside the warp's range
      if (cw < nwg * CPG) {
        const int chl = wg0 * CPG + cw;  // chunk index inside the CTA's range
        const int gl = chl / CPG;
        // x of the chunk for every token as bf16 pairs (x[2i], x[2i+1])
        uint32_t xw[MT][16];
#pragma unroll
        for (int t = 0; t < MT; t++) {
          const uint4* xp = reinterpret_cast<const uint4*>(xs + (size_t)t * g.xstr + (size_t)chl * 64);
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const uint4 xv = xp[q];
            xw[t][4 * q] = xv.x; xw[t][4 * q + 1] = xv.y; xw[t][4 * q + 2] = xv.z; xw[t][4 * q + 3] = xv.w;
          }
        }
        unsigned long long sacc[4][MT];
#pragma unroll
        for (int jr = 0; jr < 4; jr++)
#pragma unroll
          for (int t = 0; t < MT; t++) sacc[jr][t] = 0ull;
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            // x pair (x[8wi+2i], x[8wi+2i+1]) for each token
            unsigned long long xp2[MT];
#pragma unroll
            for (int t = 0; t < MT; t++) {
              const uint32_t w2 = xw[t][wi * 4 + i];
              xp2[t] = pack_u2(w2 << 16, w2 & 0xFFFF0000u);
            }
#pragma unroll
            for (int jr = 0; jr < 4; jr++) {
              const uint32_t w = wi == 0 ? wv[jr].x : wi == 1 ? wv[jr].y : wi == 2 ? wv[jr].z : wv[jr].w;
              const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
              // (128 + q) as exact fp32 for nibbles 2i, 2i+1: bytes [0, 0, q, 0x43]
              const uint32_t fl = prmt(lo, 0x43000000u, 0x7044u | (i << 8));
              const uint32_t fh = prmt(hi, 0x43000000u, 0x7044u | (i << 8));
              const unsigned long long wp = pack_u2(fl, fh);
#pragma unroll
              for (int t = 0; t < MT; t++) ffma2(sacc[jr][t], wp, xp2[t]);
            }
          }
        }
        // fold the chunk: scale * sum(x (128 + q)) + (bias - 128 scale) * sum(x)
#pragma unroll
        for (int jr = 0; jr < 4; jr++) {
          const int r = s * 16 + rs + 4 * jr;
          const float sv = __bfloat162float(*reinterpret_cast<const bf16*>(scb + (size_t)r * g.sbrow + gl * 2));
          const float bv = fmaf(-128.f, sv,
                                __bfloat162float(*reinterpret_cast<const bf16*>(scb + (size_t)(rows + r) * g.sbrow + gl * 2)));
#pragma unroll
          for (int t = 0; t < MT; t++) {
            const float2 sp = unpack_f2(sacc[jr][t]);
            res[jr][t] = fmaf(sv, sp.x + sp.y, fmaf(bv, xsum[chl * QG_TOKP + t], res[jr][t]));
          }
        }
      }
    }
    // the 8 chunk lanes of each row, then res -> red[warp][row][token]
#pragma unroll
    for (int jr = 0; jr < 4; jr++)
#pragma unroll
      for (int t = 0; t < MT; t++) {
        float v = res[jr][t];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        res[jr][t] = v;
      }
    if (kc == 0) {
      float* rw = red + (size_t)warp * 16 * QG_TOKP;
#pragma unroll
      for (int jr = 0; jr < 4; jr++)
#pragma unroll
        for (int t = 0; t < MT; t++) rw[(rs + 4 * jr) * QG_TOKP + t] = res[jr][t];
    }

    // ---- fixed-order reduction: warps of the CTA, then the CTAs of the cluster ----
    __syncthreads();
    // the buffer of this tile's scales is free: start copying the scales two tiles ahead
    qg_load_scales(p, g, scb, (cluster_id + (ti + 2) * nclusters) * rows, KG, cg0, ncg, ti + 2 < ntl, tid, wroff);
    const int KSPLIT = QG_WARPS / S;
    for (int i = tid; i < rows * M; i += QG_THREADS) {
      const int r = i / M, t = i - r * M;
      const int ss_ = r >> 4, rr = r & 15;
      float v = 0.f;
      for (int q = 0; q < KSPLIT; q++) v += red[((size_t)(q * S + ss_) * 16 + rr) * QG_TOKP + t];
      if (C == 1) {
        const int64_t n = row0 + r;
        if (n < p.N) qg_store(p, (int64_t)t * p.N + n, v, tp, trank, ybias, tp ? s_tp_e : 0u);
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
        if (n < p.N) qg_store(p, (int64_t)t * p.N + n, v, tp, trank, ybias, tp ? s_tp_e : 0u);
      }
      cluster_arrive();  // peers have read this CTA's tile before it is overwritten or freed
      cluster_wait();
    }
  }
  if (tp) {
    // ---- row-parallel all-reduce: the rows this CTA wrote, from every rank, in rank order ----
    // (each word is polled until it carries this call's epoch; every CTA of every rank is
    // resident, the grid being one persistent wave)
    const uint32_t e = s_tp_e;
    const uint64_t deadline = globaltimer() + p.tp_timeout_ns;
    const uint64_t* slots = reinterpret_cast<const uint64_t*>(p.tp_buf[trank] + p.tp_slots_off +
                                                              (size_t)(e & 1) * p.tp_world * p.tp_slot_bytes);
    const size_t rstride = p.tp_slot_bytes / sizeof(uint64_t);
    const int rlo = C > 1 ? crank * rows / C : 0, rhi = C > 1 ? (crank + 1) * rows / C : rows;
    bool tp_ok = true;
    for (int64_t ti = 0; ti < ntl && tp_ok; ti++) {
      const int64_t row0 = (cluster_id + ti * nclusters) * rows;
      for (int i = tid; i < (rhi - rlo) * M && tp_ok; i += QG_THREADS) {
        const int r = rlo + i / M, t = i % M;
        const int64_t n = row0 + r;
        if (n >= p.N) continue;
        const int64_t idx = (int64_t)t * p.N + n;
        float sum;
        tp_ok = wait_ll_sum<QMV_TP_MAX_WORLD>(slots + idx, rstride, p.tp_world, e, deadline, sum);
        if (!tp_ok) break;
        const bf16 sb = __float2bfloat16_rn(sum);
        const int64_t yi = idx + ybias;
        p.y[yi] = p.residual ? __float2bfloat16_rn(__bfloat162float(p.residual[yi]) + __bfloat162float(sb)) : sb;
      }
    }
    if (!tp_ok && p.tp_status) atomicExch(p.tp_status, VMLX_E_PEER_TIMEOUT);
    __syncthreads();
    if (tid == 0) {  // the grid's last CTA (of this rank) advances the epoch for the next call
      uint32_t* ep = reinterpret_cast<uint32_t*>(p.tp_buf[trank] + p.tp_epoch_off);
      __threadfence();
      if (atomicAdd(ep + 1, 1u) == gridDim.x - 1) {
        ep[1] = 0;
        ep[0] = e;
        __threadfence();
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (!ok && p.status) atomicExch(p.status, VMLX_E_STATE);
}

// ---- host side -------------------------------------------------------------

// Tuning overrides read once per process: VMLX_QG (force this kernel on / off),
// VMLX_QG_S / VMLX_QG_C (force the strips per tile / the cluster size).
static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}
static int env_cached(int which) {
  static const int vals[3] = {env_int("VMLX_QG", -1), env_int("VMLX_QG_S", 0), env_int("VMLX_QG_C", 0)};
  return vals[which];
}

// Resident CTAs per SM: shared memory, and registers (up to 128 per thread: 2 CTAs of 256).
static int qg_per_sm(const QgSmem& L, int m = QG_MAXM) {
  int per = (int)((228 * 1024) / (L.total + 1024));
  const int reg_cap = 2;
  (void)m;
  return per > reg_cap ? reg_cap : per;
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
  gm.cpg = gs / 32;
  gm.ntiles = (int)((N + 16 * S - 1) / (16 * S));
}

// Geometry from (N, K, bits, group size) only.  The busiest CTA's work (tiles x ring
// stages per warp, plus a fixed cost per tile and per cluster reduction) against the
// bandwidth share of the resident CTAs; shared memory is sized for the regime's largest
// M so that the geometry never depends on M.
// Clusters of C CTAs that can be resident at once for this geometry's shared memory (whole
// clusters per GPC), queried on one instance of the kernel (the geometry must not depend on M).
static int qg_resident_clusters(int gs, int C, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(gs, C, smem, dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const void* fn = gs == 32 ? (const void*)qgemv_kernel<32, 4>
                 : gs == 64 ? (const void*)qgemv_kernel<64, 4> : (const void*)qgemv_kernel<128, 4>;
  int n = 0;
  if (!ensure_max_dynamic_smem(fn, 220 * 1024)) {
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3((unsigned)C, 1, 1);
    q.blockDim = dim3(QG_THREADS);
    q.dynamicSmemBytes = smem;
    cudaLaunchAttribute ca;
    ca.id = cudaLaunchAttributeClusterDimension;
    ca.val.clusterDim.x = (unsigned)C;
    ca.val.clusterDim.y = 1;
    ca.val.clusterDim.z = 1;
    q.attrs = &ca;
    q.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &q) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

static bool qg_choose(int64_t N, int64_t K, int bits, int gs, QgGeom& best) {
  const int64_t KG = K / gs;
  const int GC = 128 / (gs * bits / 8);
  const int sms = sm_count();
  const int forceS = env_cached(1), forceC = env_cached(2);
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
      int64_t nclu = std::min<int64_t>(gm.ntiles, (int64_t)sms * per_sm / C);
      {
        const int res = qg_resident_clusters(gs, C, L.total);
        if (res > 0 && res < nclu) nclu = res;
      }
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

template <int GS, int MT>
static int launch_qg(const QmvArgs& a, cudaStream_t st) {
  constexpr int BITS = 4;
  QgGeom g;
  if (!qg_choose(a.N, a.K, BITS, GS, g))
    return set_error(VMLX_E_UNSUPPORTED, "qgemv: no launch geometry for N=%lld K=%lld", (long long)a.N,
                     (long long)a.K);
  g.sc_async = (a.K / GS) % 8 == 0 && aligned(a.scales, 16) && aligned(a.biases, 16);
  QgSmem L;
  L.init(g, (int)a.M);
  auto kern = qgemv_kernel<GS, MT>;
  {
    const int rc = ensure_max_dynamic_smem((const void*)kern, 220 * 1024);
    if (rc) return rc;
  }
  // A loopback TP group runs every rank's grid in one launch: the ranks share the SMs.
  const int ranks = (a.tp_world > 1 && a.tp_loop) ? a.tp_world : 1;
  int64_t nclu = std::min<int64_t>(g.ntiles, (int64_t)sm_count() * qg_per_sm(L, MT) / g.C / ranks);
  {
    QgSmem L4;
    L4.init(g, QG_MAXM);
    const int res = qg_resident_clusters(GS, g.C, L4.total);
    if (res > 0 && nclu > res / ranks) nclu = std::max<int64_t>(1, res / ranks);
  }
  if (a.tp_world > 1) {
    // every CTA waits for the other ranks after its own rows: the whole grid must be resident
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3((unsigned)g.C, 1, 1);
    q.blockDim = dim3(QG_THREADS);
    q.dynamicSmemBytes = L.total;
    cudaLaunchAttribute ca;
    ca.id = cudaLaunchAttributeClusterDimension;
    ca.val.clusterDim.x = (unsigned)g.C;
    ca.val.clusterDim.y = 1;
    ca.val.clusterDim.z = 1;
    q.attrs = &ca;
    q.numAttrs = 1;
    int resident = 0;
    if (cudaOccupancyMaxActiveClusters(&resident, kern, &q) != cudaSuccess || resident < ranks) {
      cudaGetLastError();
      return set_error(VMLX_E_UNSUPPORTED, "qgemv tp: %d ranks of %d-CTA clusters cannot be resident together",
                       ranks, g.C);
    }
    if (nclu > resident / ranks) nclu = resident / ranks;
    if (nclu < 1) nclu = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nclu * g.C), (unsigned)ranks, 1);
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
  if (ranks > 1) {  // the ranks' CTAs wait on one another: all resident at once, or no launch
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  CUtensorMap tmw;
  const uint64_t rowb = (uint64_t)a.K * BITS / 8;
  if (!make_tmap_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, rowb, (uint64_t)(a.N * ranks), rowb, 128, 16,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return VMLX_E_CUDA;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, a, g, tmw), "qgemv_kernel launch");
}

bool qgemv_covers(const QmvArgs& a, int mode, int bits, int gs) {
  if (mode != QMV_DENSE) return false;
  if (a.M < 1 || a.M > QG_MAXM) return false;
  if (a.K % 8 || a.N >= (1LL << 31)) return false;
  if (!aligned(a.x, 16) || (a.norm_w && !aligned(a.norm_w, 16))) return false;
  if (bits != 4) return false;
  // By shape, never by M (one kernel per (N, K) keeps rows batch-invariant across M = 1..4):
  // measured on B200 (CUDA graph, rotated weights > L2), this kernel wins on matrices up to
  // ~8K x 8K; the ring-and-cluster kernel of qmv.cu keeps the larger ones, where its deeper
  // K split hides more latency.  VMLX_QG=1 / 0 forces the choice.
  (void)gs;
  const int force = env_cached(0);
  if (force >= 0) return force != 0;
  // (5120 x 8192, the Qwen3-32B o_proj: 13.8 us here against 11.9 us on the other kernel)
  return a.N >= 1024 && a.N <= 8192 && a.K <= 8192 && a.N * a.K <= (32LL << 20);
}

template <int GS>
static int launch_qg_m(const QmvArgs& a, cudaStream_t st) {
  switch (a.M) {
    case 1: return launch_qg<GS, 1>(a, st);
    case 2: return launch_qg<GS, 2>(a, st);
    case 3: return launch_qg<GS, 3>(a, st);
    default: return launch_qg<GS, 4>(a, st);
  }
}

int launch_qgemv(const QmvArgs& a, int bits, int gs, cudaStream_t st) {
  if (bits == 4 && gs == 32) return launch_qg_m<32>(a, st);
  if (bits == 4 && gs == 64) return launch_qg_m<64>(a, st);
  if (bits == 4 && gs == 128) return launch_qg_m<128>(a, st);
  return set_error(VMLX_E_UNSUPPORTED, "qgemv: bits=%d group_size=%d not supported", bits, gs);
}

}  // namespace vmlx
