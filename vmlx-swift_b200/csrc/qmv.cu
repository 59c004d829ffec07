// qmv.cu -- decode GEMV / skinny GEMM (M <= 32) for MLX affine-quantized weights.
//
// Computes y[tok, n] = sum_k x[tok, k] * (scale[n, k/g] * q[n, k] + bias[n, k/g])
// for the decode regime, replacing MLX's affine_qmv_fast / affine_qmv
// (Source/Cmlx/mlx-generated/metal/quantized.h:799-1025) and the gathered
// variants affine_gather_qmv(_fast) (:1875-1997) / sorted affine_gather_qmm_rhs
// (:2197-2391) for small runs.
//
// B200 design.  The op is HBM-bound (0.5625 B/weight at 4-bit g64 with bf16
// scale+bias), so the kernel is built to keep HBM busy:
//  * Persistent CTAs.  A work item is a tile of 64 output rows (x one expert
//    in the gathered modes).  The K range is split over a thread-block
//    cluster of C CTAs (1..8) whose partial tiles are added through
//    distributed shared memory: no global scratch, no atomics.
//  * Warp 4 is the producer: one TMA instruction (cp.async.bulk.tensor.2d,
//    128-byte swizzle, no multicast) moves a 64-row x 128-byte stage of packed
//    weights into a ring of shared-memory stages completing on mbarriers, and
//    two more move the item's bf16 scales and biases.  It runs ahead across
//    item boundaries, so HBM stays busy while consumers finish a tile.
//  * Warps 0-3 are consumers, 16 rows each (one m16 tile of mma.m16n8k16).
//    They unpack codes from shared memory into bf16 A fragments holding q
//    exactly (4-bit: prmt with a 0x43 exponent byte gives 128+q; 8-bit: the
//    2^23 float trick) and form sum(x*q) per group with exact products in
//    fp32.  x was staged once per CTA in fragment order together with its
//    per-group sums, so each group is folded as scale*sum(x*q) + bias*sum(x),
//    the factorisation of MLX's qdot (quantized.h:209-316); no rounded bf16
//    weight is ever formed.
//  * A dot product does not care about the order of k: the nibbles are used
//    in the order the unpack produces them and x is permuted to match.
//  * Tokens are the MMA's N dimension (8 per tile, up to 4 tiles = 32 rows).
// Each row's result does not depend on M (batch invariance, as the
// reference's QuantizedSmallMScalingBenchTests.swift:110-127 requires).
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

#include "kernels.cuh"
#include "sm100_util.cuh"
#include "tmap.cuh"
#include "qmv_util.cuh"

namespace vmlx {

namespace cg = cooperative_groups;

constexpr int QMV_CWARPS = 4;                 // consumer warps
constexpr int QMV_ROWS = 16 * QMV_CWARPS;     // rows per work item
constexpr int QMV_THREADS = 32 * (QMV_CWARPS + 1);
constexpr int QMV_STAGES = 6;
constexpr int QMV_MAX_CLUSTER = 8;
#ifndef QMV_MAX_PER_SM
#define QMV_MAX_PER_SM 3  // cap on resident CTAs per SM assumed by the cost model
#endif
#ifndef QMV_CC_MAX_TOKENS
#define QMV_CC_MAX_TOKENS 4  // token rows up to which 4-bit GEMVs use the CUDA-core consumer
#endif


template <int BITS, int GS>
struct QT {
  static constexpr int WPL = GS * BITS / 128;   // words per lane per row per group
  static constexpr int VPL = GS / 4;            // k values per lane per group
  static constexpr int GB = GS * BITS / 8;      // bytes per row per group
  static constexpr int SG = 128 / GB;           // groups per stage: one 128-byte swizzle span per row
  static constexpr int FB = BITS == 4 ? 16 : 8; // x fragment bytes per lane per word
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
    tok += b_or_r0;  // 0, or a loopback rank's first row
    xr = p.x + tok * (p.x_swiglu ? 2 * p.K : p.K);
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

// Store one output element, with the optional fused residual add.  Under row-parallel
// TP the bf16 partial goes to slot [parity][tp_rank] of every rank instead, as one
// low-latency word {bf16 bits, epoch} per element (P2P 8-byte stores).
// (trank: this CTA's rank; ybias: offset of that rank's rows in a loopback group's y).
template <bool TP>
__device__ __forceinline__ void store_y(const QmvArgs& p, bf16* yr, int64_t col, float v, uint32_t tp_e,
                                        int trank, int64_t ybias) {
  if constexpr (TP) {
    const uint32_t hv = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
    const size_t off = p.tp_slots_off + ((size_t)(tp_e & 1) * p.tp_world + trank) * p.tp_slot_bytes +
                       (size_t)((yr - p.y) - ybias + col) * sizeof(uint64_t);
    for (int r = 0; r < p.tp_world; r++) st_ll(reinterpret_cast<uint64_t*>(p.tp_buf[r] + off), hv, tp_e);
    return;
  }
  if (p.residual) {
    const bf16* rr = p.residual + (yr - p.y);
    const float s = __bfloat162float(__float2bfloat16_rn(v));
    yr[col] = __float2bfloat16_rn(__bfloat162float(rr[col]) + s);
  } else {
    yr[col] = __float2bfloat16_rn(v);
  }
}

// Shared-memory plan of one CTA; sizes depend on the K-slice (ks groups) and
// on the number of token rows staged at once (tok).  The ring is 1024-byte
// aligned (the 128-byte TMA swizzle atom).
struct QmvPlan {
  int ks, tok, tokx, ws, wpl, fb;
  size_t o_ring, o_sc, o_bar, o_xfrag, o_xsum, o_red, total;
  // cc: CUDA-core consumer (4-bit, <= 4 tokens): x staged as fp32 per 16-byte
  // weight chunk (32 values) with per-chunk sums instead of MMA fragments.
  __host__ __device__ void init(int bits, int gs, int ks_, int tok_, bool cc = false) {
    ks = ks_;
    tok = tok_;
    tokx = (tok + 7) / 8 * 8;  // xsum row stride: whole 8-token MMA tiles
    ws = ((ks + 7) + 7) / 8 * 8;  // scale window (elements), 16-byte multiple
    wpl = gs * bits / 128;
    fb = bits == 4 ? 16 : 8;
    o_ring = 0;
    o_sc = o_ring + (size_t)QMV_STAGES * QMV_ROWS * 128;
    o_bar = o_sc + (size_t)2 * 2 * QMV_ROWS * ws * 2;
    o_xfrag = o_bar + (2 * QMV_STAGES + 4) * sizeof(uint64_t);
    const size_t nchunks = (size_t)ks * (gs * bits / 8) / 16;
    o_xsum = o_xfrag + (cc ? nchunks * (tok * 32 + 4) * 4 : (size_t)ks * wpl * tok * 4 * fb);
    o_red = o_xsum + (((cc ? nchunks * tok : (size_t)ks * tokx) * 4 + 15) / 16) * 16;
    total = o_red + (size_t)2 * QMV_ROWS * tok * 4 + 1024;  // + alignment slack
  }
};

// Work item -> (row tile, z) and the token set / expert of z.
struct QmvItem {
  int64_t n0, base, ntok, e;  // e: expert (0 for dense)
  bool zero_rows;
};

// lr: a loopback rank (0 otherwise), whose rows and weight shard the dense item uses.
__device__ __forceinline__ QmvItem qmv_item(const QmvArgs& p, int mode, int64_t item, int64_t rowtiles, int lr = 0) {
  QmvItem it;
  const int64_t z = item / rowtiles;
  it.n0 = (item - z * rowtiles) * QMV_ROWS;
  it.base = (int64_t)lr * p.M;
  it.ntok = p.M;
  it.e = lr;
  it.zero_rows = false;
  if (mode == QMV_GATHER) {
    it.base = z;
    it.e = p.rhs ? (int64_t)p.rhs[z] : z * p.n_experts / p.batch;
    if (it.e >= p.n_experts) { it.zero_rows = true; it.e = 0; }
  } else if (mode == QMV_SORTED) {
    it.e = z;
    const int64_t lo = lower_bound_u32(p.rhs, p.batch, (uint32_t)z);
    const int64_t hi = lower_bound_u32(p.rhs, p.batch, (uint32_t)z + 1);
    it.base = lo * p.M;
    it.ntok = (hi - lo) * p.M;
  }
  return it;
}

// Byte offset of (row, byte o) inside a 128B-swizzled [rows][128] TMA tile:
// 16-byte chunk index XOR (row mod 8).
__device__ __forceinline__ uint32_t swz128(int r, int o) {
  return (uint32_t)(r * 128 + ((((o >> 4) ^ (r & 7))) << 4) + (o & 15));
}

template <int BITS, int GS, int NT, bool CC, bool TP>
__global__ void __launch_bounds__(QMV_THREADS, 1)
qmv_kernel(QmvArgs p, const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tms,
           const __grid_constant__ CUtensorMap tmb, int sc_tma, int mode, int Ks, int C, int TOKA,
           int64_t rowtiles, int64_t n_items) {
  using T = QT<BITS, GS>;
  constexpr int WPL = T::WPL, VPL = T::VPL, GB = T::GB, SG = T::SG, FB = T::FB;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  static_assert(!CC || BITS == 4, "the CUDA-core consumer is 4-bit only");
  QmvPlan L;
  L.init(BITS, GS, Ks, TOKA, CC);
  const int WS = L.ws;
  constexpr int CPS = 128 / 16;     // 16-byte chunks per row per stage
  constexpr int CPG = GB / 16;      // chunks per group
  const int XST = TOKA * 32 + 4;    // fp32 x stride per chunk (CUDA-core path), padded

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // TP ranks: trank = this CTA's rank in the group; lr = the same for a loopback group
  // (all ranks in one grid, rank = blockIdx.y), else 0.
  const int lr = (TP && p.tp_loop) ? (int)blockIdx.y : 0;
  const int trank = TP ? (p.tp_loop ? lr : p.tp_rank) : 0;
  const int64_t ybias = (int64_t)lr * p.M * p.N;
  const int rank = (int)(blockIdx.x % C);  // K-slice == rank in the cluster (cluster dims (C,1,1))
  const int64_t cluster_id = blockIdx.x / C, n_clusters = gridDim.x / C;
  const int64_t KG = p.K / GS;
  const int64_t gs0 = (int64_t)rank * Ks;
  const int nG = (int)(gs0 >= KG ? 0 : (KG - gs0 < Ks ? KG - gs0 : Ks));
  const int nst = (nG + SG - 1) / SG;
  const int xs0 = (int)(gs0 & ~(int64_t)7);  // scale window start (16-byte aligned column)
  const int soff = (int)(gs0 - xs0);

  uint8_t* ring = smem + L.o_ring;
  bf16* scb = reinterpret_cast<bf16*>(smem + L.o_sc);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.o_bar);
  uint64_t* empty = full + QMV_STAGES;
  uint64_t* scfull = empty + QMV_STAGES;
  uint64_t* scempty = scfull + 2;
  uint8_t* xfrag = smem + L.o_xfrag;
  float* xfrag_f = reinterpret_cast<float*>(xfrag);
  __shared__ float xinv[32];  // fused RMSNorm: 1 / rms per staged token
  float* xsum = reinterpret_cast<float*>(smem + L.o_xsum);
  const int TOKX = L.tokx;
  float* red = reinterpret_cast<float*>(smem + L.o_red);

  if (tid == 0) {
    for (int s = 0; s < QMV_STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], QMV_CWARPS);
    }
    for (int s = 0; s < 2; s++) {
      mbar_init(&scfull[s], 1);
      mbar_init(&scempty[s], QMV_CWARPS);
    }
    fence_mbar_init();
  }
  if (warp == QMV_CWARPS && lane == 0) {
    tma_prefetch_desc(&tmw);
    if (sc_tma) { tma_prefetch_desc(&tms); tma_prefetch_desc(&tmb); }
  }
  __syncthreads();
  // Let the next kernel in the stream launch now (when launch overlap is on):
  // its producer may start streaming its own weights while this grid drains.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  bool ok = true;
  uint32_t it_stage = 0, ic = 0;
  // Item order: round-robin over clusters for dense calls (x is staged once per CTA); a
  // contiguous block per cluster in the gather modes, so that consecutive items share an
  // expert's (or batch element's) token rows and x is staged once per token set, not per item.
  const bool blocked = mode != QMV_DENSE;
  const int64_t it_lo = blocked ? cluster_id * n_items / n_clusters : cluster_id;
  const int64_t it_hi = blocked ? (cluster_id + 1) * n_items / n_clusters : n_items;
  const int64_t it_step = blocked ? 1 : n_clusters;

  if (warp == QMV_CWARPS) {
    // ======================= producer warp (lane 0 issues) =======================
    // In the gathered modes the work items depend on the expert indices, which the
    // previous kernel may still be writing: wait for it before the first item (the
    // dense mode streams static weights ahead of the wait).
    if (mode != QMV_DENSE) asm volatile("griddepcontrol.wait;" ::: "memory");
    bool pend = false;
    for (int64_t item = it_lo; item < it_hi; item += it_step) {
      const QmvItem I = qmv_item(p, mode, item, rowtiles, lr);
      if (I.ntok == 0) continue;
      const int ybase = (int)(I.e * p.N + I.n0);  // row coordinate in the [E*N, .] maps
      if (!I.zero_rows) {
        const int slot = ic & 1;
        const uint32_t use = ic >> 1;
        ic++;
        if (sc_tma && lane == 0) {
          if (use > 0) ok &= mbar_wait(&scempty[slot], (use - 1) & 1);
          mbar_arrive_expect_tx(&scfull[slot], 2u * QMV_ROWS * WS * 2);
          tma_load_2d(scb + ((size_t)slot * 2 + 0) * QMV_ROWS * WS, &tms, xs0, ybase, &scfull[slot]);
          tma_load_2d(scb + ((size_t)slot * 2 + 1) * QMV_ROWS * WS, &tmb, xs0, ybase, &scfull[slot]);
        }
      }
      for (int64_t chunk = 0; chunk < I.ntok; chunk += TOKA) {
        if (!I.zero_rows && lane == 0) {
          for (int st = 0; st < nst; st++, it_stage++) {
            const int slot = it_stage % QMV_STAGES;
            const uint32_t use = it_stage / QMV_STAGES;
            if (use > 0) ok &= mbar_wait(&empty[slot], (use - 1) & 1);
            mbar_arrive_expect_tx(&full[slot], QMV_ROWS * 128);
            tma_load_2d(ring + (size_t)slot * QMV_ROWS * 128, &tmw, (int)((gs0 + st * SG) * GB), ybase,
                        &full[slot]);
          }
        }
        __syncwarp();
        if (C > 1) {  // one cluster-barrier phase per output tile; wait lazily to run ahead
          if (pend) cluster_wait();
          cluster_arrive();
          pend = true;
        }
      }
    }
    if (C > 1) {
      if (pend) cluster_wait();
      cluster_arrive();
      cluster_wait();
    }
  } else {
    // ======================= consumer warps =======================
    const int gq = lane >> 2, c = lane & 3;
    const int r0 = warp * 16 + gq, r1 = r0 + 8;
    const int crow_lo = rank * QMV_ROWS / C, crow_hi = (rank + 1) * QMV_ROWS / C;
    uint32_t red_count = 0;
    bool x_staged = false;
    // x and y may be produced / consumed by the previous kernel: wait for it
    // (a no-op unless this grid was launched with programmatic overlap).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // Row-parallel TP: this call's epoch (advanced by the grid's last CTA) picks the slot parity.
    __shared__ uint32_t s_tp_e;
    if constexpr (TP) {
      if (tid == 0) s_tp_e = *reinterpret_cast<const uint32_t*>(p.tp_buf[trank] + p.tp_epoch_off) + 1;
      named_bar_sync(1, 32 * QMV_CWARPS);
    }
    const uint32_t tp_e = TP ? s_tp_e : 0u;
    int64_t staged_z = -1;  // token set (item / rowtiles) whose x is staged
    for (int64_t item = it_lo; item < it_hi; item += it_step) {
      const QmvItem I = qmv_item(p, mode, item, rowtiles, lr);
      if (I.ntok == 0) continue;
      int slot_sc = 0;
      if (!I.zero_rows) {
        slot_sc = ic & 1;
        if (sc_tma) {
          ok &= mbar_wait(&scfull[slot_sc], (ic >> 1) & 1);
        } else {
          // scales whose rows are not 16-byte strided: plain loads into the same layout
          named_bar_sync(1, 32 * QMV_CWARPS);
          for (int i = tid; i < 2 * QMV_ROWS * nG; i += 32 * QMV_CWARPS) {
            const int kind = i / (QMV_ROWS * nG), rem = i - kind * QMV_ROWS * nG;
            const int r = rem / nG, gl = rem - r * nG;
            const int64_t row = I.e * p.N + (I.n0 + r < p.N ? I.n0 + r : p.N - 1);
            scb[(((size_t)slot_sc * 2 + kind) * QMV_ROWS + r) * WS + soff + gl] =
                (kind ? p.biases : p.scales)[row * KG + gs0 + gl];
          }
          named_bar_sync(1, 32 * QMV_CWARPS);
        }
        ic++;
      }
      // (scale, bias') in fp32 per (row, group); bias' folds the +128 of 4-bit codes
      // this lane's two rows of the item's bf16 scale / bias windows
      const bf16* sbase = scb + (size_t)slot_sc * 2 * QMV_ROWS * WS;
      const bf16* s0p = sbase + r0 * WS + soff;
      const bf16* s1p = sbase + r1 * WS + soff;
      const bf16* b0p = sbase + (QMV_ROWS + r0) * WS + soff;
      const bf16* b1p = sbase + (QMV_ROWS + r1) * WS + soff;

      for (int64_t chunk = 0; chunk < I.ntok; chunk += TOKA) {
        const int ntok = (int)((I.ntok - chunk) < TOKA ? (I.ntok - chunk) : TOKA);
        const int64_t z = item / rowtiles;
        if (!x_staged || I.ntok > TOKA || (mode != QMV_DENSE && z != staged_z)) {
          staged_z = z;
          // stage x of this chunk in fragment order, with per-group sums
          named_bar_sync(1, 32 * QMV_CWARPS);  // nobody still reads the previous chunk
          if (p.norm_w) {
            // fused RMSNorm: 1 / rms of each token's full row (warp w takes tokens w, w+4, ...)
            for (int tok = warp; tok < ntok; tok += QMV_CWARPS) {
              const bf16* xr;
              bf16* yr_unused;
              token_rows(p, mode, I.base, chunk + tok, xr, yr_unused);
              float ss = 0.f;
              for (int64_t k = lane * 8; k < p.K; k += 256) {
                const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                  const float2 f = __bfloat1622float2(u32_as_bf162(u[j]));
                  ss = fmaf(f.x, f.x, ss);
                  ss = fmaf(f.y, f.y, ss);
                }
              }
              for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
              if (lane == 0) xinv[tok] = rsqrtf(ss / (float)p.K + p.eps);
            }
            named_bar_sync(1, 32 * QMV_CWARPS);
          }
          if constexpr (CC) {
            // fp32 x, 32 values per 16-byte weight chunk, plus the chunk's sum
            const int nch = nG * CPG;
            for (int it = tid; it < TOKA * nch; it += 32 * QMV_CWARPS) {
              const int ci = it / TOKA, tok = it - ci * TOKA;
              const bf16* xrow = nullptr;
              if (tok < ntok && !I.zero_rows) {
                bf16* yr_unused;
                token_rows(p, mode, I.base, chunk + tok, xrow, yr_unused);
                xrow += gs0 * GS + ci * 32;
              }
              float* dst = xfrag_f + (size_t)ci * XST + tok * 32;
              float sum = 0.f;
#pragma unroll
              for (int q = 0; q < 4; q++) {
                uint4 v = make_uint4(0, 0, 0, 0);
                if (xrow) v = load_x8(p, xrow + q * 8);
                if (xrow && p.norm_w) v = norm8(v, xinv[tok], p.norm_w + gs0 * GS + ci * 32 + q * 8);
                const float2 a = __bfloat1622float2(u32_as_bf162(v.x)), b2 = __bfloat1622float2(u32_as_bf162(v.y));
                const float2 c2 = __bfloat1622float2(u32_as_bf162(v.z)), d2 = __bfloat1622float2(u32_as_bf162(v.w));
                reinterpret_cast<float4*>(dst + q * 8)[0] = make_float4(a.x, a.y, b2.x, b2.y);
                reinterpret_cast<float4*>(dst + q * 8)[1] = make_float4(c2.x, c2.y, d2.x, d2.y);
                sum += ((a.x + a.y) + (b2.x + b2.y)) + ((c2.x + c2.y) + (d2.x + d2.y));
              }
              xsum[ci * TOKA + tok] = sum;
            }
          } else
          for (int it = tid; it < TOKX * nG; it += 32 * QMV_CWARPS) {
            const int gl = it / TOKX, tok = it - gl * TOKX;
            if (tok >= TOKA) { xsum[gl * TOKX + tok] = 0.f; continue; }
            const bf16* xrow = nullptr;
            if (tok < ntok && !I.zero_rows) {
              bf16* yr_unused;
              token_rows(p, mode, I.base, chunk + tok, xrow, yr_unused);
              xrow += (gs0 + gl) * GS;
            }
            float sum = 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
#pragma unroll
              for (int wi = 0; wi < WPL; wi++) {
                uint8_t* dst = xfrag + ((((size_t)gl * WPL + wi) * TOKA + tok) * 4 + cc) * FB;
                if constexpr (BITS == 4) {
                  uint4 v = make_uint4(0, 0, 0, 0);
                  if (xrow) v = load_x8(p, xrow + cc * VPL + wi * 8);
                  if (xrow && p.norm_w) v = norm8(v, xinv[tok], p.norm_w + (gs0 + gl) * GS + cc * VPL + wi * 8);
                  uint4 f;
                  f.x = prmt(v.x, v.y, 0x5410);  // (x0, x2)
                  f.y = prmt(v.z, v.w, 0x5410);  // (x4, x6)
                  f.z = prmt(v.x, v.y, 0x7632);  // (x1, x3)
                  f.w = prmt(v.z, v.w, 0x7632);  // (x5, x7)
                  *reinterpret_cast<uint4*>(dst) = f;
                  const float2 a = __bfloat1622float2(u32_as_bf162(v.x)), b2 = __bfloat1622float2(u32_as_bf162(v.y));
                  const float2 c2 = __bfloat1622float2(u32_as_bf162(v.z)), d2 = __bfloat1622float2(u32_as_bf162(v.w));
                  sum += ((a.x + a.y) + (b2.x + b2.y)) + ((c2.x + c2.y) + (d2.x + d2.y));
                } else {
                  uint2 v = make_uint2(0, 0);
                  if (xrow) v = load_x4(p, xrow + cc * VPL + wi * 4);
                  if (xrow && p.norm_w) v = norm4(v, xinv[tok], p.norm_w + (gs0 + gl) * GS + cc * VPL + wi * 4);
                  *reinterpret_cast<uint2*>(dst) = v;
                  const float2 a = __bfloat1622float2(u32_as_bf162(v.x)), b2 = __bfloat1622float2(u32_as_bf162(v.y));
                  sum += (a.x + a.y) + (b2.x + b2.y);
                }
              }
            }
            xsum[gl * TOKX + tok] = (tok < ntok) ? sum : 0.f;
          }
          named_bar_sync(1, 32 * QMV_CWARPS);
          x_staged = true;
        }

        float* rb = red + (size_t)(red_count & 1) * QMV_ROWS * TOKA;
        if constexpr (!CC) {
        float acc[NT][4];
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
        bool tok_ok[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) tok_ok[t] = t * 8 + gq < ntok;
        if (!I.zero_rows) {
          for (int st = 0; st < nst; st++, it_stage++) {
            const int slot = it_stage % QMV_STAGES;
            ok &= mbar_wait(&full[slot], (it_stage / QMV_STAGES) & 1);
            const int ng = (nG - st * SG) < SG ? (nG - st * SG) : SG;
            const uint8_t* stg0 = ring + (size_t)slot * QMV_ROWS * 128 + r0 * 128;
            const uint8_t* stg1 = stg0 + 8 * 128;  // row r1 = r0 + 8 has the same swizzle phase
            const uint8_t* xst = xfrag + ((st * SG * WPL) * TOKA * 4 + gq * 4 + c) * FB;
#pragma unroll
            for (int gi = 0; gi < SG; gi++) {
              if (gi < ng) {
                const int gl = st * SG + gi;
                uint32_t wv0[WPL], wv1[WPL];
#pragma unroll
                for (int q = 0; q < WPL; q += (WPL < 4 ? WPL : 4)) {
                  const int o = gi * GB + c * WPL * 4 + q * 4;
                  const int so = ((((o >> 4) ^ gq)) << 4) + (o & 15);  // 128B swizzle: chunk ^ (row & 7)
                  if constexpr (WPL == 1) {
                    wv0[q] = *reinterpret_cast<const uint32_t*>(stg0 + so);
                    wv1[q] = *reinterpret_cast<const uint32_t*>(stg1 + so);
                  } else if constexpr (WPL == 2) {
                    const uint2 a0 = *reinterpret_cast<const uint2*>(stg0 + so);
                    const uint2 a1 = *reinterpret_cast<const uint2*>(stg1 + so);
                    wv0[q] = a0.x; wv0[q + 1] = a0.y; wv1[q] = a1.x; wv1[q + 1] = a1.y;
                  } else {
                    const uint4 a0 = *reinterpret_cast<const uint4*>(stg0 + so);
                    const uint4 a1 = *reinterpret_cast<const uint4*>(stg1 + so);
                    wv0[q] = a0.x; wv0[q + 1] = a0.y; wv0[q + 2] = a0.z; wv0[q + 3] = a0.w;
                    wv1[q] = a1.x; wv1[q + 1] = a1.y; wv1[q + 2] = a1.z; wv1[q + 3] = a1.w;
                  }
                }
                float ag[NT][4];
#pragma unroll
                for (int t = 0; t < NT; t++) ag[t][0] = ag[t][1] = ag[t][2] = ag[t][3] = 0.f;
#pragma unroll
                for (int wi = 0; wi < WPL; wi++) {
                  const uint8_t* xf = xst + ((gi * WPL + wi) * TOKA * 4) * FB;
                  if constexpr (BITS == 4) {
                    uint32_t p0[4], p1[4];
                    unpack4(wv0[wi], p0);
                    unpack4(wv1[wi], p1);
                    const uint32_t a0[4] = {p0[0], p1[0], p0[1], p1[1]};
                    const uint32_t a1[4] = {p0[2], p1[2], p0[3], p1[3]};
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                      uint4 xv = make_uint4(0, 0, 0, 0);
                      if (tok_ok[t]) xv = *reinterpret_cast<const uint4*>(xf + t * 32 * FB);
                      mma_bf16_16816(ag[t], a0, xv.x, xv.y);
                      mma_bf16_16816(ag[t], a1, xv.z, xv.w);
                    }
                  } else {
                    uint32_t p0[2], p1[2];
                    unpack8(wv0[wi], p0);
                    unpack8(wv1[wi], p1);
                    const uint32_t a[4] = {p0[0], p1[0], p0[1], p1[1]};
#pragma unroll
                    for (int t = 0; t < NT; t++) {
                      uint2 xv = make_uint2(0, 0);
                      if (tok_ok[t]) xv = *reinterpret_cast<const uint2*>(xf + t * 32 * FB);
                      mma_bf16_16816(ag[t], a, xv.x, xv.y);
                    }
                  }
                }
                float2 sb0, sb1;  // (scale, bias'): bias' folds the +128 of 4-bit codes
                sb0.x = __bfloat162float(s0p[gl]);
                sb1.x = __bfloat162float(s1p[gl]);
                sb0.y = BITS == 4 ? fmaf(-128.f, sb0.x, __bfloat162float(b0p[gl])) : __bfloat162float(b0p[gl]);
                sb1.y = BITS == 4 ? fmaf(-128.f, sb1.x, __bfloat162float(b1p[gl])) : __bfloat162float(b1p[gl]);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                  const float2 xs = *reinterpret_cast<const float2*>(xsum + gl * TOKX + t * 8 + 2 * c);
                  acc[t][0] = fmaf(sb0.x, ag[t][0], fmaf(sb0.y, xs.x, acc[t][0]));
                  acc[t][1] = fmaf(sb0.x, ag[t][1], fmaf(sb0.y, xs.y, acc[t][1]));
                  acc[t][2] = fmaf(sb1.x, ag[t][2], fmaf(sb1.y, xs.x, acc[t][2]));
                  acc[t][3] = fmaf(sb1.x, ag[t][3], fmaf(sb1.y, xs.y, acc[t][3]));
                }
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
          }
        }
        // ---- output tile ----
        if (C == 1) {
#pragma unroll
          for (int t = 0; t < NT; t++) {
            const int ta = t * 8 + 2 * c;
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const int tok = ta + (j & 1);
              const int64_t row = I.n0 + (j < 2 ? r0 : r1);
              if (tok < ntok && row < p.N) {
                const bf16* xr_unused;
                bf16* yr;
                token_rows(p, mode, I.base, chunk + tok, xr_unused, yr);
                store_y<TP>(p, yr, row, acc[t][j], tp_e, trank, ybias);
              }
            }
          }
        } else {
#pragma unroll
          for (int t = 0; t < NT; t++) {
            const int ta = t * 8 + 2 * c;
            if (ta < TOKA) { rb[r0 * TOKA + ta] = acc[t][0]; rb[r1 * TOKA + ta] = acc[t][2]; }
            if (ta + 1 < TOKA) { rb[r0 * TOKA + ta + 1] = acc[t][1]; rb[r1 * TOKA + ta + 1] = acc[t][3]; }
          }
        }
        } else {
          // ---------- CUDA-core consumer (4-bit, <= 4 tokens) ----------
          // lane = (rs, kc): 16-byte chunk kc of each stage row, rows rs + 4j of the warp's 16
          const int rs = lane >> 3, kc = lane & 7;
          float res[4][CC ? NT : 1];
#pragma unroll
          for (int j = 0; j < 4; j++)
#pragma unroll
            for (int t = 0; t < NT; t++) res[j][t] = 0.f;
          if (!I.zero_rows) {
            for (int st = 0; st < nst; st++, it_stage++) {
              const int slot = it_stage % QMV_STAGES;
              ok &= mbar_wait(&full[slot], (it_stage / QMV_STAGES) & 1);
              const int ng = (nG - st * SG) < SG ? (nG - st * SG) : SG;
              if (kc < ng * CPG) {
                const int ci = st * CPS + kc;  // chunk index within the slice
                const int gl = ci / CPG;
                const uint8_t* stg = ring + (size_t)slot * QMV_ROWS * 128;
                uint4 wv[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                  const int row = warp * 16 + rs + 4 * j;
                  wv[j] = *reinterpret_cast<const uint4*>(stg + row * 128 + ((kc ^ (row & 7)) << 4));
                }
                unsigned long long sacc[4][NT];
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                  for (int t = 0; t < NT; t++) sacc[j][t] = 0ull;
                const float* xc = xfrag_f + (size_t)ci * XST;
#pragma unroll
                for (int wi = 0; wi < 4; wi++) {
                  // x pairs (x[8wi+2i], x[8wi+2i+1]) for each token
                  unsigned long long xp[NT][4];
#pragma unroll
                  for (int t = 0; t < NT; t++) {
                    const float4 xa = *reinterpret_cast<const float4*>(xc + t * 32 + wi * 8);
                    const float4 xb = *reinterpret_cast<const float4*>(xc + t * 32 + wi * 8 + 4);
                    xp[t][0] = pack_f2(xa.x, xa.y);
                    xp[t][1] = pack_f2(xa.z, xa.w);
                    xp[t][2] = pack_f2(xb.x, xb.y);
                    xp[t][3] = pack_f2(xb.z, xb.w);
                  }
#pragma unroll
                  for (int j = 0; j < 4; j++) {
                    const uint32_t w = wi == 0 ? wv[j].x : wi == 1 ? wv[j].y : wi == 2 ? wv[j].z : wv[j].w;
                    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                      // (128 + q) as exact fp32: bytes [0, 0, q, 0x43]
                      const uint32_t fl = prmt(lo, 0x43000000u, 0x7044u | (i << 8));
                      const uint32_t fh = prmt(hi, 0x43000000u, 0x7044u | (i << 8));
                      const unsigned long long wp = pack_u2(fl, fh);  // nibbles (2i, 2i+1)
#pragma unroll
                      for (int t = 0; t < NT; t++) ffma2(sacc[j][t], wp, xp[t][i]);
                    }
                  }
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                  const int row = warp * 16 + rs + 4 * j;
                  const float sv = __bfloat162float(sbase[row * WS + soff + gl]);
                  const float bv = fmaf(-128.f, sv, __bfloat162float(sbase[(QMV_ROWS + row) * WS + soff + gl]));
#pragma unroll
                  for (int t = 0; t < NT; t++) {
                    const float2 sp = unpack_f2(sacc[j][t]);
                    res[j][t] = fmaf(sv, sp.x + sp.y, fmaf(bv, xsum[ci * TOKA + t], res[j][t]));
                  }
                }
              }
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[slot]);
            }
          }
          // sum the 8 chunk lanes of each row group
#pragma unroll
          for (int j = 0; j < 4; j++)
#pragma unroll
            for (int t = 0; t < NT; t++) {
              float v = res[j][t];
              v += __shfl_xor_sync(0xffffffffu, v, 1);
              v += __shfl_xor_sync(0xffffffffu, v, 2);
              v += __shfl_xor_sync(0xffffffffu, v, 4);
              res[j][t] = v;
            }
          if (kc == 0) {
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const int r = warp * 16 + rs + 4 * j;
#pragma unroll
              for (int t = 0; t < NT; t++) {
                if (t >= TOKA) continue;
                if (C == 1) {
                  if (t < ntok && I.n0 + r < p.N) {
                    const bf16* xr_unused;
                    bf16* yr;
                    token_rows(p, mode, I.base, chunk + t, xr_unused, yr);
                    store_y<TP>(p, yr, I.n0 + r, res[j][t], tp_e, trank, ybias);
                  }
                } else {
                  rb[r * TOKA + t] = res[j][t];
                }
              }
            }
          }
        }
        if (C > 1) {
          cluster_arrive();
          cluster_wait();
          cg::cluster_group cluster = cg::this_cluster();
          for (int i = tid; i < (crow_hi - crow_lo) * ntok; i += 32 * QMV_CWARPS) {
            const int r = crow_lo + i / ntok, tok = i % ntok;
            float s = 0.f;
            for (int q = 0; q < C; q++) s += cluster.map_shared_rank(rb, q)[r * TOKA + tok];
            if (I.n0 + r < p.N) {
              const bf16* xr_unused;
              bf16* yr;
              token_rows(p, mode, I.base, chunk + tok, xr_unused, yr);
              store_y<TP>(p, yr, I.n0 + r, s, tp_e, trank, ybias);
            }
          }
          red_count++;
        }
      }
      if (!I.zero_rows && sc_tma) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&scempty[slot_sc]);
      }
    }
    if constexpr (TP) {
      // ---- row-parallel all-reduce: the rows this CTA computed, from every rank, in rank order ----
      // (each word is polled until it carries this call's epoch: no separate flags or fences)
      const uint64_t deadline = globaltimer() + p.tp_timeout_ns;
      const int rlo = C > 1 ? crow_lo : 0, rhi = C > 1 ? crow_hi : QMV_ROWS, nr = rhi - rlo;
      const uint64_t* slots = reinterpret_cast<const uint64_t*>(p.tp_buf[trank] + p.tp_slots_off +
                                                                (size_t)(tp_e & 1) * p.tp_world * p.tp_slot_bytes);
      const size_t rstride = p.tp_slot_bytes / sizeof(uint64_t);
      bool tp_ok = true;
      for (int64_t item = cluster_id; item < n_items && tp_ok; item += n_clusters) {
        const QmvItem I = qmv_item(p, mode, item, rowtiles, lr);
        for (int64_t i = tid; i < (int64_t)nr * I.ntok && tp_ok; i += 32 * QMV_CWARPS) {
          const int64_t row = I.n0 + rlo + i % nr, tok = i / nr;
          if (row >= p.N) continue;
          const int64_t idx = tok * p.N + row;
          float sum;  // rank order: identical on every rank
          tp_ok = wait_ll_sum<QMV_TP_MAX_WORLD>(slots + idx, rstride, p.tp_world, tp_e, deadline, sum);
          if (!tp_ok) break;
          const bf16 sb = __float2bfloat16_rn(sum);
          const int64_t yi = idx + ybias;
          p.y[yi] = p.residual ? __float2bfloat16_rn(__bfloat162float(p.residual[yi]) + __bfloat162float(sb)) : sb;
        }
      }
      if (!tp_ok && p.tp_status) atomicExch(p.tp_status, VMLX_E_PEER_TIMEOUT);
      named_bar_sync(1, 32 * QMV_CWARPS);
      if (tid == 0) {  // the grid's last CTA advances the epoch for the next call
        uint32_t* ep = reinterpret_cast<uint32_t*>(p.tp_buf[trank] + p.tp_epoch_off);
        __threadfence();
        if (atomicAdd(ep + 1, 1u) == gridDim.x - 1) {
          ep[1] = 0;
          ep[0] = tp_e;
          __threadfence();
        }
      }
    }
    if (C > 1) {  // keep this CTA's shared memory alive until every peer has read it
      cluster_arrive();
      cluster_wait();
    }
  }
  if (!ok && p.status) atomicExch(p.status, VMLX_E_STATE);
}

// The kernel instance a launch of launch_qmv_bg will use (its template arguments do not
// depend on the cluster size), for occupancy queries.
template <int BITS, int GS, int NT, bool CC>
static const void* qmv_fn(bool tp) {
  return tp ? (const void*)qmv_kernel<BITS, GS, NT, CC, true> : (const void*)qmv_kernel<BITS, GS, NT, CC, false>;
}
template <int BITS, int GS>
static const void* qmv_kernel_for(int toka, bool cc, bool tp) {
  if constexpr (BITS == 4) {
    if (cc) {
      switch (toka) {
        case 1: return qmv_fn<BITS, GS, 1, true>(tp);
        case 2: return qmv_fn<BITS, GS, 2, true>(tp);
        case 3: return qmv_fn<BITS, GS, 3, true>(tp);
        default: return qmv_fn<BITS, GS, 4, true>(tp);
      }
    }
  }
  switch ((toka + 7) / 8) {
    case 1: return qmv_fn<BITS, GS, 1, false>(tp);
    case 2: return qmv_fn<BITS, GS, 2, false>(tp);
    case 3: return qmv_fn<BITS, GS, 3, false>(tp);
    default: return qmv_fn<BITS, GS, 4, false>(tp);
  }
}

// Clusters of C CTAs (with `smem` dynamic shared memory) that can be resident at once: the
// GPCs must hold whole clusters, so e.g. 7-CTA clusters leave SMs of every GPC idle.  Cached.
static int qmv_resident_clusters(const void* fn, int C, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(fn, C, smem, dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (ensure_max_dynamic_smem(fn, 226 * 1024)) return 0;
  cudaLaunchConfig_t q = {};
  q.gridDim = dim3((unsigned)C, 1, 1);
  q.blockDim = dim3(QMV_THREADS);
  q.dynamicSmemBytes = smem;
  cudaLaunchAttribute ca;
  ca.id = cudaLaunchAttributeClusterDimension;
  ca.val.clusterDim.x = (unsigned)C;
  ca.val.clusterDim.y = 1;
  ca.val.clusterDim.z = 1;
  q.attrs = &ca;
  q.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fn, &q) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

template <int BITS, int GS, int NT, bool CC, bool TP>
static int launch_qmv_k(const QmvArgs& a, int mode, int64_t zcount, int ks, int C, int toka, cudaStream_t st) {
  auto kern = qmv_kernel<BITS, GS, NT, CC, TP>;
  QmvPlan L;
  L.init(BITS, GS, ks, toka, CC);
  {
    const int rc = ensure_max_dynamic_smem((const void*)kern, 226 * 1024);  // + static smem <= 227 KB
    if (rc) return rc;
  }
  const int64_t E = (mode == QMV_DENSE) ? (a.tp_loop ? a.tp_world : 1) : a.n_experts;
  const int64_t KG = a.K / GS;
  CUtensorMap tmw, tms, tmb;
  if (!make_tmap_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, (uint64_t)a.K * BITS / 8, (uint64_t)(E * a.N),
                    (uint64_t)a.K * BITS / 8, 128, QMV_ROWS, CU_TENSOR_MAP_SWIZZLE_128B))
    return VMLX_E_CUDA;
  int sc_tma = ((KG * 2) % 16 == 0) && L.ws <= 256 && aligned(a.scales, 16) && aligned(a.biases, 16);
  if (sc_tma) {
    if (!make_tmap_2d(&tms, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.scales, (uint64_t)KG, (uint64_t)(E * a.N),
                      (uint64_t)KG * 2, (uint32_t)L.ws, QMV_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_tmap_2d(&tmb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.biases, (uint64_t)KG, (uint64_t)(E * a.N),
                      (uint64_t)KG * 2, (uint32_t)L.ws, QMV_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE))
      return VMLX_E_CUDA;
  } else {
    tms = tmw;  // unused
    tmb = tmw;
  }
  const int64_t rowtiles = (a.N + QMV_ROWS - 1) / QMV_ROWS;
  const int64_t n_items = rowtiles * zcount;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, QMV_THREADS, L.total);
  if (e != cudaSuccess || per_sm < 1) per_sm = 1;
  if (per_sm > QMV_MAX_PER_SM) per_sm = QMV_MAX_PER_SM;
  // A loopback group runs every rank's grid in one launch: the ranks share the SMs.
  const int ranks = (TP && a.tp_loop) ? a.tp_world : 1;
  int64_t max_clusters = (int64_t)sm_count() * per_sm / C / ranks;
  {  // no more clusters than can be resident at once (the grid is persistent)
    const int res = qmv_resident_clusters((const void*)kern, C, L.total);
    if (res > 0 && max_clusters > res / ranks) max_clusters = res / ranks;
  }
  if (max_clusters < 1) max_clusters = 1;
  if (ranks > 1) {  // clusters of C CTAs that can be resident at once, shared by the ranks
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3((unsigned)C, 1, 1);
    q.blockDim = dim3(QMV_THREADS);
    q.dynamicSmemBytes = L.total;
    cudaLaunchAttribute ca;
    ca.id = cudaLaunchAttributeClusterDimension;
    ca.val.clusterDim.x = (unsigned)C;
    ca.val.clusterDim.y = 1;
    ca.val.clusterDim.z = 1;
    q.attrs = &ca;
    q.numAttrs = 1;
    int resident = 0;
    if (cudaOccupancyMaxActiveClusters(&resident, kern, &q) != cudaSuccess || resident < ranks) {
      cudaGetLastError();
      return set_error(VMLX_E_UNSUPPORTED, "tp loopback: %d ranks of %d-CTA clusters cannot be resident together",
                       ranks, C);
    }
    if (max_clusters > resident / ranks) max_clusters = resident / ranks;
  }
  const int64_t n_clusters = n_items < max_clusters ? n_items : max_clusters;

  if (a.tp_world > 1 && n_clusters * C > TP_FUSED_MAXC)
    return set_error(VMLX_E_UNSUPPORTED, "tp: fused grid of %lld CTAs exceeds %d", (long long)(n_clusters * C),
                     TP_FUSED_MAXC);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(n_clusters * C), (unsigned)ranks, 1);
  cfg.blockDim = dim3(QMV_THREADS);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = launch_overlap() ? 2 : 1;
  if (ranks > 1) {
    // The ranks' CTAs wait on one another: a cooperative launch guarantees that the whole
    // grid is resident at once (or refuses the launch).  No programmatic overlap.
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.numAttrs = 2;
  }
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, a, tmw, tms, tmb, sc_tma, mode, ks, C, toka, rowtiles, n_items),
                    "qmv_kernel launch");
}

// Row-parallel TP (dense mode) is its own instantiation so that the plain GEMV keeps its registers.
template <int BITS, int GS, int NT, bool CC>
static int launch_qmv_t(const QmvArgs& a, int mode, int64_t zcount, int ks, int C, int toka, cudaStream_t st) {
  if (a.tp_world > 1) {
    if (mode != QMV_DENSE) return set_error(VMLX_E_UNSUPPORTED, "tp: row-parallel fusion is dense-only");
    return launch_qmv_k<BITS, GS, NT, CC, true>(a, mode, zcount, ks, C, toka, st);
  }
  return launch_qmv_k<BITS, GS, NT, CC, false>(a, mode, zcount, ks, C, toka, st);
}

// K-slice width for a cluster of C CTAs: whole stages of groups where the
// rounding does not leave a slice empty.
static int slice_groups(int64_t KG, int C, int SG) {
  int ks = (int)((KG + C - 1) / C);
  if (ks % SG && (int64_t)((ks + SG - 1) / SG * SG) * (C - 1) < KG) ks = (ks + SG - 1) / SG * SG;
  return ks;
}

template <int BITS, int GS>
static int launch_qmv_bg(const QmvArgs& a, int mode, int64_t zcount, int toka, cudaStream_t st) {
  constexpr int SG = QT<BITS, GS>::SG;
  const int64_t KG = a.K / GS;
  const int64_t items = ((a.N + QMV_ROWS - 1) / QMV_ROWS) * zcount;
  // 4-bit with <= QMV_CC_MAX_TOKENS token rows: the CUDA-core consumer (fewer
  // instructions per weight than an m16n8 MMA that would be mostly empty)
  const bool cc = BITS == 4 && toka <= QMV_CC_MAX_TOKENS;
  const void* kfn = qmv_kernel_for<BITS, GS>(toka, cc, a.tp_world > 1);
  auto smem_of = [&](int ks_, int toka_) {
    QmvPlan L;
    L.init(BITS, GS, ks_, toka_, cc);
    return L.total;
  };
  // Pick the cluster size that minimises the busiest cluster's work:
  // ceil(items / resident clusters) * groups per slice.  Persistent clusters
  // loop over items, so a grid one item past a full wave doubles the time.
  int bestC = 1;
  double best = 1e30;
  for (int C = 1; C <= QMV_MAX_CLUSTER && C <= KG; C++) {
    const int ks = slice_groups(KG, C, SG);
    if ((KG + ks - 1) / ks != C) continue;  // this C rounds to another one
    const size_t sm = smem_of(ks, toka);
    if (sm > 226 * 1024) continue;
    int per_sm = (int)((228 * 1024) / (sm + 1024));
    int reg_cap = cc ? 2 : 3;  // 160 threads x ~150 (CUDA-core) / ~128 (MMA) registers
    if (reg_cap > QMV_MAX_PER_SM) reg_cap = QMV_MAX_PER_SM;
    per_sm = per_sm > reg_cap ? reg_cap : (per_sm < 1 ? 1 : per_sm);
    int64_t clusters = (int64_t)sm_count() * per_sm / C;
    const int res = qmv_resident_clusters(kfn, C, sm);
    if (res > 0 && res < clusters) clusters = res;
    if (clusters < 1) continue;
    // each item also pays a fixed cost (x / scale staging, pipeline fill, the
    // cluster reduction) worth roughly 8 groups of streaming
    const double cost = (double)((items + clusters - 1) / clusters) * (ks + 8.0) + 0.5 * C;
    if (cost < best) { best = cost; bestC = C; }
  }
  int C = bestC;
  {  // tuning override (read once): VMLX_QMV_C forces the cluster size when it is valid
    static const int forceC = [] { const char* v = getenv("VMLX_QMV_C"); return v && *v ? atoi(v) : 0; }();
    if (forceC >= 1 && forceC <= QMV_MAX_CLUSTER && forceC <= KG) C = forceC;
  }

  int ks = slice_groups(KG, C, SG);
  while (smem_of(ks, toka) > 226 * 1024 && toka > 8) toka -= 8;
  if (smem_of(ks, toka) > 226 * 1024)
    return set_error(VMLX_E_UNSUPPORTED, "qmv: K=%lld too large for the shared-memory plan", (long long)a.K);
  C = (int)((KG + ks - 1) / ks);
  if constexpr (BITS == 4) {
    if (cc) {
      switch (toka) {
        case 1: return launch_qmv_t<BITS, GS, 1, true>(a, mode, zcount, ks, C, toka, st);
        case 2: return launch_qmv_t<BITS, GS, 2, true>(a, mode, zcount, ks, C, toka, st);
        case 3: return launch_qmv_t<BITS, GS, 3, true>(a, mode, zcount, ks, C, toka, st);
        default: return launch_qmv_t<BITS, GS, 4, true>(a, mode, zcount, ks, C, toka, st);
      }
    }
  }
  const int nt = (toka + 7) / 8;
  switch (nt) {
    case 1: return launch_qmv_t<BITS, GS, 1, false>(a, mode, zcount, ks, C, toka, st);
    case 2: return launch_qmv_t<BITS, GS, 2, false>(a, mode, zcount, ks, C, toka, st);
    case 3: return launch_qmv_t<BITS, GS, 3, false>(a, mode, zcount, ks, C, toka, st);
    default: return launch_qmv_t<BITS, GS, 4, false>(a, mode, zcount, ks, C, toka, st);
  }
}

// Host launcher shared by the dense and gathered entry points.  `toka` is the
// number of token rows staged per pass (<= 32); zcount the number of
// (batch element | expert) weight selections.
int launch_qmv(const QmvArgs& a, int mode, int bits, int gs, int64_t zcount, int toka, cudaStream_t st) {
  if (qgemv_covers(a, mode, bits, gs)) return launch_qgemv(a, bits, gs, st);
  if (toka < 1) toka = 1;
  if (toka > 32) toka = 32;
  if (bits == 4 && gs == 32) return launch_qmv_bg<4, 32>(a, mode, zcount, toka, st);
  if (bits == 4 && gs == 64) return launch_qmv_bg<4, 64>(a, mode, zcount, toka, st);
  if (bits == 4 && gs == 128) return launch_qmv_bg<4, 128>(a, mode, zcount, toka, st);
  if (bits == 8 && gs == 32) return launch_qmv_bg<8, 32>(a, mode, zcount, toka, st);
  if (bits == 8 && gs == 64) return launch_qmv_bg<8, 64>(a, mode, zcount, toka, st);
  if (bits == 8 && gs == 128) return launch_qmv_bg<8, 128>(a, mode, zcount, toka, st);
  return set_error(VMLX_E_UNSUPPORTED, "matmul: bits=%d group_size=%d not supported", bits, gs);
}

}  // namespace vmlx
