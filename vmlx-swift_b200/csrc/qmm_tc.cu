// qmm_tc.cu -- tcgen05 / TMEM tensor-core GEMM for prefill and batched tiles (M > 32).
//
// y[M, N] = x[M, K] @ dequantize(W[N, K])^T, the op of MLX's affine_qmm_t
// (Source/Cmlx/mlx-generated/metal/quantized.h:1136-1261, 1756-1813): like the
// reference, W tiles are dequantized to the activation dtype (bf16,
// QuantizedBlockLoader / dequantize, :525-739) and multiplied on the matrix
// units with fp32 accumulation.
//
// One CTA computes a BN (128 or 256 weight rows: one or two M=128 MMA halves
// sharing each x stage) x BT (64, 128 or 256 tokens) tile of y^T over one K
// split; S > 1 splits of a tile form a thread-block cluster and reduce through
// distributed shared memory in a fixed order (deterministic).
//   warp 0    TMA producer: x tile [BT tokens x 64 k] (128-byte swizzle = the
//             UMMA K-major SW128 layout) and the raw packed W tile [BN rows x
//             128 B] into rings completing on mbarriers;
//   warp 1    allocates TMEM (a BT-column accumulator per 128-row half + 4 A
//             stages of 32 columns per half); one thread issues
//             tcgen05.mma (kind::f16, M=128, N=BT, K=16; A = dequantized W from
//             TMEM, B = x K-major from shared memory) and tcgen05.commit;
//   warps 4.. dequantize: warp group g = (row half, k half) owns rows
//             [128*(g>>1), +128) and k [32*(g&1), +32) of every stage, thread t
//             of the group weight row t = TMEM lane t; codes become bf16
//             scale*q + bias stored with tcgen05.st straight into the A stage
//             (row = lane, two k per 32-bit column), so the weight operand never
//             touches shared memory, whose bandwidth the x operand and the TMA
//             writes need.  After the K loop they move the fp32 accumulator
//             TMEM -> shared memory (token-major);
//   all warps reduce the S splits and store bf16 y with coalesced 8-byte stores.
// No multicast anywhere (this path may run in multi-GPU processes).
#include <cooperative_groups.h>

#include "kernels.cuh"
#include "sm100_util.cuh"
#include "tmap.cuh"

namespace cg = cooperative_groups;

namespace vmlx {


constexpr int TC_BK = 64;   // k per stage (one 128-byte swizzle row of bf16)

// 8 4-bit codes (one packed word, LSB first) -> 8 bf16 s*q + b, each rounded once.
// Codes are made exact as bf16 128+q (high byte 0x43, q in the low mantissa bits).
__device__ __forceinline__ uint4 dq8_4bit(uint32_t w, bf162 s2, bf162 b2) {
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;  // even / odd codes per byte
  const bf162 c128 = u32_as_bf162(0x43004300u);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint32_t sel = (uint32_t)j | ((uint32_t)j << 4) | ((uint32_t)(4 + j) << 8) | ((uint32_t)(4 + j) << 12);
    const uint32_t pr = (prmt(lo, hi, sel) & 0x00FF00FFu) | 0x43004300u;  // (q_2j, q_2j+1) as 128+q
    o[j] = bf162_as_u32(__hfma2(__hsub2(u32_as_bf162(pr), c128), s2, b2));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 8-bit codes (two words) -> 8 bf16: code byte into an fp32 2^23 + q, exact q,
// fp32 s*q + b (s*q exact), rounded to bf16 -- the oracle's order of operations.
__device__ __forceinline__ uint4 dq8_8bit(uint32_t w0, uint32_t w1, float s, float b) {
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint32_t w = j < 2 ? w0 : w1;
    const uint32_t i0 = (j & 1) * 2;
    const float f0 = __uint_as_float(prmt(w, 0x4B000000u, 0x7440u | i0)) - 8388608.f;
    const float f1 = __uint_as_float(prmt(w, 0x4B000000u, 0x7440u | (i0 + 1))) - 8388608.f;
    o[j] = bf162_as_u32(__floats2bfloat162_rn(__fadd_rn(__fmul_rn(f0, s), b), __fadd_rn(__fmul_rn(f1, s), b)));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Ring depths per token-tile width: enough bytes in flight per SM to cover the
// L2/HBM latency of the TMA loads.  A raw W stage is one [256 rows x 128 B] box
// with the 128-byte swizzle (16-byte chunk c of row r at c ^ (r & 7)): it covers
// RKS k-stages, keeps the TMA row-request count low, and a warp's 16-byte reads
// of 32 consecutive rows are bank-conflict free.  Shared memory stays above half
// the SM's, so one CTA owns the SM's 512 TMEM columns.
// NH = 128-row MMA halves per tile (tile rows BN = 128*NH).  Warps: 0 producer, 1 MMA,
// 2-3 idle, then 8*NH dequantizing warps (NH row halves x 2 k halves x 4 lane quarters).
template <int BITS, int BT, int NH>
struct TcLayout {
  static constexpr int BN = TC_UM * NH;           // weight rows per tile
  static constexpr int DQ = 256 * NH;             // dequantizing threads
  static constexpr int WARPS = 4 + DQ / 32;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int SX = BT == 256 ? 4 : BT == 128 ? 6 : 8;  // x stages
  static constexpr int SR = 3;                    // raw W stages
  static constexpr int SA = 4;                    // dequantized A stages (TMEM)
  static constexpr int RAWB = TC_BK * BITS / 8;   // packed bytes per weight row per k-stage
  static constexpr int RKS = 128 / RAWB;          // k-stages per raw stage
  static constexpr int XS = BT * 128;             // x stage bytes
  static constexpr int RS = BN * 128;             // raw stage bytes
  static constexpr int RING = SX * XS + SR * RS;
  static constexpr int A_COL = NH * BT;           // first TMEM column of the A stages
  static constexpr int A_W = NH * 32;             // TMEM columns per A stage
  static constexpr int TCOLS = A_COL + SA * A_W <= 256 ? 256 : 512;
  static_assert(A_COL + SA * A_W <= 512, "TMEM budget");
  static constexpr int RED = BT * BN * 4;         // fp32 accumulator, token-major
  static constexpr int DATA = RING > RED ? RING : RED;
  static constexpr int BARS = (2 * SX + 2 * SR + 2 * SA + 1) * 8 + 16;
  static constexpr size_t SMEM = (size_t)DATA + BARS + 1024;
  // a CTA holding all 512 TMEM columns must own its SM: more than half the shared memory
  static_assert(SMEM <= 227 * 1024 && (TCOLS == 256 || SMEM > 116 * 1024), "one CTA per SM");
};

template <int BITS, int GS, int BT, int NH>
__global__ void __launch_bounds__(TcLayout<BITS, BT, NH>::THREADS, 1)
qmm_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
              const bf16* __restrict__ scales, const bf16* __restrict__ biases, bf16* __restrict__ y,
              int M, int N, int K, int S, int* status, const int4* __restrict__ slots) {
  using L = TcLayout<BITS, BT, NH>;
  constexpr int SX = L::SX, SA = L::SA, SR = L::SR, TC_BN = L::BN, TC_DQ = L::DQ, TC_WARPS = L::WARPS;
  extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
  uint8_t* smem = tc_smem_raw + ((1024 - (smem_u32(tc_smem_raw) & 1023)) & 1023);
  uint8_t* xs = smem;
  uint8_t* raw = xs + SX * L::XS;
  float* red = reinterpret_cast<float*>(smem);  // reuses the rings once the K loop is done
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::DATA);
  uint64_t* x_full = bars;
  uint64_t* x_empty = x_full + SX;
  uint64_t* r_full = x_empty + SX;
  uint64_t* r_empty = r_full + SR;
  uint64_t* a_full = r_empty + SR;
  uint64_t* a_empty = a_full + SA;
  uint64_t* acc_full = a_empty + SA;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = (int)blockIdx.x % S;
  const int n0 = ((int)blockIdx.x / S) * TC_BN;
  // Expert-segmented mode (sorted gather_qmm): blockIdx.y is a slot {expert, first row, rows}
  // of the expert-sorted x; the tile multiplies those rows by the expert's weights.  Unused
  // slots (rows == 0) exit before touching any barrier or TMEM (uniform across the cluster,
  // whose CTAs share blockIdx.y).
  int m0 = (int)blockIdx.y * BT, m_end = M, wrow0 = 0;
  if (slots) {
    const int4 sl = slots[blockIdx.y];
    if (sl.z <= 0) return;
    m0 = sl.y;
    m_end = sl.y + sl.z < M ? sl.y + sl.z : M;
    wrow0 = sl.x * N;
  }
  const int KB = K / TC_BK;
  const int kb0 = (int)((int64_t)split * KB / S), nkb = (int)((int64_t)(split + 1) * KB / S) - kb0;
  const int KG = K / GS;

  if (tid == 0) {
    for (int i = 0; i < SX; i++) { mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], 1); }
    for (int i = 0; i < SR; i++) { mbar_init(&r_full[i], 1); mbar_init(&r_empty[i], TC_DQ / 32); }
    for (int i = 0; i < SA; i++) { mbar_init(&a_full[i], TC_DQ / 32); mbar_init(&a_empty[i], 1); }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmx);
    tma_prefetch_desc(&tmw);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // Setup above overlaps the previous kernel's tail under programmatic launch; from here on
  // this grid reads x and writes y.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < nkb; i++) {
        const int kb = kb0 + i, sx = i % SX;
        if (i % L::RKS == 0) {  // raw stage j covers k-stages [j*RKS, j*RKS + RKS) of this split
          const int j = i / L::RKS, sr = j % SR;
          if (j >= SR) ok &= mbar_wait(&r_empty[sr], ((j / SR) - 1) & 1);
          mbar_arrive_expect_tx(&r_full[sr], L::RS);
          tma_load_2d(raw + (size_t)sr * L::RS, &tmw, kb * L::RAWB, wrow0 + n0, &r_full[sr]);
        }
        if (i >= SX) ok &= mbar_wait(&x_empty[sx], ((i / SX) - 1) & 1);
        mbar_arrive_expect_tx(&x_full[sx], L::XS);
        tma_load_2d(xs + (size_t)sx * L::XS, &tmx, kb * TC_BK, m0, &x_full[sx]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc_idesc(BT);
      for (int i = 0; i < nkb; i++) {
        const int sx = i % SX, sa = i % SA;
        ok &= mbar_wait(&a_full[sa], (i / SA) & 1);
        ok &= mbar_wait(&x_full[sx], (i / SX) & 1);
        tc_fence_after();
        const uint32_t a_tmem = tmem + (uint32_t)(L::A_COL + sa * L::A_W);
        const uint32_t b_addr = smem_u32(xs + (size_t)sx * L::XS);
#pragma unroll
        for (int k = 0; k < TC_BK / 16; k++) {
          const uint64_t db = umma_desc_sw128(b_addr + k * 32);
#pragma unroll
          for (int mh = 0; mh < NH; mh++)
            umma_f16_ts(tmem + (uint32_t)(mh * BT), a_tmem + mh * 32 + k * 8, db, idesc, (i | k) ? 1u : 0u);
        }
        umma_commit(&a_empty[sa]);
        umma_commit(&x_empty[sx]);
      }
      umma_commit(acc_full);
      // Drain: nobody else waits for the last stages' empty-barrier arrivals, which land
      // when their MMAs complete; wait for them here so that no arrival can reach this
      // shared memory after the CTA exits (a later CTA on this SM may place its own
      // barriers there).
      for (int i = nkb - SX < 0 ? 0 : nkb - SX; i < nkb; i++) ok &= mbar_wait(&x_empty[i % SX], (i / SX) & 1);
      for (int i = nkb - SA < 0 ? 0 : nkb - SA; i < nkb; i++) ok &= mbar_wait(&a_empty[i % SA], (i / SA) & 1);
    }
  } else if (warp >= 4) {
    // ---------------- dequantize W into the TMEM A stages ----------------
    const int dq = tid - 128;
    const int g = dq >> 7;     // warp group: row half g >> 1, k half g & 1
    const int mh = g >> 1, h = g & 1;
    const int r = dq & 127;    // row within the half = TMEM lane
    const int q4 = warp & 3;   // this warp's TMEM lane quarter: r == 32*q4 + lane
    const int rt = mh * TC_UM + r;  // row within the tile
    const int row = wrow0 + (n0 + rt < N ? n0 + rt : N - 1);
    const bf16* srow = scales + (int64_t)row * KG;
    const bf16* brow = biases + (int64_t)row * KG;
    // group of this thread's 32 k in stage i (32 k never straddle a group, GS >= 32);
    // loaded one stage ahead
    auto grp = [&](int i) { return ((kb0 + i) * TC_BK + h * 32) / GS; };
    bf16 sn = srow[grp(0)], bn = brow[grp(0)];
    for (int i = 0; i < nkb; i++) {
      const int j = i / L::RKS, sub = i % L::RKS, sr = j % SR, sa = i % SA;
      const bf16 sv = sn, bv = bn;
      if (i + 1 < nkb) {
        sn = srow[grp(i + 1)];
        bn = brow[grp(i + 1)];
      }
      if (sub == 0) ok &= mbar_wait(&r_full[sr], (j / SR) & 1);
      // this thread's 32 codes: 16-byte chunks c0 .. c0 + BITS/4 of its row (4 words for 4-bit, 8 for 8-bit)
      const uint8_t* rp = raw + (size_t)sr * L::RS + rt * 128;
      const int c0 = (sub * L::RAWB + h * (L::RAWB / 2)) >> 4;
      uint32_t wv[BITS];
#pragma unroll
      for (int v = 0; v < BITS / 4; v++) {
        const uint4 u = *reinterpret_cast<const uint4*>(rp + (((c0 + v) ^ (rt & 7)) << 4));
        wv[4 * v] = u.x; wv[4 * v + 1] = u.y; wv[4 * v + 2] = u.z; wv[4 * v + 3] = u.w;
      }
      if (sub == L::RKS - 1 || i == nkb - 1) {
        // the codes must be in registers before the stage is released to the next TMA
#pragma unroll
        for (int v = 0; v < BITS; v++) asm volatile("" ::"r"(wv[v]));
        __syncwarp();
        if (lane == 0) mbar_arrive(&r_empty[sr]);
      }
      uint32_t o[16];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint4 q;
        if constexpr (BITS == 4) {
          q = dq8_4bit(wv[c], __bfloat162bfloat162(sv), __bfloat162bfloat162(bv));
        } else {
          q = dq8_8bit(wv[2 * c], wv[2 * c + 1], __bfloat162float(sv), __bfloat162float(bv));
        }
        o[4 * c] = q.x; o[4 * c + 1] = q.y; o[4 * c + 2] = q.z; o[4 * c + 3] = q.w;
      }
      // Publish the previous stage: its TMEM store overlapped this stage's loads and math.
      if (i > 0) {
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[(i - 1) % SA]);
      }
      if (i >= SA) ok &= mbar_wait(&a_empty[sa], ((i / SA) - 1) & 1);
      tc_fence_after();
      // A stage sa, half mh: lane = row, columns [h*16, h*16+16) hold k [32h, 32h+32) in pairs
      tmem_st16(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(L::A_COL + sa * L::A_W + mh * 32 + h * 16), o);
    }
    if (nkb > 0) {
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[(nkb - 1) % SA]);
    }
    // ---------------- accumulator: TMEM -> shared memory (token-major) ----------------
    ok &= mbar_wait(acc_full, 0);
    tc_fence_after();
    for (int c0 = h * (BT / 2); c0 < (h + 1) * (BT / 2); c0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(mh * BT + c0), v);
#pragma unroll
      for (int j = 0; j < 16; j++) red[(c0 + j) * TC_BN + rt] = __uint_as_float(v[j]);
    }
  }
  tc_fence_before();
  if (S > 1) {
    cluster_arrive();
    cluster_wait();
  } else {
    __syncthreads();
  }
  // ---------------- reduce the splits (fixed order) and store bf16 y ----------------
  {
    const int t_lo = split * BT / S, t_hi = (split + 1) * BT / S;
    constexpr int NPL = TC_BN / 32;  // output columns per lane (4 or 8)
    const int n = n0 + NPL * lane;
    const bool vec = (N % NPL) == 0 && n + NPL <= N;
    cg::cluster_group cluster = cg::this_cluster();
    for (int t = t_lo + warp; t < t_hi; t += TC_WARPS) {
      const int m = m0 + t;
      if (m >= m_end) break;
      float acc[NPL];
#pragma unroll
      for (int j = 0; j < NPL; j++) acc[j] = 0.f;
      for (int q = 0; q < S; q++) {
        const float* src = (S > 1 ? cluster.map_shared_rank(red, q) : red) + t * TC_BN + NPL * lane;
#pragma unroll
        for (int j = 0; j < NPL; j += 4) {
          const float4 v = *reinterpret_cast<const float4*>(src + j);
          acc[j] += v.x; acc[j + 1] += v.y; acc[j + 2] += v.z; acc[j + 3] += v.w;
        }
      }
      bf16* yr = y + (int64_t)m * N;
      if (vec) {
        uint32_t o[NPL / 2];
#pragma unroll
        for (int j = 0; j < NPL / 2; j++) o[j] = bf162_as_u32(__floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]));
        if constexpr (NPL == 8) *reinterpret_cast<uint4*>(yr + n) = make_uint4(o[0], o[1], o[2], o[3]);
        else *reinterpret_cast<uint2*>(yr + n) = make_uint2(o[0], o[1]);
      } else {
        for (int j = 0; j < NPL; j++)
          if (n + j < N) yr[n + j] = __float2bfloat16_rn(acc[j]);
      }
    }
  }
  if (S > 1) {  // keep this CTA's shared memory alive until every split has read it
    cluster_arrive();
    cluster_wait();
  }
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TCOLS));
  if (!ok && status) atomicExch(status, VMLX_E_STATE);
}

template <int BITS, int GS, int BT, int NH>
static int launch_tc(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases, bf16* y, int64_t M,
                     int64_t N, int64_t K, cudaStream_t st, const int4* slots = nullptr, int64_t n_slots = 0,
                     int64_t n_experts = 1) {
  using L = TcLayout<BITS, BT, NH>;
  auto kern = qmm_tc_kernel<BITS, GS, BT, NH>;
  {
    const int rc = ensure_max_dynamic_smem((const void*)kern, (int)L::SMEM);
    if (rc) return rc;
  }
  CUtensorMap tmx, tmw;
  if (!make_tmap_2d(&tmx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, TC_BK,
                    BT, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_2d(&tmw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, (uint64_t)K * BITS / 8, (uint64_t)(N * n_experts),
                    (uint64_t)K * BITS / 8, 128, L::BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return VMLX_E_CUDA;
  // K splits fill the SMs when the tile grid is small; each split keeps >= 8 stages, and
  // clusters stay at <= 4 CTAs so that they co-schedule in one wave.
  const int64_t ntn = (N + L::BN - 1) / L::BN, ntm = slots ? n_slots : (M + BT - 1) / BT;
  const int64_t tiles = ntn * ntm, KB = K / TC_BK;
  int S = 1;
  while (S < 4 && tiles * S * 2 <= sm_count() && KB / (S * 2) >= 8) S *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(ntn * S), (unsigned)ntm, 1);
  cfg.blockDim = dim3(L::THREADS);
  cfg.dynamicSmemBytes = L::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = (unsigned)S;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = launch_overlap() ? 2 : 1;
  if (ntm > 65535) return set_error(VMLX_E_UNSUPPORTED, "qmm_tc: %lld token tiles", (long long)ntm);
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, tmx, tmw, scales, biases, y, (int)M, (int)N, (int)K, S,
                                       (int*)nullptr, slots),
                    "qmm_tc_kernel launch");
}

// Tile shape by problem shape (measured on B200, 4-bit g64 Llama FFN shapes):
//   - many token tiles: 128 weight rows x 256 tokens (least dequantization per flop);
//   - otherwise 256 weight rows (two MMA halves sharing each x stage) when that still
//     gives >= 56 tiles, else 128 rows with K splits.
template <int BITS, int GS>
static int launch_bt(const bf16* x, const uint32_t* w, const bf16* s, const bf16* b, bf16* y, int64_t M, int64_t N,
                     int64_t K, cudaStream_t st) {
  const int64_t sms = sm_count();
  const int64_t ntn1 = (N + 127) / 128, ntn2 = (N + 255) / 256;
  if (M > 128 && ntn1 * ((M + 255) / 256) >= sms / 2) return launch_tc<BITS, GS, 256, 1>(x, w, s, b, y, M, N, K, st);
  if (M > 64) {
    if (ntn2 * ((M + 127) / 128) >= 56) return launch_tc<BITS, GS, 128, 2>(x, w, s, b, y, M, N, K, st);
    return launch_tc<BITS, GS, 128, 1>(x, w, s, b, y, M, N, K, st);
  }
  if (ntn2 >= 56) return launch_tc<BITS, GS, 64, 2>(x, w, s, b, y, M, N, K, st);
  return launch_tc<BITS, GS, 64, 1>(x, w, s, b, y, M, N, K, st);
}

int launch_qmm_tc(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases, bf16* y, int64_t M,
                  int64_t N, int64_t K, int bits, int gs, cudaStream_t st, bool* handled) {
  *handled = false;
  if (K % TC_BK || !aligned(x, 16) || !aligned(w, 16) || (M + 63) / 64 > 65535 || M > (1ll << 30) ||
      N > (1ll << 30) || K > (1ll << 30))
    return VMLX_OK;  // shapes outside the tile plan run on the GEMV kernel in passes
  *handled = true;
  if (bits == 4 && gs == 32) return launch_bt<4, 32>(x, w, scales, biases, y, M, N, K, st);
  if (bits == 4 && gs == 64) return launch_bt<4, 64>(x, w, scales, biases, y, M, N, K, st);
  if (bits == 4 && gs == 128) return launch_bt<4, 128>(x, w, scales, biases, y, M, N, K, st);
  if (bits == 8 && gs == 32) return launch_bt<8, 32>(x, w, scales, biases, y, M, N, K, st);
  if (bits == 8 && gs == 64) return launch_bt<8, 64>(x, w, scales, biases, y, M, N, K, st);
  if (bits == 8 && gs == 128) return launch_bt<8, 128>(x, w, scales, biases, y, M, N, K, st);
  *handled = false;
  return VMLX_OK;
}

// Expert-segmented GEMM for sorted gather_qmm: x [M rows sorted by expert, K], slots
// {expert, first row, rows} (rows <= 64; unused slots have rows 0), w / scales / biases
// stacks of n_experts [N, ...] matrices.  One 64-token tile per slot.
int launch_qmm_tc_grouped(const bf16* x, const uint32_t* w, const bf16* scales, const bf16* biases, bf16* y,
                          int64_t M, int64_t N, int64_t K, int64_t n_experts, const int4* slots, int64_t n_slots,
                          int bits, int gs, cudaStream_t st) {
  if (K % TC_BK || !aligned(x, 16) || !aligned(w, 16) || M >= (1ll << 30) || N * n_experts >= (1ll << 31))
    return set_error(VMLX_E_UNSUPPORTED, "qmm_tc grouped: shape not covered");
  const int64_t ntn2 = (N + 255) / 256;
#define VMLX_GROUPED(B, G)                                                                                   \
  if (bits == B && gs == G) {                                                                               \
    if (ntn2 * n_slots >= 112) return launch_tc<B, G, 64, 2>(x, w, scales, biases, y, M, N, K, st, slots, n_slots, \
                                                             n_experts);                                    \
    return launch_tc<B, G, 64, 1>(x, w, scales, biases, y, M, N, K, st, slots, n_slots, n_experts);          \
  }
  VMLX_GROUPED(4, 32) VMLX_GROUPED(4, 64) VMLX_GROUPED(4, 128) VMLX_GROUPED(8, 32) VMLX_GROUPED(8, 64)
  VMLX_GROUPED(8, 128)
#undef VMLX_GROUPED
  return set_error(VMLX_E_UNSUPPORTED, "qmm_tc grouped: bits=%d group_size=%d", bits, gs);
}

}  // namespace vmlx
