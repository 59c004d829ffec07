// tp.cu -- tensor-parallel group handle and the one-shot all-reduce over NVLink P2P.
//
// Replaces the reference's collective path for row-parallel linears:
//   ShardedToAllLinear.callAsFunction (Libraries/MLXDistributedTP/LinearLayers.swift:198-205)
//   -> Collectives.allSum (Collectives.swift:27-32) -> vmlx_all_sum
//   (Libraries/CmlxDistributedShim/CmlxDistributedShim.c:54-60) -> mlx distributed::all_sum.
//
// Design (one process per GPU, or one process driving several GPUs):
//  * Every rank owns one device buffer: [2 parities][world][max_bytes] receive
//    slots, then [2][world][TP_MAX_CTAS] uint32 flags, then [TP_MAX_CTAS] epochs,
//    then the same kind of region for the fused row-parallel GEMV (below).
//    Peers map it with CUDA IPC (or get its pointer directly in one process).
//  * all_sum is one kernel: CTA c takes chunk c of the vector, stores it into
//    slot [parity][my_rank] of every rank's buffer (P2P stores over NVLink /
//    NVSwitch, including itself), fences at system scope, publishes flag
//    [parity][my_rank][c] = epoch on every rank (st.release.sys), waits for
//    the world's flags in its own buffer (ld.acquire.sys, bounded by a
//    globaltimer deadline), then sums the world slots in fixed rank order
//    (identical result on every rank) and writes the output.
//  * The call's epoch lives in device memory and is advanced by the kernel's
//    last CTA, so a captured CUDA graph can be replayed; flags are monotonic.
//    Two parities of slots let a rank run one call ahead of a slow peer
//    without overwriting data that peer still reads.
//  * A wait that runs out records VMLX_E_PEER_TIMEOUT in the handle's status
//    word and returns; the context stays usable (vmlx_tp_status reads it).
// NCCL is used only as the measured baseline, outside this library.
#include <cstdlib>
#include <cstring>

#include "kernels.cuh"
#include "sm100_util.cuh"

namespace vmlx {

constexpr int TP_MAX_WORLD = 8;
constexpr int TP_MAX_CTAS = 64;
constexpr int TP_THREADS = 256;

struct TpPeers {
  char* buf[TP_MAX_WORLD];  // every rank's buffer base, as seen from this device
};

struct TpHandle {
  int rank, world, device;
  size_t max_bytes;        // bytes per slot
  char* local;             // this rank's buffer
  size_t total_bytes;
  cudaIpcMemHandle_t ipc;
  bool ipc_valid;
  char* peer_base[TP_MAX_WORLD];  // mapped buffers (IPC-opened or given)
  bool peer_opened[TP_MAX_WORLD];
  int* status;             // device word: 0 or VMLX_E_PEER_TIMEOUT
  uint64_t timeout_ns;
  bool connected;
  bool loop;               // loopback group: every rank's buffer on this device, ranks run as one grid
};

__host__ __device__ inline size_t tp_slot_off(int parity, int src, size_t max_bytes, int world) {
  return ((size_t)parity * world + src) * max_bytes;
}
__host__ __device__ inline size_t tp_flag_off(size_t max_bytes, int world) {
  return (size_t)2 * world * max_bytes;
}
__host__ __device__ inline size_t tp_epoch_off(size_t max_bytes, int world) {
  return tp_flag_off(max_bytes, world) + (size_t)2 * world * TP_MAX_CTAS * sizeof(uint32_t);
}
// Region of the fused row-parallel GEMV + all-reduce (its own slots, so that its
// parity never aliases the standalone all_sum's): [2][world][max_bytes] slots,
// [2][world][TP_FUSED_MAXC] flags, then {epoch, finished-CTA counter}.
__host__ __device__ inline size_t tp_fused_slots_off(size_t max_bytes, int world) {
  return (tp_epoch_off(max_bytes, world) + TP_MAX_CTAS * sizeof(uint32_t) + 255) / 256 * 256;
}
__host__ __device__ inline size_t tp_fused_flags_off(size_t max_bytes, int world) {
  return tp_fused_slots_off(max_bytes, world) + (size_t)2 * world * max_bytes;
}
__host__ __device__ inline size_t tp_fused_epoch_off(size_t max_bytes, int world) {
  return tp_fused_flags_off(max_bytes, world) + (size_t)2 * world * TP_FUSED_MAXC * sizeof(uint32_t);
}
// Slots of the standalone low-latency all_sum ([2][world][max_bytes] of 8-byte {value,
// epoch} words), apart from the flag protocol's slots: a stale word of packed bf16 data
// left there by a flag-protocol call could otherwise carry a matching "epoch".
__host__ __device__ inline size_t tp_ll_slot_off(int parity, int src, size_t max_bytes, int world) {
  return ((tp_fused_epoch_off(max_bytes, world) + 256 + 255) / 256 * 256) + ((size_t)parity * world + src) * max_bytes;
}
inline size_t tp_total_bytes(size_t max_bytes, int world) { return tp_ll_slot_off(2, 0, max_bytes, world); }

// Every all_sum call (either protocol) has one epoch for all its CTAs: read from
// epoch[0] at the start, written back by the grid's last CTA (epoch[1] counts finished
// CTAs).  Slot parity = epoch & 1 alternates call by call, and a low-latency word's
// epoch is unique to its call whatever CTA wrote it.
__device__ __forceinline__ void tp_advance_epoch(uint32_t* epoch_p, uint32_t e) {
  __threadfence();
  if (atomicAdd(epoch_p + 1, 1u) == gridDim.x - 1) {
    epoch_p[1] = 0;
    epoch_p[0] = e;
    __threadfence();
  }
}

// One-shot all-reduce of n bf16 elements (n * 2 <= max_bytes, chunked over CTAs).
__global__ void __launch_bounds__(TP_THREADS)
tp_all_sum_kernel(TpPeers peers, int rank, int world, size_t max_bytes, const bf16* __restrict__ in,
                  bf16* __restrict__ out, int64_t n, int64_t chunk, int* status, uint64_t timeout_ns, int loop) {
  if (loop) {  // loopback group: rank = blockIdx.y, in / out stacked [world, n]
    rank = blockIdx.y;
    in += (int64_t)rank * n;
    out += (int64_t)rank * n;
  }
  const int c = blockIdx.x;
  const int64_t e0 = (int64_t)c * chunk;
  const int64_t e1 = e0 + chunk < n ? e0 + chunk : n;
  char* mine = peers.buf[rank];
  uint32_t* epoch_p = reinterpret_cast<uint32_t*>(mine + tp_epoch_off(max_bytes, world));
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_epoch = epoch_p[0] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int parity = e & 1;

  // 1. push my chunk into slot [parity][rank] of every rank (16-byte stores when aligned)
  const bool vec = ((e0 | e1) & 7) == 0;
  for (int r = 0; r < world; r++) {
    bf16* dst = reinterpret_cast<bf16*>(peers.buf[r] + tp_slot_off(parity, rank, max_bytes, world));
    if (vec) {
      for (int64_t i = e0 + threadIdx.x * 8; i < e1; i += TP_THREADS * 8)
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(in + i);
    } else {
      for (int64_t i = e0 + threadIdx.x; i < e1; i += TP_THREADS) dst[i] = in[i];
    }
  }
  __syncthreads();
  // 2. publish: flag [parity][rank][c] = e on every rank
  if (threadIdx.x < world) {
    __threadfence_system();
    uint32_t* f = reinterpret_cast<uint32_t*>(peers.buf[threadIdx.x] + tp_flag_off(max_bytes, world)) +
                  ((size_t)parity * world + rank) * TP_MAX_CTAS + c;
    st_release_sys(f, e);
  }
  // 3. wait for every rank's chunk in my buffer (bounded)
  if (threadIdx.x < world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + tp_flag_off(max_bytes, world)) +
                        ((size_t)parity * world + threadIdx.x) * TP_MAX_CTAS + c;
    if (!wait_flag_sys(f, e, timeout_ns)) {
      s_ok = 0;
      atomicExch(status, VMLX_E_PEER_TIMEOUT);
    }
  }
  __syncthreads();
  // 4. reduce in rank order (bitwise identical on every rank)
  if (s_ok) {
    for (int64_t i = e0 + threadIdx.x; i < e1; i += TP_THREADS) {
      float s = 0.f;
      for (int r = 0; r < world; r++)
        s += __bfloat162float(reinterpret_cast<const bf16*>(mine + tp_slot_off(parity, r, max_bytes, world))[i]);
      out[i] = __float2bfloat16_rn(s);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) tp_advance_epoch(epoch_p, e);
}

// Low-latency all-reduce for small vectors (n * 8 <= max_bytes): every element travels as
// one 8-byte word {bf16 bits, epoch} (single system-scope store), and readers poll the
// words themselves, so there is no fence and no flag round trip.  Its own slot region
// (tp_ll_slot_off), the same parities and per-call epochs as the flag protocol above;
// same rank-order fp32 sum.
__global__ void __launch_bounds__(TP_THREADS)
tp_all_sum_ll_kernel(TpPeers peers, int rank, int world, size_t max_bytes, const bf16* __restrict__ in,
                     bf16* __restrict__ out, int64_t n, int64_t chunk, int* status, uint64_t timeout_ns, int loop) {
  if (loop) {
    rank = blockIdx.y;
    in += (int64_t)rank * n;
    out += (int64_t)rank * n;
  }
  const int c = blockIdx.x;
  const int64_t e0 = (int64_t)c * chunk;
  const int64_t e1 = e0 + chunk < n ? e0 + chunk : n;
  char* mine = peers.buf[rank];
  uint32_t* epoch_p = reinterpret_cast<uint32_t*>(mine + tp_epoch_off(max_bytes, world));
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = epoch_p[0] + 1;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int parity = e & 1;
  for (int r = 0; r < world; r++) {
    uint64_t* dst = reinterpret_cast<uint64_t*>(peers.buf[r] + tp_ll_slot_off(parity, rank, max_bytes, world));
    for (int64_t i = e0 + threadIdx.x; i < e1; i += TP_THREADS)
      st_ll(dst + i, (uint32_t)__bfloat16_as_ushort(in[i]), e);
  }
  const uint64_t deadline = globaltimer() + timeout_ns;
  const uint64_t* slots = reinterpret_cast<const uint64_t*>(mine + tp_ll_slot_off(parity, 0, max_bytes, world));
  const size_t rstride = max_bytes / sizeof(uint64_t);
  bool ok = true;
  for (int64_t i = e0 + threadIdx.x; i < e1 && ok; i += TP_THREADS) {
    float s;
    ok = wait_ll_sum<TP_MAX_WORLD>(slots + i, rstride, world, e, deadline, s);
    if (ok) out[i] = __float2bfloat16_rn(s);
  }
  if (!ok) atomicExch(status, VMLX_E_PEER_TIMEOUT);
  __syncthreads();
  if (threadIdx.x == 0) tp_advance_epoch(epoch_p, e);
}

// MoE block output under expert-intermediate TP: scatterUnsort + score-weighted sum of this
// rank's partial expert outputs (vmlx_cuda_moe_combine's arithmetic, rounded to bf16 per rank),
// all-reduced over the group in the same kernel (the low-latency word protocol of
// tp_all_sum_ll_kernel, same slots and epochs: it is one more all_sum call in the group's
// sequence), optionally plus a residual.  One thread = 8 consecutive outputs of one token row.
// The epoch is advanced by the grid's last CTA (of gridDim.x * gridDim.y per rank).
template <typename TS>
__global__ void __launch_bounds__(128)
tp_moe_combine_kernel(TpPeers peers, int rank, int world, size_t max_bytes, const bf16* __restrict__ y,
                      const uint32_t* __restrict__ inv, const TS* __restrict__ scores, int64_t T, int k, int64_t D,
                      const bf16* __restrict__ residual, bf16* __restrict__ out, int* status, uint64_t timeout_ns,
                      int loop) {
  if (loop) {  // loopback group: rank = blockIdx.z, every operand stacked along a leading rank axis
    rank = blockIdx.z;
    y += (int64_t)rank * T * k * D;
    if (inv) inv += (int64_t)rank * T * k;
    scores += (int64_t)rank * T * k;
    out += (int64_t)rank * T * D;
    if (residual) residual += (int64_t)rank * T * D;
  }
  char* mine = peers.buf[rank];
  uint32_t* epoch_p = reinterpret_cast<uint32_t*>(mine + tp_epoch_off(max_bytes, world));
  __shared__ uint32_t s_epoch;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) s_epoch = epoch_p[0] + 1;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int parity = e & 1;
  const int64_t t = blockIdx.y;
  const int64_t d0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const bool act = d0 < D;
  // 1. this rank's combined partial, rounded to bf16 as the separate combine kernel does
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (act) {
    for (int j = 0; j < k; j++) {
      const int64_t pair = t * k + j;
      const int64_t src = inv ? (int64_t)inv[pair] : pair;
      float sc;
      if constexpr (sizeof(TS) == 4) sc = scores[pair];
      else sc = __bfloat162float(scores[pair]);
      const uint4 v = *reinterpret_cast<const uint4*>(y + src * D + d0);
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 f = __bfloat1622float2(u32_as_bf162(u[q]));
        float p0 = f.x * sc, p1 = f.y * sc;
        if constexpr (sizeof(TS) == 2) {  // bf16 scores: each product rounds to bf16 (MLX's bf16 multiply)
          p0 = __bfloat162float(__float2bfloat16_rn(p0));
          p1 = __bfloat162float(__float2bfloat16_rn(p1));
        }
        acc[2 * q] += p0;
        acc[2 * q + 1] += p1;
      }
    }
    // 2. push the 8 bf16 partials to every rank as {value, epoch} words
    for (int r = 0; r < world; r++) {
      uint64_t* dst = reinterpret_cast<uint64_t*>(peers.buf[r] + tp_ll_slot_off(parity, rank, max_bytes, world)) +
                      t * D + d0;
#pragma unroll
      for (int q = 0; q < 8; q++) st_ll(dst + q, (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc[q])), e);
    }
  }
  // 3. sum every rank's words of these outputs in rank order (bounded waits)
  bool ok = true;
  if (act) {
    const uint64_t deadline = globaltimer() + timeout_ns;
    const uint64_t* slots = reinterpret_cast<const uint64_t*>(mine + tp_ll_slot_off(parity, 0, max_bytes, world));
    const size_t rstride = max_bytes / sizeof(uint64_t);
    for (int q = 0; q < 8 && ok; q++) {
      float sum;
      ok = wait_ll_sum<TP_MAX_WORLD>(slots + t * D + d0 + q, rstride, world, e, deadline, sum);
      if (!ok) break;
      const int64_t idx = t * D + d0 + q;
      const bf16 sb = __float2bfloat16_rn(sum);
      out[idx] = residual ? __float2bfloat16_rn(__bfloat162float(residual[idx]) + __bfloat162float(sb)) : sb;
    }
    if (!ok) atomicExch(status, VMLX_E_PEER_TIMEOUT);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(epoch_p + 1, 1u) == gridDim.x * gridDim.y - 1) {
      epoch_p[1] = 0;
      epoch_p[0] = e;
      __threadfence();
    }
  }
}

static int tp_check(TpHandle* h) {
  if (!h) return set_error(VMLX_E_INVALID, "tp: null handle");
  return VMLX_OK;
}

}  // namespace vmlx

using namespace vmlx;

extern "C" int vmlx_tp_create(int rank, int world, size_t max_bytes, void** out) {
  if (!out) return set_error(VMLX_E_INVALID, "tp_create: null out");
  if (world < 1 || world > TP_MAX_WORLD || rank < 0 || rank >= world)
    return set_error(VMLX_E_INVALID, "tp_create: rank %d / world %d (world 1..%d)", rank, world, TP_MAX_WORLD);
  if (max_bytes == 0 || max_bytes % 16) return set_error(VMLX_E_INVALID, "tp_create: max_bytes must be a positive multiple of 16");
  TpHandle* h = new TpHandle();
  std::memset(h, 0, sizeof(*h));
  h->rank = rank;
  h->world = world;
  h->max_bytes = max_bytes;
  h->timeout_ns = 2000000000ull;  // 2 s
  int rc = check_cuda(cudaGetDevice(&h->device), "tp_create: cudaGetDevice");
  h->total_bytes = tp_total_bytes(max_bytes, world);
  if (!rc) rc = check_cuda(cudaMalloc(&h->local, h->total_bytes), "tp_create: cudaMalloc");
  if (!rc) rc = check_cuda(cudaMemset(h->local, 0, h->total_bytes), "tp_create: cudaMemset");
  if (!rc) rc = check_cuda(cudaMalloc(&h->status, sizeof(int)), "tp_create: cudaMalloc status");
  if (!rc) rc = check_cuda(cudaMemset(h->status, 0, sizeof(int)), "tp_create: cudaMemset status");
  if (!rc) {
    h->ipc_valid = cudaIpcGetMemHandle(&h->ipc, h->local) == cudaSuccess;
    cudaGetLastError();
  }
  if (rc) {
    if (h->local) cudaFree(h->local);
    if (h->status) cudaFree(h->status);
    delete h;
    return rc;
  }
  h->peer_base[rank] = h->local;
  *out = h;
  return VMLX_OK;
}

extern "C" int vmlx_tp_create_loopback(int world, size_t max_bytes, void** out) {
  if (!out) return set_error(VMLX_E_INVALID, "tp_create_loopback: null out");
  if (world < 2 || world > TP_MAX_WORLD)
    return set_error(VMLX_E_INVALID, "tp_create_loopback: world %d (2..%d)", world, TP_MAX_WORLD);
  if (max_bytes == 0 || max_bytes % 16)
    return set_error(VMLX_E_INVALID, "tp_create_loopback: max_bytes must be a positive multiple of 16");
  TpHandle* h = new TpHandle();
  std::memset(h, 0, sizeof(*h));
  h->rank = 0;
  h->world = world;
  h->max_bytes = max_bytes;
  h->timeout_ns = 2000000000ull;
  h->loop = true;
  int rc = check_cuda(cudaGetDevice(&h->device), "tp_create_loopback: cudaGetDevice");
  h->total_bytes = tp_total_bytes(max_bytes, world);
  const size_t stride = (h->total_bytes + 255) / 256 * 256;
  if (!rc) rc = check_cuda(cudaMalloc(&h->local, stride * world), "tp_create_loopback: cudaMalloc");
  if (!rc) rc = check_cuda(cudaMemset(h->local, 0, stride * world), "tp_create_loopback: cudaMemset");
  if (!rc) rc = check_cuda(cudaMalloc(&h->status, sizeof(int)), "tp_create_loopback: cudaMalloc status");
  if (!rc) rc = check_cuda(cudaMemset(h->status, 0, sizeof(int)), "tp_create_loopback: cudaMemset status");
  if (rc) {
    if (h->local) cudaFree(h->local);
    if (h->status) cudaFree(h->status);
    delete h;
    return rc;
  }
  for (int r = 0; r < world; r++) h->peer_base[r] = h->local + (size_t)r * stride;
  h->connected = true;
  *out = h;
  return VMLX_OK;
}

extern "C" int vmlx_tp_rank(void* tp) { return tp ? static_cast<TpHandle*>(tp)->rank : -1; }
extern "C" int vmlx_tp_size(void* tp) { return tp ? static_cast<TpHandle*>(tp)->world : -1; }

extern "C" int vmlx_tp_ipc_handle(void* tp, void* handle_out) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  if (!handle_out) return set_error(VMLX_E_INVALID, "tp_ipc_handle: null out");
  if (!h->ipc_valid) return set_error(VMLX_E_CUDA, "tp_ipc_handle: the buffer has no IPC handle");
  std::memcpy(handle_out, &h->ipc, sizeof(cudaIpcMemHandle_t));
  return VMLX_OK;
}

extern "C" int vmlx_tp_open_peers(void* tp, const void* handles) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  if (!handles) return set_error(VMLX_E_INVALID, "tp_open_peers: null handles");
  for (int r = 0; r < h->world; r++) {
    if (r == h->rank) continue;
    cudaIpcMemHandle_t ph;
    std::memcpy(&ph, static_cast<const char*>(handles) + (size_t)r * sizeof(cudaIpcMemHandle_t), sizeof(ph));
    void* p = nullptr;
    rc = check_cuda(cudaIpcOpenMemHandle(&p, ph, cudaIpcMemLazyEnablePeerAccess), "tp_open_peers: cudaIpcOpenMemHandle");
    if (rc) return rc;
    h->peer_base[r] = static_cast<char*>(p);
    h->peer_opened[r] = true;
  }
  h->connected = true;
  return VMLX_OK;
}

extern "C" int vmlx_tp_set_peer(void* tp, int peer, void* device_ptr) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  if (peer < 0 || peer >= h->world || peer == h->rank || !device_ptr)
    return set_error(VMLX_E_INVALID, "tp_set_peer: bad peer %d", peer);
  h->peer_base[peer] = static_cast<char*>(device_ptr);
  bool all = true;
  for (int r = 0; r < h->world; r++) all &= h->peer_base[r] != nullptr;
  h->connected = all;
  return VMLX_OK;
}

extern "C" void* vmlx_tp_buffer(void* tp) { return tp ? static_cast<TpHandle*>(tp)->local : nullptr; }

extern "C" int vmlx_tp_set_timeout_us(void* tp, uint64_t us) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  h->timeout_ns = us * 1000ull;
  return VMLX_OK;
}

extern "C" int vmlx_tp_all_sum(void* tp, void* out, const void* in, int64_t n, void* stream) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  if (!out || !in) return set_error(VMLX_E_INVALID, "tp_all_sum: null pointer");
  if (n < 0 || (size_t)n * 2 > h->max_bytes)
    return set_error(VMLX_E_INVALID, "tp_all_sum: %lld elements exceed the %zu-byte slots", (long long)n, h->max_bytes);
  if (n == 0) return VMLX_OK;
  if (!aligned(out, 16) || !aligned(in, 16)) return set_error(VMLX_E_INVALID, "tp_all_sum: pointers must be 16-byte aligned");
  if (h->world == 1) {
    if (out != in) return check_cuda(cudaMemcpyAsync(out, in, (size_t)n * 2, cudaMemcpyDeviceToDevice, as_stream(stream)),
                                     "tp_all_sum: copy");
    return VMLX_OK;
  }
  if (!h->connected) return set_error(VMLX_E_STATE, "tp_all_sum: peers not connected");
  // chunks of >= 2048 elements, at most TP_MAX_CTAS CTAs, multiples of 8 elements
  int64_t ctas = (n + 2047) / 2048;
  if (ctas > TP_MAX_CTAS) ctas = TP_MAX_CTAS;
  int64_t chunk = ((n + ctas - 1) / ctas + 7) / 8 * 8;
  ctas = (n + chunk - 1) / chunk;
  TpPeers peers;
  for (int r = 0; r < TP_MAX_WORLD; r++) peers.buf[r] = r < h->world ? h->peer_base[r] : nullptr;
  if ((size_t)n * 8 <= h->max_bytes) {
    // low-latency words: one element per thread where TP_MAX_CTAS CTAs allow it
    ctas = (n + TP_THREADS - 1) / TP_THREADS;
    if (ctas > TP_MAX_CTAS) ctas = TP_MAX_CTAS;
    chunk = (n + ctas - 1) / ctas;
    ctas = (n + chunk - 1) / chunk;
  }
  const bool ll = (size_t)n * 8 <= h->max_bytes;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas, h->loop ? (unsigned)h->world : 1u, 1);
  cfg.blockDim = dim3(TP_THREADS);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr;
  if (h->loop) {  // the ranks' CTAs wait on one another: all resident at once, or no launch
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
  }
  const int rank = h->loop ? 0 : h->rank, loop = h->loop ? 1 : 0;
  return check_cuda(ll ? cudaLaunchKernelEx(&cfg, tp_all_sum_ll_kernel, peers, rank, h->world, h->max_bytes,
                                            (const bf16*)in, (bf16*)out, n, chunk, h->status, h->timeout_ns, loop)
                       : cudaLaunchKernelEx(&cfg, tp_all_sum_kernel, peers, rank, h->world, h->max_bytes,
                                            (const bf16*)in, (bf16*)out, n, chunk, h->status, h->timeout_ns, loop),
                    "tp_all_sum_kernel launch");
}

// Row-parallel quantized linear fused with its all-reduce (and the residual add):
//   y = residual + all_sum(x_shard @ dequantize(w_shard)^T)
// replacing QuantizedShardedToAllLinear.callAsFunction -> allSum
// (Libraries/MLXDistributedTP/LinearLayers.swift:198-205, Collectives.swift:27-32) followed by
// the decoder's residual add (Libraries/MLXLLM/Models/Llama.swift:110-114).  Decode sizes
// (M <= 32): the GEMV pushes its bf16 partial rows straight into every rank's slot
// over NVLink and reduces them in the same kernel.
static int tp_qmm_all_sum(void* tp, void* y, const void* x, const uint32_t* w, const void* scales,
                          const void* biases, int group_size, int bits, int64_t M, int64_t N, int64_t K,
                          const void* residual, int swiglu, void* stream);

extern "C" int vmlx_tp_quantized_matmul_all_sum(void* tp, void* y, const void* x, const uint32_t* w,
                                                const void* scales, const void* biases, int group_size, int bits,
                                                int64_t M, int64_t N, int64_t K, const void* residual,
                                                void* stream) {
  return tp_qmm_all_sum(tp, y, x, w, scales, biases, group_size, bits, M, N, K, residual, 0, stream);
}

// The same with the MLP's SwiGLU fused into the staging of x: x is the [M, 2K] gate||up buffer.
extern "C" int vmlx_tp_quantized_matmul_swiglu_all_sum(void* tp, void* y, const void* gate_up, const uint32_t* w,
                                                       const void* scales, const void* biases, int group_size,
                                                       int bits, int64_t M, int64_t N, int64_t K,
                                                       const void* residual, void* stream) {
  return tp_qmm_all_sum(tp, y, gate_up, w, scales, biases, group_size, bits, M, N, K, residual, 1, stream);
}

static int tp_qmm_all_sum(void* tp, void* y, const void* x, const uint32_t* w, const void* scales,
                          const void* biases, int group_size, int bits, int64_t M, int64_t N, int64_t K,
                          const void* residual, int swiglu, void* stream) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  if (M == 0 && N > 0 && K > 0) return VMLX_OK;
  if (M < 1 || M > 32) return set_error(VMLX_E_UNSUPPORTED, "tp_quantized_matmul_all_sum: M=%lld (1..32)", (long long)M);
  if ((size_t)M * N * 8 > h->max_bytes)
    return set_error(VMLX_E_INVALID, "tp_quantized_matmul_all_sum: %lld x %lld output exceeds the %zu-byte slots",
                     (long long)M, (long long)N, h->max_bytes);
  if (h->world == 1)
    return swiglu ? vmlx_cuda_quantized_matmul_swiglu(y, x, w, scales, biases, group_size, bits, M, N, K, residual,
                                                      stream)
                  : vmlx_cuda_quantized_matmul_fused(y, x, w, scales, biases, group_size, bits, M, N, K, nullptr, 0.f,
                                                     residual, stream);
  if (!h->connected) return set_error(VMLX_E_STATE, "tp_quantized_matmul_all_sum: peers not connected");
  if (!y || !x || !w || !scales || !biases) return set_error(VMLX_E_INVALID, "tp_quantized_matmul_all_sum: null pointer");
  if (bits != 4 && bits != 8) return set_error(VMLX_E_UNSUPPORTED, "bits=%d not supported (4, 8)", bits);
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return set_error(VMLX_E_UNSUPPORTED, "group_size=%d not supported", group_size);
  if (N <= 0 || K <= 0 || K % group_size || !aligned(x, 16) || !aligned(w, 16))
    return set_error(VMLX_E_INVALID, "tp_quantized_matmul_all_sum: bad shape or alignment");
  QmvArgs a{(const bf16*)x, w, (const bf16*)scales, (const bf16*)biases, (bf16*)y, nullptr, nullptr,
            M, N, K, 0, 1, 1, nullptr, nullptr, 0.f, (const bf16*)residual};
  for (int r = 0; r < TP_MAX_WORLD; r++) a.tp_buf[r] = r < h->world ? h->peer_base[r] : nullptr;
  a.tp_rank = h->loop ? 0 : h->rank;
  a.tp_world = h->world;
  a.tp_slot_bytes = h->max_bytes;
  a.tp_slots_off = tp_fused_slots_off(h->max_bytes, h->world);
  a.tp_flags_off = tp_fused_flags_off(h->max_bytes, h->world);
  a.tp_epoch_off = tp_fused_epoch_off(h->max_bytes, h->world);
  a.tp_timeout_ns = h->timeout_ns;
  a.tp_status = h->status;
  a.x_swiglu = swiglu;
  a.tp_loop = h->loop ? 1 : 0;
  if (swiglu && K % 8) return set_error(VMLX_E_INVALID, "tp: SwiGLU input needs K a multiple of 8");
  return launch_qmv(a, QMV_DENSE, bits, group_size, 1, (int)M, as_stream(stream));
}

extern "C" int vmlx_tp_moe_combine_all_sum(void* tp, void* out, const void* y, const uint32_t* inverse_order,
                                           const void* scores, int scores_dtype, int64_t rows, int k, int64_t dims,
                                           const void* residual, void* stream) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  if (rows < 0 || k < 1 || dims < 1) return set_error(VMLX_E_INVALID, "tp_moe_combine_all_sum: bad shape");
  if (rows == 0) return VMLX_OK;
  if (!out || !y || !scores) return set_error(VMLX_E_INVALID, "tp_moe_combine_all_sum: null pointer");
  if (dims % 8 || !aligned(y, 16)) return set_error(VMLX_E_INVALID, "tp_moe_combine_all_sum: dims must be a multiple of 8");
  if (rows > 65535) return set_error(VMLX_E_UNSUPPORTED, "tp_moe_combine_all_sum: rows=%lld > 65535", (long long)rows);
  if (scores_dtype != VMLX_F32 && scores_dtype != VMLX_BF16)
    return set_error(VMLX_E_UNSUPPORTED, "tp_moe_combine_all_sum: scores dtype %d", scores_dtype);
  if (h->world == 1) {  // a size-1 group: the combine, then the residual add
    rc = vmlx_cuda_moe_combine(y, inverse_order, scores, scores_dtype, rows, k, dims, out, stream);
    if (rc || !residual) return rc;
    return vmlx_cuda_add(out, residual, out, rows * dims, stream);
  }
  if (!h->connected) return set_error(VMLX_E_STATE, "tp_moe_combine_all_sum: peers not connected");
  if ((size_t)rows * dims * 8 > h->max_bytes)
    return set_error(VMLX_E_INVALID, "tp_moe_combine_all_sum: %lld x %lld output exceeds the %zu-byte slots",
                     (long long)rows, (long long)dims, h->max_bytes);
  TpPeers peers;
  for (int r = 0; r < TP_MAX_WORLD; r++) peers.buf[r] = r < h->world ? h->peer_base[r] : nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((dims / 8 + 127) / 128), (unsigned)rows, h->loop ? (unsigned)h->world : 1u);
  cfg.blockDim = dim3(128);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr;
  // every CTA waits for the other ranks' words: all CTAs must be resident together (a
  // cooperative launch for the loopback group, whose ranks share this GPU)
  if (h->loop) {
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
  }
  const int rank = h->loop ? 0 : h->rank, loop = h->loop ? 1 : 0;
  cudaError_t e;
  if (scores_dtype == VMLX_F32)
    e = cudaLaunchKernelEx(&cfg, tp_moe_combine_kernel<float>, peers, rank, h->world, h->max_bytes, (const bf16*)y,
                           inverse_order, (const float*)scores, rows, k, dims, (const bf16*)residual, (bf16*)out,
                           h->status, h->timeout_ns, loop);
  else
    e = cudaLaunchKernelEx(&cfg, tp_moe_combine_kernel<bf16>, peers, rank, h->world, h->max_bytes, (const bf16*)y,
                           inverse_order, (const bf16*)scores, rows, k, dims, (const bf16*)residual, (bf16*)out,
                           h->status, h->timeout_ns, loop);
  return check_cuda(e, "tp_moe_combine_kernel launch");
}

extern "C" int vmlx_tp_status(void* tp, int* code) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  int rc = tp_check(h);
  if (rc) return rc;
  int v = 0;
  rc = check_cuda(cudaMemcpy(&v, h->status, sizeof(int), cudaMemcpyDeviceToHost), "tp_status: read");
  if (rc) return rc;
  if (code) *code = v;
  if (v) cudaMemset(h->status, 0, sizeof(int));
  return VMLX_OK;
}

extern "C" int vmlx_tp_destroy(void* tp) {
  TpHandle* h = static_cast<TpHandle*>(tp);
  if (!h) return VMLX_OK;
  for (int r = 0; r < h->world; r++)
    if (h->peer_opened[r]) cudaIpcCloseMemHandle(h->peer_base[r]);
  if (h->local) cudaFree(h->local);
  if (h->status) cudaFree(h->status);
  delete h;
  return VMLX_OK;
}
