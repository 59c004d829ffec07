// sm100_util.cuh -- mbarrier / bulk-copy / cluster helpers (inline PTX, sm_90+ / sm_100a).
#pragma once
#include <cooperative_groups.h>

#include "common.cuh"

namespace vmlx {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase with the given parity to complete.  Returns false
// if the bound ran out (the caller records an error instead of hanging).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t max_iter = 1u << 26) {
  uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < max_iter; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// System-scope publish / observe for flags written over NVLink P2P, and the
// global nanosecond timer used to bound waits on peers.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Low-latency words: {payload (low 32 bits), epoch (high 32 bits)} written with one
// 8-byte system-scope store (single-copy atomic), so a reader that sees the epoch
// also sees the payload -- no fence or separate flag round trip.
__device__ __forceinline__ void st_ll(uint64_t* p, uint32_t payload, uint32_t epoch) {
  const uint64_t v = ((uint64_t)epoch << 32) | payload;
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_ll(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Poll a low-latency word until it carries epoch e; false once the deadline passes.
__device__ __forceinline__ bool wait_ll(const uint64_t* p, uint32_t e, uint64_t deadline_ns, uint32_t& payload) {
  for (uint32_t it = 0;; it++) {
    const uint64_t v = ld_ll(p);
    if ((uint32_t)(v >> 32) == e) { payload = (uint32_t)v; return true; }
    if ((it & 255) == 255 && globaltimer() > deadline_ns) return false;
  }
}

// Poll world low-latency words (p, p + stride, ...) until each carries epoch e, with
// every pending load in flight at once: one NVLink/L2 round trip per pass instead of
// one per word.  Returns the fp32 sum of their bf16 payloads in index (rank) order;
// false once the deadline passes.
template <int MAXW>
__device__ __forceinline__ bool wait_ll_sum(const uint64_t* p, size_t stride, int world, uint32_t e,
                                            uint64_t deadline_ns, float& sum) {
  uint32_t pay[MAXW];
  uint32_t pending = (world >= 32 ? ~0u : (1u << world) - 1u);
  for (uint32_t it = 0; pending; it++) {
    uint64_t v[MAXW];
#pragma unroll
    for (int r = 0; r < MAXW; r++)
      if (pending >> r & 1u) v[r] = ld_ll(p + r * stride);
#pragma unroll
    for (int r = 0; r < MAXW; r++)
      if ((pending >> r & 1u) && (uint32_t)(v[r] >> 32) == e) {
        pay[r] = (uint32_t)v[r];
        pending &= ~(1u << r);
      }
    if (pending && (it & 255) == 255 && globaltimer() > deadline_ns) return false;
  }
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < MAXW; r++)
    if (r < world) s += __bfloat162float(__ushort_as_bfloat16((unsigned short)pay[r]));
  sum = s;
  return true;
}

// Wait until *f - e >= 0 (wrapping 32-bit epochs); false once deadline_ns has passed.
__device__ __forceinline__ bool wait_flag_sys(const uint32_t* f, uint32_t e, uint64_t timeout_ns) {
  const uint64_t deadline = globaltimer() + timeout_ns;
  for (uint32_t it = 0;; it++) {
    if ((int32_t)(ld_acquire_sys(f) - e) >= 0) return true;
    if ((it & 1023) == 1023 && globaltimer() > deadline) return false;
  }
}

__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }


// ---- tcgen05 / TMEM helpers (kind::f16 MMAs with bf16 operands, fp32 accumulators) ----
constexpr int TC_UM = 128;  // UMMA M (weight rows per MMA = TMEM lanes)

// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzle layout
// (rows of 128 bytes, 16-byte chunk c of row r at c ^ (r & 7), 8-row groups 1024 bytes apart).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  // start address >> 4 | LBO (unused for swizzled K-major, 1) | SBO = 1024 B between
  // 8-row groups | descriptor version 1 | layout SWIZZLE_128B
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, M=128.
__host__ __device__ constexpr uint32_t tc_idesc(int bt) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bt >> 3) << 17) | ((uint32_t)(TC_UM >> 4) << 24);
}

// A from tensor memory (row = lane, K-major, two bf16 per column), B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }


__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

}  // namespace vmlx
