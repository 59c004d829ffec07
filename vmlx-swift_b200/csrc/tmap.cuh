// tmap.cuh -- TMA tensor-map encoding (host) and 2-D tiled loads (device).
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace vmlx {

// 2-D row-major tensor [outer rows][inner elements] with a row stride in bytes.
// Returns false (with vmlx_last_error set) if the driver rejects the map.
bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle);

// Tiled 2-D TMA load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
      "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace vmlx
