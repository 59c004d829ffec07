// common.cuh -- shared helpers of the sm_100a quantized-linear library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/vmlx_cuda.h"

namespace vmlx {

typedef __nv_bfloat16 bf16;
typedef __nv_bfloat162 bf162;

// Records an error message for vmlx_last_error() on the calling thread and
// returns `code` (mirrors mlx-c's int return + error handler).
int set_error(int code, const char* fmt, ...);
void clear_error();

// Raises a kernel's dynamic shared-memory limit on the current device (once per
// kernel and device; thread-safe).
int ensure_max_dynamic_smem(const void* func, int bytes);
// Multiprocessor count of the current device.
int sm_count();

// Programmatic dependent launch of the streaming kernels (vmlx_set_launch_overlap).
bool launch_overlap();

inline bool mode_is_affine(const char* mode) {
  return mode == nullptr || mode[0] == 0 || std::strcmp(mode, "affine") == 0;
}

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(VMLX_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return VMLX_OK;
}

inline int check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return set_error(VMLX_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return VMLX_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- device helpers ---------------------------------------------------------

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t bf162_as_u32(bf162 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ bf162 u32_as_bf162(uint32_t v) {
  return *reinterpret_cast<bf162*>(&v);
}

// Read-only streaming loads: weights are touched once per call, so keep them
// out of L1.
__device__ __forceinline__ uint32_t ldg_stream(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream(const uint2* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace vmlx
