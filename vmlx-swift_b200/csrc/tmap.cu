// tmap.cu -- host-side TMA tensor-map encoding.
//
// cuTensorMapEncodeTiled is a driver-API call; it is looked up through the
// runtime's driver entry-point query so the library itself does not link
// libcuda (it then loads on machines without a GPU driver, e.g. for the
// symbol/ABI checks).
#include <cudaTypedefs.h>

#include "tmap.cuh"

namespace vmlx {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) {
    set_error(VMLX_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error(VMLX_E_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return false;
  }
  return true;
}

}  // namespace vmlx
