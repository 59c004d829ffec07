// tmap.cu -- host-side TMA tensor-map encoding.
#include "tmap.cuh"

namespace vmlx {

bool make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = cuTensorMapEncodeTiled(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    const char* msg = nullptr;
    cuGetErrorString(r, &msg);
    set_error(VMLX_E_CUDA, "cuTensorMapEncodeTiled: %s", msg ? msg : "error");
    return false;
  }
  return true;
}

}  // namespace vmlx
