// tmap.cpp — TMA tensor-map encoding (see tmap.h).
#include "tmap.h"
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <mutex>
#include "internal.h"

namespace ojx {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tmap_2d_sw128(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                       const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(OJX_ERR_INVALID, "TMA base address %p is not 16-byte aligned", base);
  if (row_stride_bytes % 16 != 0)
    return set_error(OJX_ERR_INVALID, "TMA row stride %llu bytes is not a multiple of 16",
                     (unsigned long long)row_stride_bytes);
  if (box_inner * elem_bytes > 128 || box_inner == 0 || box_outer == 0 || box_outer > 256)
    return set_error(OJX_ERR_INVALID, "bad TMA box %u x %u", box_inner, box_outer);
  auto fn = encode_fn();
  if (!fn) return set_error(OJX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(OJX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %llux%llu box %ux%u",
                     int(r), (unsigned long long)inner, (unsigned long long)outer, box_inner,
                     box_outer);
  return OJX_OK;
}

}  // namespace ojx
