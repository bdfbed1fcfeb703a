// tmap.h — host-side creation of TMA tensor maps (cuTensorMapEncodeTiled,
// fetched through the runtime's driver entry point so the library does not link
// libcuda directly).
#pragma once
#include <cuda.h>
#include <cstdint>

namespace ojx {

// 2-D row-major tensor: `inner` elements per row (contiguous), `outer` rows,
// rows `row_stride_bytes` apart.  Box = box_inner x box_outer elements, 128-byte
// swizzle, zero fill outside the tensor.  Returns OJX_OK or an error code (the
// message is recorded).  Constraints checked here: base 16-byte aligned,
// row stride a multiple of 16 bytes, box_inner * elem_bytes <= 128.
int make_tmap_2d_sw128(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                       const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);

// Same encoding without the descriptor cache: touches no host or device heap
// (the caller owns `map`).
int make_tmap_2d_sw128_uncached(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                                const void* base, uint64_t inner, uint64_t outer,
                                uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);

// 3-D: `batch` matrices of outer x inner, `batch_stride_bytes` apart (a multiple of
// 16); the box covers one matrix (box_inner x box_outer x 1).
int make_tmap_3d_sw128(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                       const void* base, uint64_t inner, uint64_t outer, uint64_t batch,
                       uint64_t row_stride_bytes, uint64_t batch_stride_bytes,
                       uint32_t box_inner, uint32_t box_outer);

}  // namespace ojx
