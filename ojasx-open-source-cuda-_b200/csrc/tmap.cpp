// tmap.cpp — TMA tensor-map encoding (see tmap.h).
#include "tmap.h"
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cstring>
#include <mutex>
#include <unordered_map>
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

namespace {
struct MapKey {
  int dev;
  int dtype;
  const void* base;
  uint64_t inner, outer, stride;
  uint32_t box_inner, box_outer;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
    size_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
  }
};
}  // namespace

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
  // Encoding costs microseconds of host time; decode-sized GEMMs are short enough
  // for that to show, so maps are cached by everything that defines them.
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash>* cache =
      new std::unordered_map<MapKey, CUtensorMap, MapKeyHash>();
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  cudaGetDevice(&key.dev);
  key.dtype = static_cast<int>(dtype);
  key.base = base;
  key.inner = inner;
  key.outer = outer;
  key.stride = row_stride_bytes;
  key.box_inner = box_inner;
  key.box_outer = box_outer;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache->find(key);
    if (it != cache->end()) {
      *map = it->second;
      return OJX_OK;
    }
  }
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
  std::lock_guard<std::mutex> g(mu);
  if (cache->size() >= 4096) cache->clear();
  (*cache)[key] = *map;
  return OJX_OK;
}

int make_tmap_2d_sw128_uncached(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
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
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OJX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return OJX_OK;
}

}  // namespace ojx
