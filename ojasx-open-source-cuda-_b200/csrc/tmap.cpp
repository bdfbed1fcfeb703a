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
  uint64_t inner, outer, batch, stride, batch_stride;
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

// Rank 2 (batch == 0) or rank 3 tiled map with 128-byte swizzle and zero fill.
int encode(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
           uint64_t inner, uint64_t outer, uint64_t batch, uint64_t row_stride_bytes,
           uint64_t batch_stride_bytes, uint32_t box_inner, uint32_t box_outer, bool cached) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    return set_error(OJX_ERR_INVALID, "TMA base address %p is not 16-byte aligned", base);
  if (row_stride_bytes % 16 != 0)
    return set_error(OJX_ERR_INVALID, "TMA row stride %llu bytes is not a multiple of 16",
                     (unsigned long long)row_stride_bytes);
  if (batch && batch_stride_bytes % 16 != 0)
    return set_error(OJX_ERR_INVALID, "TMA batch stride %llu bytes is not a multiple of 16",
                     (unsigned long long)batch_stride_bytes);
  if (box_inner * elem_bytes > 128 || box_inner == 0 || box_outer == 0 || box_outer > 256)
    return set_error(OJX_ERR_INVALID, "bad TMA box %u x %u", box_inner, box_outer);
  // Encoding costs microseconds of host time; decode-sized GEMMs are short enough
  // for that to show, so maps are cached by everything that defines them.
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash>* cache =
      new std::unordered_map<MapKey, CUtensorMap, MapKeyHash>();
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  if (cached) {
    cudaGetDevice(&key.dev);
    key.dtype = static_cast<int>(dtype);
    key.base = base;
    key.inner = inner;
    key.outer = outer;
    key.batch = batch;
    key.stride = row_stride_bytes;
    key.batch_stride = batch ? batch_stride_bytes : 0;
    key.box_inner = box_inner;
    key.box_outer = box_outer;
    std::lock_guard<std::mutex> g(mu);
    auto it = cache->find(key);
    if (it != cache->end()) {
      *map = it->second;
      return OJX_OK;
    }
  }
  auto fn = encode_fn();
  if (!fn) return set_error(OJX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint32_t rank = batch ? 3 : 2;
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {row_stride_bytes, batch_stride_bytes};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, rank, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(OJX_ERR_CUDA,
                     "cuTensorMapEncodeTiled failed (%d) for %llux%llux%llu box %ux%u", int(r),
                     (unsigned long long)inner, (unsigned long long)outer,
                     (unsigned long long)(batch ? batch : 1), box_inner, box_outer);
  if (cached) {
    std::lock_guard<std::mutex> g(mu);
    if (cache->size() >= 4096) cache->clear();
    (*cache)[key] = *map;
  }
  return OJX_OK;
}
}  // namespace

int make_tmap_2d_sw128(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                       const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  return encode(map, dtype, elem_bytes, base, inner, outer, 0, row_stride_bytes, 0, box_inner,
                box_outer, true);
}

int make_tmap_2d_sw128_uncached(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                                const void* base, uint64_t inner, uint64_t outer,
                                uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  return encode(map, dtype, elem_bytes, base, inner, outer, 0, row_stride_bytes, 0, box_inner,
                box_outer, false);
}

int make_tmap_3d_sw128(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                       const void* base, uint64_t inner, uint64_t outer, uint64_t batch,
                       uint64_t row_stride_bytes, uint64_t batch_stride_bytes,
                       uint32_t box_inner, uint32_t box_outer) {
  if (batch == 0) return set_error(OJX_ERR_INVALID, "TMA batch extent 0");
  return encode(map, dtype, elem_bytes, base, inner, outer, batch, row_stride_bytes,
                batch_stride_bytes, box_inner, box_outer, true);
}

}  // namespace ojx
