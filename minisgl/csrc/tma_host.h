// Host-side TMA tensor-map creation with a small cache.
//
// The encoder is fetched from the driver through cudaGetDriverEntryPoint so
// the extension does not link libcuda directly. Maps are cached by their full
// description (address, extents, strides, box, swizzle): a CUDA-graph replay
// bakes the map into the kernel parameters, and eager calls hit the cache.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

namespace minisgl {

inline PFN_cuTensorMapEncodeTiled_v12000 tma_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      throw std::runtime_error("minisgl: cuTensorMapEncodeTiled is not available");
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct TmapKey {
  uint64_t addr;
  uint64_t dims[3];
  uint64_t strides[2];
  uint32_t box[3];
  int rank, dtype, swizzle;
  bool operator==(const TmapKey& o) const { return std::memcmp(this, &o, sizeof(TmapKey)) == 0; }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    const uint64_t* p = reinterpret_cast<const uint64_t*>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(TmapKey) / 8; ++i) h = (h ^ p[i]) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};

// Tiled map over a row-major tensor whose innermost dimension is dims[0].
// strides_bytes[i] is the byte stride of dimension i+1. The box is
// box[0] x box[1] (x box[2]) elements; swizzle applies to the 128-byte span.
inline CUtensorMap make_tmap(const void* base, CUtensorMapDataType dtype, int elem_bytes, int rank,
                             const uint64_t* dims, const uint64_t* strides_bytes,
                             const uint32_t* box, CUtensorMapSwizzle swizzle) {
  TmapKey key;
  std::memset(&key, 0, sizeof(key));
  key.addr = reinterpret_cast<uint64_t>(base);
  for (int i = 0; i < rank; ++i) key.dims[i] = dims[i], key.box[i] = box[i];
  for (int i = 0; i < rank - 1; ++i) key.strides[i] = strides_bytes[i];
  key.rank = rank;
  key.dtype = static_cast<int>(dtype);
  key.swizzle = static_cast<int>(swizzle);

  static std::mutex mu;
  static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;

  if ((key.addr & 15) != 0) throw std::runtime_error("minisgl: TMA base address must be 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i)
    if (strides_bytes[i] % 16 != 0) throw std::runtime_error("minisgl: TMA strides must be multiples of 16 bytes");
  if ((uint64_t)box[0] * elem_bytes % 16 != 0) throw std::runtime_error("minisgl: TMA inner box must span a multiple of 16 bytes");

  CUtensorMap map;
  cuuint64_t gdim[3];
  cuuint64_t gstride[2];
  cuuint32_t bdim[3];
  cuuint32_t estride[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gdim[i] = dims[i], bdim[i] = box[i];
  for (int i = 0; i < rank - 1; ++i) gstride[i] = strides_bytes[i];
  CUresult r = tma_encoder()(&map, dtype, rank, const_cast<void*>(base), gdim, gstride, bdim,
                             estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    throw std::runtime_error("minisgl: cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  }
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, map);
  return map;
}

// 2-D bf16 map over a [rows, cols] matrix with row stride `ld` elements,
// box = [64 cols (128 bytes), box_rows], 128-byte swizzle.
inline CUtensorMap make_tmap_bf16_2d_sw128(const void* base, uint64_t rows, uint64_t cols,
                                           uint64_t ld, uint32_t box_rows) {
  uint64_t dims[2] = {cols, rows};
  uint64_t strides[1] = {ld * 2};
  uint32_t box[2] = {64, box_rows};
  return make_tmap(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 2, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// 3-D bf16 map that moves `kps` consecutive 64-column k-blocks of box_rows
// rows in one TMA instruction: dims {64, rows, cols / 64} with strides
// {ld * 2, 128} bytes, box {64, box_rows, kps}. The box lands in shared
// memory as kps back-to-back [box_rows][128 B] sub-tiles, each with the same
// 128-byte swizzle as the 2-D map (cols must be a multiple of 64).
inline CUtensorMap make_tmap_bf16_kblocks(const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                                          uint32_t box_rows, uint32_t kps) {
  uint64_t dims[3] = {64, rows, cols / 64};
  uint64_t strides[2] = {ld * 2, 128};
  uint32_t box[3] = {64, box_rows, kps};
  return make_tmap(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace minisgl
