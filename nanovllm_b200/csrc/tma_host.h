// Host-side TMA tensor-map encoding.  The driver entry point cuTensorMapEncodeTiled is fetched once through
// the runtime (cudaGetDriverEntryPoint), so the extension does not link libcuda directly.  Maps are cached by
// (address, shape, box) because encoding happens on every call of an op whose operands did not change
// (weights, the KV arena).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <array>
#include <cstring>
#include <mutex>
#include <unordered_map>

namespace nvb {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled is not available from the CUDA driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct TmapKey {
  uint64_t addr;
  int rank;
  std::array<uint64_t, 5> dims;
  std::array<uint64_t, 4> strides;
  std::array<uint32_t, 5> box;
  int swizzle;
  int dtype;
  bool operator==(const TmapKey& o) const {
    return addr == o.addr && rank == o.rank && dims == o.dims && strides == o.strides && box == o.box &&
           swizzle == o.swizzle && dtype == o.dtype;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    size_t h = std::hash<uint64_t>()(k.addr) ^ (k.rank * 0x9E3779B97F4A7C15ull);
    for (auto d : k.dims) h = h * 1315423911u + d;
    for (auto d : k.box) h = h * 2654435761u + d;
    return h ^ (size_t)k.swizzle;
  }
};

// dims/strides follow the driver convention: dims[0] is the innermost (contiguous) dimension, strides[i] is
// the byte stride of dims[i+1].
inline CUtensorMap make_tmap(void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                             const uint64_t* strides_bytes, const uint32_t* box,
                             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  static std::mutex mu;
  TmapKey key{};
  key.addr = reinterpret_cast<uint64_t>(base);
  key.rank = rank;
  key.dims.fill(0);
  key.strides.fill(0);
  key.box.fill(0);
  for (int i = 0; i < rank; ++i) key.dims[i] = dims[i], key.box[i] = box[i];
  for (int i = 0; i + 1 < rank; ++i) key.strides[i] = strides_bytes[i];
  key.swizzle = (int)swizzle;
  key.dtype = (int)dtype;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  TORCH_CHECK((key.addr & 15) == 0, "TMA base address must be 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i) TORCH_CHECK(strides_bytes[i] % 16 == 0, "TMA strides must be multiples of 16 B");
  CUtensorMap m;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) d[i] = dims[i], b[i] = box[i], e[i] = 1;
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  CUresult r = get_encode_fn()(&m, dtype, rank, base, d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  return m;
}

// 2-D bf16 map over a row-major matrix [rows, cols] (row stride ``row_stride`` elements) with a box of
// [box_rows, 64 columns] and the 128-byte swizzle.
inline CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride,
                                     uint32_t box_rows, uint32_t box_cols = 64) {
  uint64_t dims[2] = {cols, rows};
  uint64_t strides[1] = {row_stride * 2};
  uint32_t box[2] = {box_cols, box_rows};
  return make_tmap(const_cast<void*>(base), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box);
}

}  // namespace nvb
