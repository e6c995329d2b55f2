// Host side of tensor_map.h: cuTensorMapEncodeTiled through the runtime's driver entry point
// (no link-time dependency on libcuda), with a small cache so a weight tensor is encoded once.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

#include "tensor_map.h"

namespace bolt {

namespace {

struct Key {
  const void* base;
  int64_t rows, row_bytes;
  int pieces;
  int piece_bytes;
  int box_rows;
  int device;
  bool operator==(const Key& o) const {
    return base == o.base && rows == o.rows && row_bytes == o.row_bytes && pieces == o.pieces &&
           piece_bytes == o.piece_bytes && box_rows == o.box_rows && device == o.device;
  }
};

struct KeyHash {
  size_t operator()(const Key& k) const {
    size_t h = std::hash<const void*>()(k.base);
    h ^= std::hash<int64_t>()(k.rows * 1315423911ll + k.row_bytes) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= static_cast<size_t>(k.pieces * 131 + k.device * 7 + k.piece_bytes + k.box_rows * 65537);
    return h;
  }
};

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

}  // namespace

bool row_tile_map(CUtensorMap* out, const void* base, int64_t rows, int64_t row_bytes, int pieces, int piece_bytes,
                  int box_rows) {
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, KeyHash> cache;
  if ((piece_bytes != 128 && piece_bytes != 64 && piece_bytes != 16) || row_bytes % piece_bytes != 0 || pieces < 1 ||
      pieces > 256 ||
      rows < 1 || box_rows < 1 || box_rows > 256 || (reinterpret_cast<uintptr_t>(base) & 15))
    return false;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{base, rows, row_bytes, pieces, piece_bytes, box_rows, dev};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  auto enc = encoder();
  if (!enc) return false;
  CUtensorMap m;
  const cuuint64_t pb = static_cast<cuuint64_t>(piece_bytes);
  cuuint64_t dims[3] = {pb, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(row_bytes) / pb};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes), pb};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(pb), static_cast<cuuint32_t>(box_rows), static_cast<cuuint32_t>(pieces)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   piece_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                      : (piece_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE),
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  *out = m;
  return true;
}

}  // namespace bolt
