// Tensor-map encoding with a small cache (see tmap.h).
#include "tmap.h"

#include <cuda_runtime.h>

#include <mutex>
#include <string.h>
#include <unordered_map>

namespace {

struct Key {
  const void *base;
  uint64_t cols, rows, ld;
  uint32_t box_cols, box_rows;
  int elem, swz, dev, rank, box_kb, pad;
  bool operator==(const Key &o) const { return memcmp(this, &o, sizeof(Key)) == 0; }
};

struct KeyHash {
  size_t operator()(const Key &k) const {
    const uint64_t *p = reinterpret_cast<const uint64_t *>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(Key) / 8; i++)
      h = (h ^ p[i]) * 1099511628211ull;
    return (size_t)h;
  }
};

// The driver entry point, looked up through the runtime so the library has no link-time dependency on libcuda
// (it must load on machines without a GPU driver, where only its symbols are inspected).
bool lookup(const Key &k, CUtensorMap *out);
void store(const Key &k, const CUtensorMap &map);

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

std::mutex cache_mutex;
std::unordered_map<Key, CUtensorMap, KeyHash> cache;
constexpr size_t kCacheLimit = 1 << 14;

}  // namespace

bool kc_tmap_2d(CUtensorMap *out, const void *base, int elem_bytes, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  int dev = 0;
  cudaGetDevice(&dev);
  Key k;
  memset(&k, 0, sizeof(k));
  k.base = base, k.cols = cols, k.rows = rows, k.ld = ld_bytes, k.box_cols = box_cols, k.box_rows = box_rows;
  k.elem = elem_bytes, k.swz = swizzle128 ? 1 : 0, k.dev = dev;
  {
    std::lock_guard<std::mutex> lock(cache_mutex);
    auto it = cache.find(k);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType type = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  EncodeTiledFn encode = encode_fn();
  if (!encode)
    return false;
  CUresult r = encode(&map, type, 2, const_cast<void *>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                                      swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return false;
  std::lock_guard<std::mutex> lock(cache_mutex);
  if (cache.size() >= kCacheLimit)
    cache.clear();
  cache.emplace(k, map);
  *out = map;
  return true;
}

namespace {
bool lookup(const Key &k, CUtensorMap *out) {
  std::lock_guard<std::mutex> lock(cache_mutex);
  auto it = cache.find(k);
  if (it == cache.end())
    return false;
  *out = it->second;
  return true;
}
void store(const Key &k, const CUtensorMap &map) {
  std::lock_guard<std::mutex> lock(cache_mutex);
  if (cache.size() >= kCacheLimit)
    cache.clear();
  cache.emplace(k, map);
}
}  // namespace

bool kc_tmap_kblocks(CUtensorMap *out, const void *base, uint64_t k, uint64_t rows, uint64_t ld_bytes, uint32_t box_kb,
                     uint32_t box_rows) {
  if (k % 128)
    return false;
  int dev = 0;
  cudaGetDevice(&dev);
  Key key;
  memset(&key, 0, sizeof(key));
  key.base = base, key.cols = k, key.rows = rows, key.ld = ld_bytes, key.box_cols = 128, key.box_rows = box_rows;
  key.elem = 1, key.swz = 1, key.dev = dev, key.rank = 3, key.box_kb = (int)box_kb;
  if (lookup(key, out))
    return true;
  EncodeTiledFn encode = encode_fn();
  if (!encode)
    return false;
  CUtensorMap map;
  cuuint64_t dims[3] = {128, rows, k / 128};
  cuuint64_t strides[2] = {ld_bytes, 128};
  cuuint32_t box[3] = {128, box_rows, box_kb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return false;
  store(key, map);
  *out = map;
  return true;
}
