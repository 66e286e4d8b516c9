// host_common.cu — see host_common.h.
#include "host_common.h"

#include <map>
#include <mutex>
#include <tuple>
#include <utility>

namespace b2d {

static std::mutex g_mu;

int device_sm_count(int* sms) {
  static std::map<int, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  auto it = cache.find(dev);
  if (it == cache.end()) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    it = cache.emplace(dev, n).first;
  }
  *sms = it->second;
  return 0;
}

int ensure_dynamic_smem(const void* func, size_t bytes) {
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  auto key = std::make_pair(func, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return 0;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
      cudaSuccess)
    return -1;
  // Prefer the largest shared-memory carveout so two CTAs fit per SM.
  if (cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    return -1;
  done[key] = bytes;
  return 0;
}

int occupancy_per_sm(const void* func, int threads, size_t smem, int* per_sm) {
  static std::map<std::tuple<const void*, int, int, size_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> g(g_mu);
  auto key = std::make_tuple(func, dev, threads, smem);
  auto it = cache.find(key);
  if (it == cache.end()) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, smem) != cudaSuccess)
      return -1;
    it = cache.emplace(key, n).first;
  }
  *per_sm = it->second;
  return 0;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_tiled_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return -1;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base),
                  reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes),
                  reinterpret_cast<const cuuint32_t*>(box), estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -1;
}

}  // namespace b2d
