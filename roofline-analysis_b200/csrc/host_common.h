// host_common.h — host helpers shared by the launchers: cached device
// properties, dynamic shared-memory opt-in, and TMA descriptor encoding
// through the driver entry point (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b2d {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// SM count of the current device (cached per device).  0 on success.
int device_sm_count(int* sms);

// Raise the dynamic shared-memory limit of `func` on the current device to at
// least `bytes` (cached per device and function).  0 on success.
int ensure_dynamic_smem(const void* func, size_t bytes);

// Resident CTAs per SM of `func` at this block size and dynamic shared
// memory on the current device (cached).  0 on success.
int occupancy_per_sm(const void* func, int threads, size_t smem, int* per_sm);

// cuTensorMapEncodeTiled with no interleave, the given swizzle, 256-byte L2
// promotion and zero out-of-bounds fill.  0 on success.
int encode_tiled_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE);

// Warps that merge one (row, query head) in the combine kernel: up to 8
// when there are few merges, so small batches still fill the GPU.
inline int combine_warps_per_merge(int64_t merges) {
  return merges <= 256 ? 8 : merges <= 512 ? 4 : merges <= 1024 ? 2 : 1;
}

}  // namespace b2d
