// gqa_static_scratch.cu — b2d_decode_gqa_static_scratch: the GQA decode for
// callers that cannot allocate device memory.
//
// Some callers have no way to hand the library a workspace: an inference
// plugin whose enqueue step is not allowed to allocate, a serving loop that
// reserved all free HBM for its KV-cache pool at start-up, or a thin FFI
// binding with no device allocator of its own (cudaMalloc would also
// synchronise the whole device in the middle of a decode step).  For them,
// the split partials, the row table and the status word live in one
// file-scope device array that every GPU which loads this library holds
// until the process exits.
//
// Limits and rules:
//   * kStaticScratchBytes (16 MiB) is the most workspace a call may need;
//     larger problems are rejected with B2D_ERR_TOO_LARGE (the regular
//     b2d_decode_gqa with a caller-provided workspace has no such limit).
//     16 MiB covers BASELINE configs 2, 3 and 5 (at most ~9.1 MB).
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and clears the
//     workspace header (status word and split-merge counters); make that
//     first call before any stream capture.
//   * In-kernel errors (a wait that ran out, a page id out of range) are
//     recorded in the array's status word: read and clear them with
//     b2d_static_scratch_check_status.
//   * All calls on a device share the one array, which keeps the previous
//     call's contents.  Calls whose work overlaps on the GPU (different
//     streams, or different host threads) race on it: serialise them.
//   * Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <mutex>

#include "b2d_decode.h"
#include "common.cuh"
#include "host_common.h"

namespace b2d {

constexpr size_t kStaticScratchBytes = 16u << 20;
constexpr int kMaxDevices = 64;

// Device-side scratch.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

static std::mutex g_scratch_mu;
static void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device (set up once).
static int static_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2D_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return B2D_ERR_TOO_LARGE;
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || p == nullptr)
      return B2D_ERR_CUDA;
    // The workspace header (status word, merge counters) must start at zero.
    if (cudaMemset(p, 0, kWsHeaderBytes) != cudaSuccess) return B2D_ERR_CUDA;
    if (cudaDeviceSynchronize() != cudaSuccess) return B2D_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return B2D_OK;
}

}  // namespace b2d

extern "C" int b2d_decode_gqa_static_scratch(const b2d_gqa_args* args, void* stream) {
  if (args == nullptr) return B2D_ERR_INVALID_ARG;
  size_t need = 0;
  int rc = b2d_gqa_workspace_bytes(args, &need);
  if (rc) return rc;
  if (need > b2d::kStaticScratchBytes) return B2D_ERR_TOO_LARGE;
  void* scratch = nullptr;
  rc = b2d::static_scratch_address(&scratch);
  if (rc) return rc;
  b2d_gqa_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = b2d::kStaticScratchBytes;
  return b2d_decode_gqa(&a, stream);
}

extern "C" int b2d_static_scratch_check_status(int clear, void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return B2D_ERR_CUDA;
  if (dev < 0 || dev >= b2d::kMaxDevices) return B2D_ERR_TOO_LARGE;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> g(b2d::g_scratch_mu);
    scratch = b2d::g_scratch_ptr[dev];
  }
  if (scratch == nullptr) return B2D_OK;  // no call has used the array on this device
  return b2d_check_device_status(scratch, clear, stream);
}
