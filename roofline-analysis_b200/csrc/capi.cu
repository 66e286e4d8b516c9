// capi.cu — library-wide C entry points: error strings, version, and the
// device status word read-back.
#include "b2d_decode.h"
#include "common.cuh"
#include "host_common.h"

extern "C" const char* b2d_error_string(int status) {
  switch (status) {
    case B2D_OK: return "ok";
    case B2D_ERR_INVALID_ARG: return "invalid argument (null pointer, bad size or stride)";
    case B2D_ERR_UNSUPPORTED: return "unsupported configuration (head_dim, dtype or group size)";
    case B2D_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case B2D_ERR_WORKSPACE: return "workspace missing or too small";
    case B2D_ERR_CUDA: return "CUDA runtime or driver call failed";
    case B2D_ERR_DEVICE_TIMEOUT: return "a kernel gave up waiting on a pipeline barrier";
    case B2D_ERR_DEVICE_BOUNDS: return "a block-table page id was out of range";
    case B2D_ERR_TOO_LARGE: return "size beyond the supported maximum";
    default: return "unknown b2d status";
  }
}

extern "C" const char* b2d_version(void) { return "b2d 0.1.0 sm_100a"; }

extern "C" int b2d_check_device_status(void* workspace, int clear, void* stream) {
  if (!workspace) return B2D_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int word = 0;
  if (cudaMemcpyAsync(&word, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return B2D_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return B2D_ERR_CUDA;
  if (clear && word != 0) {
    // A kernel that gave up waiting may have left split-merge arrival
    // counters half counted: clear them with the word.
    const size_t n = (word & 1) ? b2d::kWsHeaderBytes : sizeof(int);
    if (cudaMemsetAsync(workspace, 0, n, st) != cudaSuccess) return B2D_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return B2D_ERR_CUDA;
  }
  if (word & 1) return B2D_ERR_DEVICE_TIMEOUT;
  if (word & 2) return B2D_ERR_DEVICE_BOUNDS;
  return B2D_OK;
}

static_assert(b2d::kWsHeaderBytes == B2D_WORKSPACE_HEADER_BYTES,
              "workspace header size in b2d_decode.h");
