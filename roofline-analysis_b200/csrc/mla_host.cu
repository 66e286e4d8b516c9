// mla_host.cu — absorbed-MLA decode entry points (kernel pending).
#include "b2d_decode.h"

extern "C" int b2d_mla_workspace_bytes(const b2d_mla_args* a, size_t* bytes) {
  if (!a || !bytes) return B2D_ERR_INVALID_ARG;
  *bytes = 256;
  return B2D_OK;
}

extern "C" int b2d_decode_mla(const b2d_mla_args* a, void* stream) {
  (void)a;
  (void)stream;
  return B2D_ERR_UNSUPPORTED;
}
