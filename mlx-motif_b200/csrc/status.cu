// Status codes and per-thread error detail for the C ABI.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace motif {

static thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MOTIF_OK;
}

}  // namespace motif

extern "C" {

const char* motif_status_string(int status) {
  switch (status) {
    case MOTIF_OK: return "ok";
    case MOTIF_ERR_NULL: return "null pointer";
    case MOTIF_ERR_BAD_SHAPE: return "bad shape";
    case MOTIF_ERR_BAD_CONTRACT: return "shape outside kernel contract";
    case MOTIF_ERR_DTYPE: return "unsupported dtype";
    case MOTIF_ERR_CUDA: return "cuda error";
    case MOTIF_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

const char* motif_last_error(void) { return motif::g_last_error; }

int motif_abi_version(void) { return 3; }

}  // extern "C"
