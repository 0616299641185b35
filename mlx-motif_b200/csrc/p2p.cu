// Peer-to-peer exchange buffers for tensor parallelism inside one node.
//
// Each rank allocates one device buffer and exports a CUDA IPC handle; the ranks
// trade handles over the host process group and open each other's buffers, so a
// kernel can store straight into a peer's memory over NVLink (NVSwitch). The
// q4 GEMVs use this for the row-parallel outputs and the PolyNorm statistics
// (see qlinear.cu): no collective library call sits on the decode step.
#include "common.cuh"

#include <cstring>

using namespace motif;

extern "C" {

size_t motif_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int motif_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  MOTIF_REQUIRE(ptr && handle && bytes > 0, MOTIF_ERR_NULL, "ipc_alloc: null pointer or zero size");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "ipc_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return fail(MOTIF_ERR_CUDA, "ipc_alloc: %s", cudaGetErrorString(e));
  }
  return MOTIF_OK;
}

int motif_ipc_open(const void* handle, void** ptr) {
  MOTIF_REQUIRE(ptr && handle, MOTIF_ERR_NULL, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "ipc_open: %s", cudaGetErrorString(e));
  return MOTIF_OK;
}

int motif_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(e));
  return MOTIF_OK;
}

int motif_ipc_zero(void* ptr, size_t bytes, void* stream) {
  MOTIF_REQUIRE(ptr, MOTIF_ERR_NULL, "ipc_zero: null pointer");
  const cudaError_t e = cudaMemsetAsync(ptr, 0, bytes, as_stream(stream));
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "ipc_zero: %s", cudaGetErrorString(e));
  return MOTIF_OK;
}

int motif_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(MOTIF_ERR_CUDA, "ipc_free: %s", cudaGetErrorString(e));
  return MOTIF_OK;
}

}  // extern "C"
