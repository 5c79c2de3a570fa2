// Tensor-parallel exchange buffers: one device allocation per rank that every
// rank maps (CUDA IPC between the processes of one node), written by the
// peers' projection kernels over NVLink and read locally.
//
// The buffer is a dedicated cudaMalloc allocation (not a slice of a caching
// allocator's block), so its IPC handle maps exactly this buffer at offset 0.
#include <cuda_runtime.h>

#include <cstring>

#include "cascade_b200.h"
#include "gemv_device.cuh"
#include "internal.h"

using namespace cb;

extern "C" int cb_exchange_alloc(void** out) {
  if (!out) return fail(kErrInvalid, "cb_exchange_alloc: null output");
  *out = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, kXchgBytes);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_exchange_alloc: %s", cudaGetErrorString(e));
  // flags start at zero: the first sequence number a launch waits for is 1
  e = cudaMemset(p, 0, kXchgBytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(kErrCuda, "cb_exchange_alloc: %s", cudaGetErrorString(e));
  }
  *out = p;
  return kOk;
}

extern "C" int cb_exchange_free(void* buffer) {
  if (!buffer) return kOk;
  cudaError_t e = cudaFree(buffer);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_exchange_free: %s", cudaGetErrorString(e));
  return kOk;
}

extern "C" int cb_ipc_handle(const void* buffer, void* handle_out) {
  if (!buffer || !handle_out) return fail(kErrInvalid, "cb_ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(buffer));
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ipc_handle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == CB_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return kOk;
}

extern "C" int cb_ipc_open(const void* handle, void** buffer_out) {
  if (!handle || !buffer_out) return fail(kErrInvalid, "cb_ipc_open: null argument");
  *buffer_out = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ipc_open: %s", cudaGetErrorString(e));
  *buffer_out = p;
  return kOk;
}

extern "C" int cb_ipc_close(void* buffer) {
  if (!buffer) return kOk;
  cudaError_t e = cudaIpcCloseMemHandle(buffer);
  if (e != cudaSuccess) return fail(kErrCuda, "cb_ipc_close: %s", cudaGetErrorString(e));
  return kOk;
}
