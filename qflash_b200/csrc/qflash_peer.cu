// CUDA IPC plumbing for the gathered output (qflash_i8_fwd_gather): a buffer
// allocated here can be mapped by the other processes of a job, one per GPU,
// so that each rank's attention epilogue stores its rows into every rank's
// copy over NVLink.  Host code only; the handles are exchanged by the caller
// (torch.distributed in qflash_b200/shard.py).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/qflash_b200.h"
#include "qfb_internal.h"

static_assert(sizeof(cudaIpcMemHandle_t) == QFLASH_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int qflash_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return qfb::set_err(QFLASH_ERR_ARG, "ipc_alloc: null argument or zero size");
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess)
    return qfb::set_err(QFLASH_ERR_DEVICE, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(cudaGetLastError()));
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {  // signal words start at 0
    const cudaError_t e = cudaGetLastError();
    cudaFree(p);
    return qfb::set_err(QFLASH_ERR_DEVICE, "cudaMemset: %s", cudaGetErrorString(e));
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    cudaFree(p);
    return qfb::set_err(QFLASH_ERR_DEVICE, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return QFLASH_OK;
}

extern "C" int qflash_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return qfb::set_err(QFLASH_ERR_ARG, "ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return qfb::set_err(QFLASH_ERR_DEVICE, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(cudaGetLastError()));
  *ptr = p;
  return QFLASH_OK;
}

extern "C" int qflash_ipc_close(void* ptr) {
  if (!ptr) return qfb::set_err(QFLASH_ERR_ARG, "ipc_close: null pointer");
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess)
    return qfb::set_err(QFLASH_ERR_DEVICE, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(cudaGetLastError()));
  return QFLASH_OK;
}

extern "C" int qflash_ipc_free(void* ptr) {
  if (!ptr) return qfb::set_err(QFLASH_ERR_ARG, "ipc_free: null pointer");
  if (cudaFree(ptr) != cudaSuccess)
    return qfb::set_err(QFLASH_ERR_DEVICE, "cudaFree: %s", cudaGetErrorString(cudaGetLastError()));
  return QFLASH_OK;
}
