// qflash_fwd_fused without a caller-provided workspace.
//
// qflash_fwd_fused needs a small device workspace (the fixed-point constants,
// the partial maxima of the scale reduction and, with a mask, the int32 bias).
// Some callers cannot allocate one: their device memory is owned by a pool or
// runtime they cannot extend, or cudaMalloc/cudaFree (which can synchronise
// the whole device) are not allowed on their path.  For them this file keeps
// the workspace in a fixed array in the library's own device memory.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/qflash_b200.h"
#include "qfb_internal.h"

namespace qfb {

// 4 MiB, held on every GPU that loads the library until the process exits:
// the constants and partial maxima (12.5 KiB) plus an int32 bias of up to
// ~4 MiB (e.g. a Swin per-window bias, 64 windows x 3 heads x 49 x 52 x 4 B).
constexpr size_t kNoAllocScratchBytes = 4u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevs = 64;

// Device address of g_noalloc_scratch on `dev` (which must be current).  In host
// code the array's name is only a stand-in for the symbol, so its device
// address is looked up with cudaGetSymbolAddress.  The lookup is repeated on
// every call made outside a stream capture (a device reset reloads the module
// and may move the array); during a capture the address cached by the last
// call outside one is used, so a device's first call must come before any
// capture.
static int scratch_on(int dev, cudaStream_t stream, void** out) {
  static void* addr[kMaxDevs] = {nullptr};
  static std::mutex mu;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    cudaGetLastError();
    cs = cudaStreamCaptureStatusNone;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (cs == cudaStreamCaptureStatusNone || !addr[dev]) {
    if (cs != cudaStreamCaptureStatusNone)
      return set_err(QFLASH_ERR_UNSUPPORTED, "first no-alloc call on device %d inside a stream capture", dev);
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_err(QFLASH_ERR_DEVICE, "cudaGetSymbolAddress(scratch) on device %d: %s", dev, cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return QFLASH_OK;
}

}  // namespace qfb

extern "C" int qflash_fwd_fused_noalloc(const void* q, const void* k, const void* v, int dtype,
                                        const int64_t q_strides[4], const int64_t k_strides[4],
                                        const int64_t v_strides[4], const void* mask, int mask_dtype,
                                        const int64_t mask_strides[4], int mask_zb, int mask_hb, int mask_z_period,
                                        int8_t* q8, int8_t* k8, int8_t* v8, int8_t* o8, void* out, int Z, int H,
                                        int N, int D, double scale_log2e, int32_t l_shift, int32_t acc_shift,
                                        uint32_t flags, void* stream) {
  const bool has_mask = mask != nullptr;
  // the sizes first: the scratch requirement below assumes valid extents
  if (Z < 0 || H < 0 || N < 0) return qfb::set_err(QFLASH_ERR_ARG, "negative shape");
  if (has_mask && (mask_zb < 1 || mask_hb < 1))
    return qfb::set_err(QFLASH_ERR_ARG, "mask batch / head extents must be >= 1");
  const size_t need = qfb::fused_workspace_bytes(has_mask ? mask_zb : 0, has_mask ? mask_hb : 0, N);
  if (need > qfb::kNoAllocScratchBytes)
    return qfb::set_err(QFLASH_ERR_UNSUPPORTED,
                        "qflash_fwd_fused_noalloc: this call needs %zu bytes of scratch, the built-in scratch holds "
                        "%zu (a mask of %d x %d x %d x %d is too large); use qflash_fwd_fused with a workspace",
                        need, qfb::kNoAllocScratchBytes, mask_zb, mask_hb, N, N);
  if (Z == 0 || H == 0 || N == 0) return QFLASH_OK;
  if (!q) return qfb::set_err(QFLASH_ERR_ARG, "null pointer");
  qfb::DeviceGuard keep_device;  // the caller's current device is restored on return
  int dev = 0;
  if (int rc = qfb::select_device(q, &dev)) return rc;  // makes q's device current
  if (dev >= qfb::kMaxDevs) return qfb::set_err(QFLASH_ERR_DEVICE, "device %d", dev);
  void* ws = nullptr;
  if (int rc = qfb::scratch_on(dev, (cudaStream_t)stream, &ws)) return rc;
  if (!o8) return qfb::set_err(QFLASH_ERR_ARG, "null pointer");
  return qfb::fused_fwd(q, k, v, dtype, q_strides, k_strides, v_strides, mask, mask_dtype, mask_strides, mask_zb,
                        mask_hb, mask_z_period, q8, k8, v8, o8, out, nullptr, Z, H, N, D, scale_log2e, l_shift,
                        acc_shift, flags, ws, qfb::kNoAllocScratchBytes, stream);
}

extern "C" int qflash_fused_noalloc_status(const void* q, void* stream, int64_t* status) {
  if (!q || !status) return qfb::set_err(QFLASH_ERR_ARG, "null pointer");
  qfb::DeviceGuard keep_device;
  int dev = 0;
  if (int rc = qfb::select_device(q, &dev)) return rc;
  if (dev >= qfb::kMaxDevs) return qfb::set_err(QFLASH_ERR_DEVICE, "device %d", dev);
  void* ws = nullptr;
  if (int rc = qfb::scratch_on(dev, (cudaStream_t)stream, &ws)) return rc;
  return qflash_fused_status(ws, stream, status);
}
