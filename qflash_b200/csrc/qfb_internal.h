// Declarations shared by the library's translation units (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace qfb {

// element types of float tensors at the boundary (and the mask's bool)
enum : int { kF32 = 0, kF16 = 1, kBF16 = 2, kBool = 3 };

// int64 slots of the device parameter block written by the on-device
// parameter kernel (qflash_quant.cu) and read by the attention kernel
enum : int { P_STATUS = 0, P_RS = 1, P_EM = 2, P_RM = 3, P_LM = 4, P_ACCM = 5, P_MLIM = 6, P_SM = 8, P_QS = 9,
             P_KS = 10, P_OS = 11, P_INVSM = 12 };

// Dequantised output written by the attention epilogue instead of int8 O:
// out = int8(acc / l) * o_scale in `dtype` (kF32 / kF16 / kBF16) at element
// `strides`, o_scale taken from the device parameter block (P_OS).
struct OutSpec {
  void* p;
  int dtype;
  int64_t strides[4];
};

// Swin window bias built on the device (qflash/attention.py:58-76): entry
// (w, h, i, j) of the float mask is table[index[i * N + j], h] (+ mask[w, i, j]
// when a window mask is given, added in the promoted dtype of the two).
struct WindowBiasSpec {
  const void* table;
  int table_dtype;
  int64_t table_strides[2];
  int table_rows;
  const int64_t* index;  // [N * N], contiguous
  const void* mask;      // [nW, N, N] contiguous, or null
  int mask_dtype;
  int num_windows;
};

int set_err(int code, const char* fmt, ...);

// Restores the calling thread's current device when it goes out of scope: the
// entry points make the device that owns the data current for their launches
// and leave the caller's choice as they found it.
struct DeviceGuard {
  int prev = -1;
  DeviceGuard() {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      cudaGetLastError();
      prev = -1;
    }
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;
};
int select_device(const void* p, int* dev);

// Copies of the int8 output tensor in other GPUs' memory (CUDA IPC mappings of
// the same [Z, H, N, D] layout): the attention epilogue stores every O row into
// o and into each peer copy at the same offset (an all-gather fused into the
// kernel).  n <= kMaxPeers.
constexpr int kMaxPeers = 7;
// signal words of the gather barrier: one flag per rank, then the finished-CTA counter
constexpr int kSigCount = kMaxPeers + 1;
constexpr int kSigWords = kSigCount + 1;
struct PeerSpec {
  int n;
  int8_t* o[kMaxPeers];
  // Optional barrier inside the kernel (null sig: none): kSigWords uint32 per
  // rank, zero-initialised, mapped like the copies; sig_peer in o's order;
  // rank in [0, n]; epoch != 0, the same on every rank for one launch and
  // growing from launch to launch.
  uint32_t* sig;
  uint32_t* sig_peer[kMaxPeers];
  int rank;
  uint32_t epoch;
};
int sm_count(int dev);

// The attention launch behind qflash_i8_fwd_ex; with `dparams` the fixed-point
// constants are read from device memory (see KArgs::dparams).
int attention_fwd(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                  const int64_t q_strides[4], const int64_t k_strides[4], const int64_t v_strides[4],
                  const int64_t o_strides[4], const int64_t bias_strides[4], int bias_z_period, int Z, int H, int N,
                  int D, int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M, int64_t acc_M, int32_t l_shift,
                  int32_t acc_shift, uint32_t flags, const long long* dparams, const OutSpec* out, void* stream,
                  const PeerSpec* peers = nullptr);


// The on-device forward behind qflash_fwd_fused and the workspace it needs.
size_t fused_workspace_bytes(int bias_zb, int bias_hb, int N);
int fused_fwd(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
              const int64_t k_strides[4], const int64_t v_strides[4], const void* mask, int mask_dtype,
              const int64_t mask_strides[4], int mask_zb, int mask_hb, int mask_z_period, int8_t* q8, int8_t* k8,
              int8_t* v8, int8_t* o8, void* out, const int64_t out_strides[4], int Z, int H, int N, int D,
              double scale_log2e, int32_t l_shift, int32_t acc_shift, uint32_t flags, void* ws, size_t ws_bytes,
              void* stream, const WindowBiasSpec* wb = nullptr);

}  // namespace qfb
