// Dense int8 tensor-core throughput of this GPU, for the roofline the
// benchmark reports the attention kernel's two contractions against
// (tl.dot(q, k) and tl.dot(p, v) at qflash/kernel.py:153,171 become
// tcgen05.mma kind::i8 here).
//
// One CTA per SM: thread 0 issues `iters` back-to-back tcgen05.mma kind::i8 of
// M = 128, N = 256, K = 32 (s8 x s8 -> s32, 2 * 128 * 256 * 32 ops each) from
// shared-memory operands into a TMEM accumulator, then waits (bounded) for
// their completion.  Operand values do not matter for the timing; shared memory
// is zero-filled.  No TMA, no multicast, no cluster.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/qflash_b200.h"
#include "qfb_internal.h"
#include "sm100_ptx.cuh"

namespace qfb {

constexpr int kPeakM = 128, kPeakN = 256, kPeakK = 32;

__global__ void __launch_bounds__(128) i8_mma_peak_kernel(int iters, unsigned* err) {
  __shared__ __align__(1024) uint8_t a_tile[kPeakM * kPeakK];
  __shared__ __align__(1024) uint8_t b_tile[kPeakN * kPeakK];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  for (int i = threadIdx.x; i < kPeakM * kPeakK / 16; i += blockDim.x) ((uint4*)a_tile)[i] = make_uint4(0, 0, 0, 0);
  for (int i = threadIdx.x; i < kPeakN * kPeakK / 16; i += blockDim.x) ((uint4*)b_tile)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();  // the MMAs read the tiles through the async proxy
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&done_bar), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) {
    // K-major tiles of 32-byte rows in the 32-byte swizzle layout (8-row groups 256 bytes apart)
    const uint64_t ad = smem_desc(smem_u32(a_tile), 16, 8 * kPeakK, kSw32);
    const uint64_t bd = smem_desc(smem_u32(b_tile), 16, 8 * kPeakK, kSw32);
    constexpr uint32_t idesc = idesc_i8(kPeakM, kPeakN, false);
    for (int i = 0; i < iters; ++i) mma_i8_ss(tmem, ad, bd, idesc, i > 0 ? 1u : 0u);
    tc_commit(smem_u32(&done_bar));
    if (!mbar_wait(smem_u32(&done_bar), 0)) atomicOr(err, 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

static __device__ unsigned g_peak_err;

}  // namespace qfb

extern "C" int qflash_i8_mma_peak(int ctas_per_sm, int iters, void* stream) {
  if (ctas_per_sm < 1 || ctas_per_sm > 2 || iters < 1 || iters > (1 << 24))
    return qfb::set_err(QFLASH_ERR_ARG, "ctas_per_sm in {1, 2} and iters in [1, 2^24]");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return qfb::set_err(QFLASH_ERR_DEVICE, "no device");
  unsigned* err = nullptr;
  if (cudaGetSymbolAddress((void**)&err, qfb::g_peak_err) != cudaSuccess)
    return qfb::set_err(QFLASH_ERR_DEVICE, "error word: %s", cudaGetErrorString(cudaGetLastError()));
  qfb::i8_mma_peak_kernel<<<qfb::sm_count(dev) * ctas_per_sm, 128, 0, (cudaStream_t)stream>>>(iters, err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return qfb::set_err(QFLASH_ERR_LAUNCH, "peak launch: %s", cudaGetErrorString(e));
  return QFLASH_OK;
}

extern "C" int qflash_i8_mma_peak_status(void* stream, uint32_t* out) {
  if (!out) return qfb::set_err(QFLASH_ERR_ARG, "null out");
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess)
    return qfb::set_err(QFLASH_ERR_LAUNCH, "sync: %s", cudaGetErrorString(cudaGetLastError()));
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, qfb::g_peak_err, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(qfb::g_peak_err, &zero, sizeof(zero)) != cudaSuccess)
    return qfb::set_err(QFLASH_ERR_LAUNCH, "error word: %s", cudaGetErrorString(cudaGetLastError()));
  *out = v;
  return QFLASH_OK;
}
