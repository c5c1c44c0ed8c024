// On-device host math of qflash.forward (qflash/kernel.py:290-311, 328-336,
// 351): per-tensor scales, the fixed-point constants, int8 quantisation, bias
// quantisation and the final dequantisation, so that a whole forward runs on
// one stream without the reference's `.item()` synchronisation.
//
// Every step reproduces how torch evaluates the reference's expressions on a
// CUDA device, bit for bit:
//   x.abs().amax() / 127      max, then x * fl32(1/127) in fp32 (a CPU-scalar
//                             divisor is applied as a reciprocal), rounded to T
//   (q_scale * k_scale).item()  fp32 product rounded to T, widened to double
//   round(...) on doubles      round half to even (Python's round)
//   x / q_scale               fp32 division (q_scale is a device tensor), to T
//   torch.round, clamp, .to(int8)
//   mask * LOG2E / sm_scale   fp32 multiplies by LOG2E and by fl32(1/sm_scale) (double reciprocal),
//                             each rounded to the mask dtype
//   o * o_scale               fp32 product rounded to T
// where T is the input dtype (fp32, fp16 or bf16).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>

#include "../../include/qflash_b200.h"
#include "qfb_internal.h"

namespace qfb {

enum : int { kF32 = 0, kF16 = 1, kBF16 = 2, kBool = 3 };

// params block (int64 slots) written by params_kernel, read by the others
enum : int { P_STATUS = 0, P_RS = 1, P_EM = 2, P_RM = 3, P_LM = 4, P_ACCM = 5, P_MLIM = 6, P_SM = 8, P_QS = 9,
             P_KS = 10, P_OS = 11, P_INVSM = 12 };
constexpr int kParamsBytes = 256;
constexpr int kMaxPartials = 1024;  // blocks of the |max| reduction
constexpr int kNegInfI = -(1 << 20);

template <int T>
struct Elt;
template <>
struct Elt<kF32> {
  using type = float;
  static __device__ __forceinline__ float f(type x) { return x; }
  static __device__ __forceinline__ type t(float x) { return x; }
};
template <>
struct Elt<kF16> {
  using type = __half;
  static __device__ __forceinline__ float f(type x) { return __half2float(x); }
  static __device__ __forceinline__ type t(float x) { return __float2half_rn(x); }
};
template <>
struct Elt<kBF16> {
  using type = __nv_bfloat16;
  static __device__ __forceinline__ float f(type x) { return __bfloat162float(x); }
  static __device__ __forceinline__ type t(float x) { return __float2bfloat16_rn(x); }
};
// round a float to dtype T and back
template <int T>
__device__ __forceinline__ float rt(float x) {
  return Elt<T>::f(Elt<T>::t(x));
}

struct Rows {
  const void* p;
  long long s0, s1, s2;  // element strides of Z, H, N (the head dim is contiguous)
};

// max with NaN propagation (torch.amax returns NaN if any element is NaN)
__device__ __forceinline__ float nmax(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}

// |max| of Q, K, V (blockIdx.y picks the tensor); one warp per row of D elements
template <int T>
__global__ void amax3_kernel(Rows q, Rows k, Rows v, int H, int N, int D, int nrows, float* partials) {
  using E = Elt<T>;
  const Rows r = blockIdx.y == 0 ? q : (blockIdx.y == 1 ? k : v);
  const typename E::type* x = (const typename E::type*)r.p;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  float m = 0.f;
  for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < nrows; row += gridDim.x * wpb) {
    const int c = row % N, t = row / N, b = t % H, a = t / H;
    const typename E::type* p = x + a * r.s0 + b * r.s1 + c * r.s2;
    for (int d = lane; d < D; d += 32) m = nmax(m, fabsf(E::f(p[d])));
  }
  for (int o = 16; o; o >>= 1) m = nmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float sm[32];
  if (lane == 0) sm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = sm[0];
    for (int i = 1; i < wpb; ++i) mm = nmax(mm, sm[i]);
    partials[blockIdx.y * gridDim.x + blockIdx.x] = mm;
  }
}

__device__ __forceinline__ bool fits_i32(double x) { return x >= -2147483648.0 && x <= 2147483647.0; }

// Scales and fixed-point constants (qflash/kernel.py:290-307); one block
// reduces the partial maxima, its first thread does the scalar math.
template <int T>
__global__ void params_kernel(const float* partials, int P, double scale_log2e, int l_shift, int acc_shift, int D,
                              long long* dp) {
  __shared__ float red[3][32];
  float m[3] = {0.f, 0.f, 0.f};
  for (int i = threadIdx.x; i < P; i += blockDim.x)
    for (int t = 0; t < 3; ++t) m[t] = nmax(m[t], partials[t * P + i]);
  for (int t = 0; t < 3; ++t) {
    float v = m[t];
    for (int o = 16; o; o >>= 1) v = nmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[t][threadIdx.x >> 5] = v;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int t = 0; t < 3; ++t) {
    m[t] = red[t][0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m[t] = nmax(m[t], red[t][w]);
  }
  const float inv127 = (float)(1.0 / 127.0);
  const float qs = rt<T>(m[0] * inv127), ks = rt<T>(m[1] * inv127), os = rt<T>(m[2] * inv127);
  const float qk = rt<T>(qs * ks);
  const double sm = scale_log2e * (double)qk;
  long long st = 0;
  long long rs = 0, eM = 0, rM = 0, lM = 0, aM = 0, mlim = 0;
  if (sm == 0.0) {
    st = 1;  // 1.0 / sm_scale: ZeroDivisionError in the reference
  } else if (!(fabs(sm) < INFINITY)) {
    st = 2;  // NaN / inf: round() raises in the reference
  } else {
    const double rsd = rint(1.0 / sm);
    const double eMd = rint(-sm * 65536.0);
    const double rMd = rint(sm * 127.0 * 65536.0);
    if (rsd == 0.0) {
      st = 1;  // (1 << L_SHIFT) / sm_rscale
    } else if (!fits_i32(rsd) || !fits_i32(eMd) || !fits_i32(rMd) || rsd < 0.0) {
      st = 2;  // outside what the int32 kernel arguments hold
    } else {
      rs = (long long)rsd;
      eM = (long long)eMd;
      rM = (long long)rMd;
      lM = (long long)rint((double)(1ll << l_shift) / rsd);
      aM = (long long)rint((double)(1ll << acc_shift) / rsd);
      // the exp2_fast range bound (see attention_fwd)
      const long long S0 = ((long long)D << 14) > (1ll << 20) ? ((long long)D << 14) : (1ll << 20);
      const long long aem = -eM;
      const long long lim31 = (1ll << 31) - 1;
      long long X = aem > 0 ? (lim31 - 65536) / aem : lim31;
      const long long X2 = ((lim31 - 2ll * rs - 2) * 65536) / (aem * rs + 65536);
      X = X < X2 ? X : X2;
      mlim = eM > 0 ? -(1ll << 31) : X - S0;
      if (mlim > lim31) mlim = lim31;
      if (mlim < -(1ll << 31)) mlim = -(1ll << 31);
    }
  }
  dp[P_STATUS] = st;
  dp[P_RS] = rs;
  dp[P_EM] = eM;
  dp[P_RM] = rM;
  dp[P_LM] = lM;
  dp[P_ACCM] = aM;
  dp[P_MLIM] = mlim;
  dp[P_SM] = __double_as_longlong(sm);
  dp[P_QS] = __float_as_int(qs);
  dp[P_KS] = __float_as_int(ks);
  dp[P_OS] = __float_as_int(os);
  dp[P_INVSM] = __float_as_int((float)(1.0 / sm));  // torch forms the reciprocal of a scalar in double
}

// int8(clamp(round(x / scale), -128, 127)) into contiguous [Z, H, N, D]
template <int T>
__global__ void quantize3_kernel(Rows q, Rows k, Rows v, int H, int N, int D, int nrows, const long long* dp,
                                 int8_t* q8, int8_t* k8, int8_t* v8) {
  using E = Elt<T>;
  if (dp[P_STATUS] != 0) return;
  const int t = blockIdx.y;
  const Rows r = t == 0 ? q : (t == 1 ? k : v);
  int8_t* out = t == 0 ? q8 : (t == 1 ? k8 : v8);
  const float s = __int_as_float((int)dp[P_QS + t]);
  const typename E::type* x = (const typename E::type*)r.p;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < nrows; row += gridDim.x * wpb) {
    const int c = row % N, tt = row / N, b = tt % H, a = tt / H;
    const typename E::type* p = x + a * r.s0 + b * r.s1 + c * r.s2;
    int8_t* o = out + (long long)row * D;
    for (int d = lane; d < D; d += 32) {
      const float y = rt<T>(__fdiv_rn(E::f(p[d]), s));
      float rr = rt<T>(rintf(y));
      rr = rr < -128.f ? -128.f : (rr > 127.f ? 127.f : rr);  // NaN passes through; the conversion makes it 0
      o[d] = (int8_t)__float2int_rz(rr);
    }
  }
}

// int32 bias (qflash/kernel.py:328-336) of a mask broadcast to [Zb, Hb, N, N],
// written as [Zb, Hb, N, N4] with rows padded to a multiple of 4 elements
template <int M>
__global__ void bias_kernel(const void* mask, long long s0, long long s1, long long s2, long long s3, int Hb, int N,
                            int N4, int nrows, const long long* dp, int32_t* bias) {
  if (dp[P_STATUS] != 0) return;
  const float inv = __int_as_float((int)dp[P_INVSM]);
  const float log2e = 1.44269504f;
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < nrows;
       row += gridDim.x * (blockDim.x >> 5)) {
    const int i = row % N, t = row / N, hb = t % Hb, zb = t / Hb;
    int32_t* o = bias + (long long)row * N4;
    for (int j = threadIdx.x & 31; j < N; j += 32) {
      const long long off = zb * s0 + hb * s1 + i * s2 + j * s3;
      int32_t val;
      if constexpr (M == kBool) {
        val = ((const bool*)mask)[off] ? 0 : kNegInfI;
      } else {
        const float a = Elt<M>::f(((const typename Elt<M>::type*)mask)[off]);
        const bool masked = a < -100.0f;
        const float c = masked ? 0.0f : a;
        const float t1 = rt<M>(__fmul_rn(c, log2e));
        const float t2 = rt<M>(__fmul_rn(t1, inv));
        const float rr = rt<M>(rintf(t2));
        val = masked ? kNegInfI : __float2int_rz(rr);
      }
      o[j] = val;
    }
  }
}

// out = o8 * o_scale in dtype T, contiguous (NaN everywhere when the
// constants could not be formed, so the failure is visible)
template <int T>
__global__ void dequant_kernel(const int8_t* o8, long long n, const long long* dp, void* out) {
  using E = Elt<T>;
  const bool bad = dp[P_STATUS] != 0;
  const float os = __int_as_float((int)dp[P_OS]);
  typename E::type* y = (typename E::type*)out;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = E::t(bad ? __int_as_float(0x7fc00000) : (float)o8[i] * os);
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t fused_workspace_bytes(int bias_zb, int bias_hb, int N) {
  size_t b = kParamsBytes + align256(3 * kMaxPartials * sizeof(float));
  if (bias_zb > 0 && bias_hb > 0) b += align256((size_t)bias_zb * bias_hb * N * ((N + 3) / 4 * 4) * 4);
  return b;
}

// The fused forward; `ws` is device memory of at least fused_workspace_bytes().
int fused_fwd(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
              const int64_t k_strides[4], const int64_t v_strides[4], const void* mask, int mask_dtype,
              const int64_t mask_strides[4], int mask_zb, int mask_hb, int mask_z_period, int8_t* q8, int8_t* k8,
              int8_t* v8, int8_t* o8, void* out, int Z, int H, int N, int D, double scale_log2e, int32_t l_shift,
              int32_t acc_shift, uint32_t flags, void* ws, size_t ws_bytes, void* stream_) {
  cudaStream_t stream = (cudaStream_t)stream_;
  if (Z < 0 || H < 0 || N < 0) return set_err(QFLASH_ERR_ARG, "negative shape");
  if (!(D == 32 || D == 64 || D == 128 || D == 256)) return set_err(QFLASH_ERR_ARG, "head dim %d not in {32,64,128,256}", D);
  if (dtype < kF32 || dtype > kBF16) return set_err(QFLASH_ERR_ARG, "dtype %d not in {0 f32, 1 f16, 2 bf16}", dtype);
  if (Z == 0 || H == 0 || N == 0) return QFLASH_OK;
  if (!q || !k || !v || !q8 || !k8 || !v8 || !o8 || !out || !ws || !q_strides || !k_strides || !v_strides)
    return set_err(QFLASH_ERR_ARG, "null pointer");
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1)
    return set_err(QFLASH_ERR_ARG, "innermost (head-dim) stride must be 1");
  if (l_shift < 1 || l_shift > 62 || acc_shift < 1 || acc_shift > 62) return set_err(QFLASH_ERR_ARG, "shift out of [1, 62]");
  const bool has_mask = mask != nullptr;
  if (has_mask) {
    if (mask_dtype < kF32 || mask_dtype > kBool) return set_err(QFLASH_ERR_ARG, "mask dtype %d", mask_dtype);
    if (!mask_strides || mask_zb < 1 || mask_hb < 1 || (mask_hb != 1 && mask_hb != H))
      return set_err(QFLASH_ERR_ARG, "mask must broadcast to [Z, H, N, N]");
    if (mask_z_period > 0 ? mask_zb != mask_z_period : (mask_zb != 1 && mask_zb != Z))
      return set_err(QFLASH_ERR_ARG, "mask batch %d does not match Z=%d / period %d", mask_zb, Z, mask_z_period);
  }
  const size_t need = fused_workspace_bytes(has_mask ? mask_zb : 0, has_mask ? mask_hb : 0, N);
  if (ws_bytes < need) return set_err(QFLASH_ERR_ARG, "workspace of %zu bytes, %zu needed", ws_bytes, need);
  if ((uintptr_t)ws & 255) return set_err(QFLASH_ERR_ALIGN, "workspace must be 256-byte aligned");
  int dev = 0;
  if (int rc0 = select_device(q, &dev)) return rc0;

  long long* dp = (long long*)ws;
  float* partials = (float*)((char*)ws + kParamsBytes);
  int32_t* bias = (int32_t*)((char*)ws + kParamsBytes + align256(3 * kMaxPartials * sizeof(float)));
  const long long nrows_ll = (long long)Z * H * N;
  if (nrows_ll > 0x7fffffffLL) return set_err(QFLASH_ERR_ARG, "too many rows");
  const int nrows = (int)nrows_ll;
  const Rows rq{q, q_strides[0], q_strides[1], q_strides[2]};
  const Rows rk{k, k_strides[0], k_strides[1], k_strides[2]};
  const Rows rv{v, v_strides[0], v_strides[1], v_strides[2]};
  const int threads = 256, wpb = threads / 32;
  int P = (nrows + wpb - 1) / wpb;
  const int cap = 8 * sm_count(dev);
  P = P < cap ? P : cap;
  P = P < kMaxPartials ? P : kMaxPartials;
  const dim3 g3(P, 3);
  const double sl = scale_log2e;
  switch (dtype) {
    case kF32:
      amax3_kernel<kF32><<<g3, threads, 0, stream>>>(rq, rk, rv, H, N, D, nrows, partials);
      params_kernel<kF32><<<1, 256, 0, stream>>>(partials, P, sl, l_shift, acc_shift, D, dp);
      quantize3_kernel<kF32><<<g3, threads, 0, stream>>>(rq, rk, rv, H, N, D, nrows, dp, q8, k8, v8);
      break;
    case kF16:
      amax3_kernel<kF16><<<g3, threads, 0, stream>>>(rq, rk, rv, H, N, D, nrows, partials);
      params_kernel<kF16><<<1, 256, 0, stream>>>(partials, P, sl, l_shift, acc_shift, D, dp);
      quantize3_kernel<kF16><<<g3, threads, 0, stream>>>(rq, rk, rv, H, N, D, nrows, dp, q8, k8, v8);
      break;
    default:
      amax3_kernel<kBF16><<<g3, threads, 0, stream>>>(rq, rk, rv, H, N, D, nrows, partials);
      params_kernel<kBF16><<<1, 256, 0, stream>>>(partials, P, sl, l_shift, acc_shift, D, dp);
      quantize3_kernel<kBF16><<<g3, threads, 0, stream>>>(rq, rk, rv, H, N, D, nrows, dp, q8, k8, v8);
      break;
  }
  int64_t bstr[4] = {0, 0, 0, 1};
  if (has_mask) {
    const int N4 = (N + 3) / 4 * 4;
    const int brows = mask_zb * mask_hb * N;
    const int bgrid = (brows + wpb - 1) / wpb < cap ? (brows + wpb - 1) / wpb : cap;
    const int64_t* ms = mask_strides;
    switch (mask_dtype) {
      case kF32:
        bias_kernel<kF32><<<bgrid, threads, 0, stream>>>(mask, ms[0], ms[1], ms[2], ms[3], mask_hb, N, N4, brows, dp, bias);
        break;
      case kF16:
        bias_kernel<kF16><<<bgrid, threads, 0, stream>>>(mask, ms[0], ms[1], ms[2], ms[3], mask_hb, N, N4, brows, dp, bias);
        break;
      case kBF16:
        bias_kernel<kBF16><<<bgrid, threads, 0, stream>>>(mask, ms[0], ms[1], ms[2], ms[3], mask_hb, N, N4, brows, dp, bias);
        break;
      default:
        bias_kernel<kBool><<<bgrid, threads, 0, stream>>>(mask, ms[0], ms[1], ms[2], ms[3], mask_hb, N, N4, brows, dp, bias);
        break;
    }
    bstr[0] = mask_zb > 1 ? (int64_t)mask_hb * N * N4 : 0;
    bstr[1] = mask_hb > 1 ? (int64_t)N * N4 : 0;
    bstr[2] = N4;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_err(QFLASH_ERR_LAUNCH, "quantisation launch: %s", cudaGetErrorString(e));
  const int64_t st8[4] = {(int64_t)H * N * D, (int64_t)N * D, D, 1};
  int rc = attention_fwd(q8, k8, v8, o8, has_mask ? bias : nullptr, st8, st8, st8, st8, has_mask ? bstr : nullptr,
                         has_mask ? mask_z_period : 0, Z, H, N, D, 0, 0, 0, 0, 0, l_shift, acc_shift, flags, dp,
                         stream);
  if (rc) return rc;
  const long long n = (long long)nrows * D;
  const int dgrid = cap * 4;
  switch (dtype) {
    case kF32: dequant_kernel<kF32><<<dgrid, 256, 0, stream>>>(o8, n, dp, out); break;
    case kF16: dequant_kernel<kF16><<<dgrid, 256, 0, stream>>>(o8, n, dp, out); break;
    default: dequant_kernel<kBF16><<<dgrid, 256, 0, stream>>>(o8, n, dp, out); break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_err(QFLASH_ERR_LAUNCH, "dequantisation launch: %s", cudaGetErrorString(e));
  return QFLASH_OK;
}

}  // namespace qfb

extern "C" size_t qflash_fused_workspace_bytes(int mask_zb, int mask_hb, int N) {
  return qfb::fused_workspace_bytes(mask_zb, mask_hb, N);
}

extern "C" int qflash_fwd_fused(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
                                const int64_t k_strides[4], const int64_t v_strides[4], const void* mask,
                                int mask_dtype, const int64_t mask_strides[4], int mask_zb, int mask_hb,
                                int mask_z_period, int8_t* q8, int8_t* k8, int8_t* v8, int8_t* o8, void* out, int Z,
                                int H, int N, int D, double scale_log2e, int32_t l_shift, int32_t acc_shift,
                                uint32_t flags, void* workspace, size_t workspace_bytes, void* stream) {
  return qfb::fused_fwd(q, k, v, dtype, q_strides, k_strides, v_strides, mask, mask_dtype, mask_strides, mask_zb,
                        mask_hb, mask_z_period, q8, k8, v8, o8, out, Z, H, N, D, scale_log2e, l_shift, acc_shift,
                        flags, workspace, workspace_bytes, stream);
}

extern "C" int qflash_fused_status(const void* workspace, void* stream, int64_t* status) {
  if (!workspace || !status) return qfb::set_err(QFLASH_ERR_ARG, "null pointer");
  cudaError_t e = cudaMemcpyAsync(status, workspace, sizeof(int64_t), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return qfb::set_err(QFLASH_ERR_LAUNCH, "status read: %s", cudaGetErrorString(e));
  return QFLASH_OK;
}
