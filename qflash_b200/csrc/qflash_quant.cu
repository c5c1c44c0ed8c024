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
#include <type_traits>
#include <cstring>

#include "../../include/qflash_b200.h"
#include "qfb_internal.h"

namespace qfb {

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
  int dense;             // rows packed one after another: element offset = row * D
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

// ---- vectorised forms: one thread per 16-byte vector of a row (rows 16-byte
// aligned; D * element size is a power of two >= 64, so vectors per row are too)
template <int T>
constexpr int kVecElems = T == kF32 ? 4 : 8;

// element e (0 .. kVecElems - 1) of a 16-byte vector as float
template <int T>
__device__ __forceinline__ float vec_elem(const uint4& u, int e) {
  if constexpr (T == kF32) {
    const uint32_t x = e == 0 ? u.x : (e == 1 ? u.y : (e == 2 ? u.z : u.w));
    return __int_as_float((int)x);
  } else {
    const uint32_t x = (e >> 1) == 0 ? u.x : ((e >> 1) == 1 ? u.y : ((e >> 1) == 2 ? u.z : u.w));
    const uint16_t b = (uint16_t)(x >> (16 * (e & 1)));
    if constexpr (T == kF16) return __half2float(__ushort_as_half(b));
    else return __bfloat162float(__ushort_as_bfloat16(b));
  }
}

// element offset of vector i of a [Z, H, N, D] strided tensor (vpr = 1 << vshift vectors per row)
__device__ __forceinline__ long long vec_offset(const Rows& r, unsigned i, int vshift, int H, int N, int ve) {
  if (r.dense) return (long long)i * ve;
  const unsigned row = i >> vshift, cv = i & ((1u << vshift) - 1);
  const unsigned c = row % (unsigned)N, t = row / (unsigned)N, b = t % (unsigned)H, a = t / (unsigned)H;
  return (long long)a * r.s0 + (long long)b * r.s1 + (long long)c * r.s2 + (long long)cv * ve;
}

template <int T>
__global__ void __launch_bounds__(256, 8) amax3v_kernel(Rows q, Rows k, Rows v, int H, int N, int vshift, unsigned nvec, float* partials) {
  using E = Elt<T>;
  constexpr int VE = kVecElems<T>;
  const Rows r = blockIdx.y == 0 ? q : (blockIdx.y == 1 ? k : v);
  const typename E::type* x = (const typename E::type*)r.p;
  float m = 0.f;
  // four vectors in flight per thread
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < nvec; i0 += 4 * stride) {
    uint4 u[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const unsigned i = i0 + j * stride;
      u[j] = i < nvec ? __ldg((const uint4*)(x + vec_offset(r, i, vshift, H, N, VE))) : make_uint4(0, 0, 0, 0);
    }
    if constexpr (T == kF32) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < VE; ++e) m = nmax(m, fabsf(vec_elem<T>(u[j], e)));
    } else {
      // |x| max on packed pairs in the input type (exact; NaN propagates like torch.amax)
      using P2 = typename std::conditional<T == kF16, __half2, __nv_bfloat162>::type;
      P2 mm2 = *(const P2*)&u[0].x;
      mm2 = __habs2(mm2);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t w[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) mm2 = __hmax2_nan(mm2, __habs2(*(const P2*)&w[c]));
      }
      if constexpr (T == kF16) {
        m = nmax(m, nmax(__low2float(mm2), __high2float(mm2)));
      } else {
        m = nmax(m, nmax(__low2float(mm2), __high2float(mm2)));
      }
    }
  }
  for (int o = 16; o; o >>= 1) m = nmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float sm[32];
  if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = sm[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) mm = nmax(mm, sm[i]);
    partials[blockIdx.y * gridDim.x + blockIdx.x] = mm;
  }
}

__device__ __forceinline__ bool fits_i32(double x) { return x >= -2147483648.0 && x <= 2147483647.0; }

// Scales and fixed-point constants (qflash/kernel.py:290-307); one block
// reduces the partial maxima, its first thread does the scalar math.
template <int T>
__device__ __noinline__ void block_params(const float* partials, int P, double scale_log2e, int l_shift, int acc_shift, int D,
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

template <int T>
__global__ void params_kernel(const float* partials, int P, double scale_log2e, int l_shift, int acc_shift, int D,
                              long long* dp) {
  block_params<T>(partials, P, scale_log2e, l_shift, acc_shift, D, dp);
}

// The scale of tensor t as block_params forms it: rt<T>(max of its P partial
// maxima * fl32(1/127)), reduced by one block.
template <int T>
__device__ float block_tensor_scale(const float* partials, int P, int t) {
  __shared__ float red[32];
  __shared__ float s_out;
  float m = 0.f;
  for (int i = threadIdx.x; i < P; i += blockDim.x) m = nmax(m, partials[t * P + i]);
  for (int o = 16; o; o >>= 1) m = nmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mm = nmax(mm, red[w]);
    s_out = rt<T>(mm * (float)(1.0 / 127.0));
  }
  __syncthreads();
  return s_out;
}

template <int T>
__global__ void __launch_bounds__(256, 8)
    quantize3v_kernel(Rows q, Rows k, Rows v, int H, int N, int D, int vshift, unsigned nvec, const float* partials,
                      int P, double scale_log2e, int l_shift, int acc_shift, long long* dp, int8_t* q8, int8_t* k8,
                      int8_t* v8) {
  using E = Elt<T>;
  constexpr int VE = kVecElems<T>;
  const int t = blockIdx.y;
  const Rows r = t == 0 ? q : (t == 1 ? k : v);
  int8_t* out = t == 0 ? q8 : (t == 1 ? k8 : v8);
  // The scale comes from the |max| pass's partial maxima (as block_params forms
  // it); block (0, 0) also writes the constants at the end, for the kernels
  // after this one.  When the constants cannot be formed the int8 values are
  // unused (the output is NaN).
  const float s = block_tensor_scale<T>(partials, P, t);
  const typename E::type* x = (const typename E::type*)r.p;
  // x / s: for 16-bit inputs with s in [2^-96, 2^96] as RN(x * RN(1/s)) plus one
  // FMA residual step, which equals the IEEE quotient for every 16-bit x with
  // 1/16 <= |x / s| <= 256 (checked exhaustively over all fp16 and bf16 pairs);
  // smaller quotients round to 0 either way and |x| <= amax bounds |x / s| by
  // about 127.  Otherwise the IEEE division.
  const bool fastdiv = T != kF32 && s >= 1.2621774e-29f && s <= 7.9228163e+28f;
  const float R = __frcp_rn(s);
  // one 16-byte vector of x: q = int8(clamp(round(x / s))), packed into the int8 output
  auto convert = [&](const uint4& u, unsigned i) {
    uint32_t packed[2] = {0u, 0u};
    if constexpr (T != kF32) {
      if (fastdiv) {
        // Here s is finite and |x| <= amax (a NaN or infinite x makes s NaN or
        // infinite), so q is finite: no NaN case.  Per pair of elements: q in
        // fp32, one rounding to T, clamp, then round half to even by adding
        // 1.5 * 2^10 in fp16 (its ulp is 1 on [1024, 2048)) or 1.5 * 2^23 in
        // fp32 for bf16; the int8 value is the low byte of that sum's bits.
        const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
        uint32_t b[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          float2 f;
          if constexpr (T == kF16) f = __half22float2(*(const __half2*)&wd[p]);
          else f = __bfloat1622float2(*(const __nv_bfloat162*)&wd[p]);
          const float q0a = __fmul_rn(f.x, R), q0b = __fmul_rn(f.y, R);
          const float qa = __fmaf_rn(__fmaf_rn(-q0a, s, f.x), R, q0a);
          const float qb = __fmaf_rn(__fmaf_rn(-q0b, s, f.y), R, q0b);
          if constexpr (T == kF16) {
            __half2 y = __floats2half2_rn(qa, qb);
            y = __hadd2(__hmin2(__hmax2(y, __float2half2_rn(-128.f)), __float2half2_rn(127.f)),
                        __float2half2_rn(1536.f));
            b[p] = *(const uint32_t*)&y;  // int8 values in bytes 0 and 2
          } else {
            const float2 y = __bfloat1622float2(__floats2bfloat162_rn(qa, qb));
            const float ca = __fadd_rn(fminf(fmaxf(y.x, -128.f), 127.f), 12582912.f);
            const float cb = __fadd_rn(fminf(fmaxf(y.y, -128.f), 127.f), 12582912.f);
            b[p] = __byte_perm(__float_as_uint(ca), __float_as_uint(cb), 0x0400);
          }
        }
        *(uint2*)(out + (long long)i * VE) = make_uint2(__byte_perm(b[0], b[1], 0x6420), __byte_perm(b[2], b[3], 0x6420));
        return;
      }
    }
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      const float xe = vec_elem<T>(u, e);
      float q;
      if (fastdiv) {
        const float q0 = __fmul_rn(xe, R);
        q = __fmaf_rn(__fmaf_rn(-q0, s, xe), R, q0);
      } else {
        q = __fdiv_rn(xe, s);
      }
      const float y = rt<T>(q);
      // clamp(round(y)) == round(clamp(y)) for round-half-even; the 1.5 * 2^23
      // add rounds to an integer; NaN gives 0 like the float -> int8 conversion
      const float c = fminf(fmaxf(y, -128.f), 127.f);
      const int v8 = y != y ? 0 : __float_as_int(__fadd_rn(c, 12582912.f)) - 0x4B400000;
      packed[e >> 2] |= (uint32_t)(v8 & 0xff) << (8 * (e & 3));
    }
    // the int8 output is contiguous: vector i covers bytes [i * VE, i * VE + VE)
    int8_t* o = out + (long long)i * VE;
    if constexpr (VE == 8) *(uint2*)o = make_uint2(packed[0], packed[1]);
    else *(uint32_t*)o = packed[0];
  };
  // four vectors in flight per thread: loads first, then convert and store
  const unsigned stride = gridDim.x * blockDim.x;
  for (unsigned i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < nvec; i0 += 4 * stride) {
    uint4 uv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const unsigned i = i0 + j * stride;
      uv[j] = i < nvec ? __ldg((const uint4*)(x + vec_offset(r, i, vshift, H, N, VE))) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (i0 + j * stride < nvec) convert(uv[j], i0 + j * stride);
  }
  if (blockIdx.x == 0 && blockIdx.y == 0) block_params<T>(partials, P, scale_log2e, l_shift, acc_shift, D, dp);
  (void)D;
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
__device__ __forceinline__ float load_any(const void* p, long long i, int dt) {
  if (dt == kF32) return ((const float*)p)[i];
  if (dt == kF16) return __half2float(((const __half*)p)[i]);
  return __bfloat162float(((const __nv_bfloat16*)p)[i]);
}
__device__ __forceinline__ float round_any(float x, int dt) {
  if (dt == kF16) return rt<kF16>(x);
  if (dt == kBF16) return rt<kBF16>(x);
  return x;
}

// The Swin window bias: the float mask entry from the table (plus the window
// mask), then the bias quantisation of bias_kernel in the mask's dtype, into
// [Zb, H, N, N4] with Zb = nW (or 1 without a window mask).  An index outside
// the table sets status 3 and is not read.
__global__ void window_bias_kernel(WindowBiasSpec wb, int H, int N, int N4, int nrows, long long* dp,
                                   int32_t* bias) {
  if (dp[P_STATUS] != 0) return;
  const float inv = __int_as_float((int)dp[P_INVSM]);
  const float log2e = 1.44269504f;
  const int rdt = !wb.mask || wb.mask_dtype == wb.table_dtype ? wb.table_dtype : kF32;  // promoted dtype
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < nrows;
       row += gridDim.x * (blockDim.x >> 5)) {
    const int i = row % N, t = row / N, h = t % H, w = t / H;
    int32_t* o = bias + (long long)row * N4;
    for (int j = threadIdx.x & 31; j < N; j += 32) {
      const long long idx = wb.index[(long long)i * N + j];
      if (idx < 0 || idx >= wb.table_rows) {
        dp[P_STATUS] = 3;
        o[j] = 0;
        continue;
      }
      float a = load_any(wb.table, idx * wb.table_strides[0] + (long long)h * wb.table_strides[1], wb.table_dtype);
      if (wb.mask) a = round_any(a + load_any(wb.mask, ((long long)w * N + i) * N + j, wb.mask_dtype), rdt);
      const bool masked = a < -100.0f;
      const float c = masked ? 0.0f : a;
      const float t1 = round_any(__fmul_rn(c, log2e), rdt);
      const float t2 = round_any(__fmul_rn(t1, inv), rdt);
      const float rr = round_any(rintf(t2), rdt);
      o[j] = masked ? kNegInfI : __float2int_rz(rr);
    }
  }
}

// NaN into every element of a strided output when the constants could not be
// formed (the attention kernel then wrote nothing); does nothing otherwise

int fused_fwd(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
              const int64_t k_strides[4], const int64_t v_strides[4], const void* mask, int mask_dtype,
              const int64_t mask_strides[4], int mask_zb, int mask_hb, int mask_z_period, int8_t* q8, int8_t* k8,
              int8_t* v8, int8_t* o8, void* out, const int64_t out_strides[4], int Z, int H, int N, int D,
              double scale_log2e, int32_t l_shift, int32_t acc_shift, uint32_t flags, void* ws, size_t ws_bytes,
              void* stream_, const WindowBiasSpec* wb) {
  cudaStream_t stream = (cudaStream_t)stream_;
  if (Z < 0 || H < 0 || N < 0) return set_err(QFLASH_ERR_ARG, "negative shape");
  if (!(D == 32 || D == 64 || D == 128 || D == 256)) return set_err(QFLASH_ERR_ARG, "head dim %d not in {32,64,128,256}", D);
  if (dtype < kF32 || dtype > kBF16) return set_err(QFLASH_ERR_ARG, "dtype %d not in {0 f32, 1 f16, 2 bf16}", dtype);
  if (Z == 0 || H == 0 || N == 0) return QFLASH_OK;
  // without o8 the attention epilogue writes `out` itself (at out_strides, or contiguous)
  if (!q || !k || !v || !q8 || !k8 || !v8 || !out || !ws || !q_strides || !k_strides || !v_strides)
    return set_err(QFLASH_ERR_ARG, "null pointer");
  if (o8 && out_strides && !(out_strides[3] == 1 && out_strides[2] == D && out_strides[1] == (int64_t)N * D &&
                             out_strides[0] == (int64_t)H * N * D))
    return set_err(QFLASH_ERR_ARG, "with o8 the output must be contiguous");
  if (out_strides && out_strides[3] != 1) return set_err(QFLASH_ERR_ARG, "output head-dim stride must be 1");
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1)
    return set_err(QFLASH_ERR_ARG, "innermost (head-dim) stride must be 1");
  if (l_shift < 1 || l_shift > 62 || acc_shift < 1 || acc_shift > 62) return set_err(QFLASH_ERR_ARG, "shift out of [1, 62]");
  if (wb) {
    // the window bias replaces a dense mask: [nW, H, N, N] with period nW, or [1, H, N, N]
    if (mask) return set_err(QFLASH_ERR_ARG, "a dense mask and a window bias at once");
    if (!wb->table || !wb->index || wb->table_rows < 1 || wb->table_dtype < kF32 || wb->table_dtype > kBF16 ||
        (wb->mask && (wb->mask_dtype < kF32 || wb->mask_dtype > kBF16 || wb->num_windows < 1 || Z % wb->num_windows)))
      return set_err(QFLASH_ERR_ARG, "window bias: table, index, float dtypes and a window count dividing Z=%d", Z);
    mask_zb = wb->mask ? wb->num_windows : 1;
    mask_hb = H;
    mask_z_period = wb->mask ? wb->num_windows : 0;
  }
  const bool has_mask = mask != nullptr || wb != nullptr;
  if (has_mask && !wb) {
    if (mask_dtype < kF32 || mask_dtype > kBool) return set_err(QFLASH_ERR_ARG, "mask dtype %d", mask_dtype);
    if (!mask_strides || mask_zb < 1 || mask_hb < 1 || (mask_hb != 1 && mask_hb != H))
      return set_err(QFLASH_ERR_ARG, "mask must broadcast to [Z, H, N, N]");
    if (mask_z_period > 0 ? mask_zb != mask_z_period : (mask_zb != 1 && mask_zb != Z))
      return set_err(QFLASH_ERR_ARG, "mask batch %d does not match Z=%d / period %d", mask_zb, Z, mask_z_period);
  }
  const size_t need = fused_workspace_bytes(has_mask ? mask_zb : 0, has_mask ? mask_hb : 0, N);
  if (ws_bytes < need) return set_err(QFLASH_ERR_ARG, "workspace of %zu bytes, %zu needed", ws_bytes, need);
  if ((uintptr_t)ws & 255) return set_err(QFLASH_ERR_ALIGN, "workspace must be 256-byte aligned");
  DeviceGuard keep_device;  // the caller's current device is restored on return
  int dev = 0;
  if (int rc0 = select_device(q, &dev)) return rc0;

  long long* dp = (long long*)ws;
  float* partials = (float*)((char*)ws + kParamsBytes);
  int32_t* bias = (int32_t*)((char*)ws + kParamsBytes + align256(3 * kMaxPartials * sizeof(float)));
  const long long nrows_ll = (long long)Z * H * N;
  if (nrows_ll > 0x7fffffffLL) return set_err(QFLASH_ERR_ARG, "too many rows");
  const int nrows = (int)nrows_ll;
  auto dense = [&](const int64_t* st) {
    return st[2] == D && st[1] == (int64_t)N * D && st[0] == (int64_t)H * N * D;
  };
  const Rows rq{q, q_strides[0], q_strides[1], q_strides[2], dense(q_strides)};
  const Rows rk{k, k_strides[0], k_strides[1], k_strides[2], dense(k_strides)};
  const Rows rv{v, v_strides[0], v_strides[1], v_strides[2], dense(v_strides)};
  const int threads = 256, wpb = threads / 32;
  int P = (nrows + wpb - 1) / wpb;
  const int cap = 8 * sm_count(dev);
  P = P < cap ? P : cap;
  P = P < kMaxPartials ? P : kMaxPartials;
  const dim3 g3(P, 3);
  const double sl = scale_log2e;
  // 16-byte vectors per row when every row of Q, K, V starts 16-byte aligned
  const int esz = dtype == kF32 ? 4 : 2;
  auto aligned = [&](const Rows& r) {
    return ((uintptr_t)r.p & 15) == 0 && (r.s0 * esz) % 16 == 0 && (r.s1 * esz) % 16 == 0 && (r.s2 * esz) % 16 == 0;
  };
  const long long nvec_ll = (long long)nrows * D * esz / 16;
  if (aligned(rq) && aligned(rk) && aligned(rv) && nvec_ll < (1ll << 31)) {
    const unsigned nvec = (unsigned)nvec_ll;
    int vshift = 0;
    while ((1 << vshift) < D * esz / 16) ++vshift;
    // one resident wave over the three tensors (8 blocks of 256 threads per
    // SM: both kernels use at most 32 registers); a grid of more blocks than
    // fit runs a partly empty last wave
    int PV = (int)((nvec + 1023) / 1024);
    const int capv = 8 * sm_count(dev) / 3;
    PV = PV < capv ? PV : capv;
    PV = PV < kMaxPartials ? PV : kMaxPartials;
    PV = PV < 1 ? 1 : PV;
    const dim3 gv(PV, 3);
    switch (dtype) {
      case kF32:
        amax3v_kernel<kF32><<<gv, 256, 0, stream>>>(rq, rk, rv, H, N, vshift, nvec, partials);
        quantize3v_kernel<kF32><<<gv, 256, 0, stream>>>(rq, rk, rv, H, N, D, vshift, nvec, partials, PV, sl, l_shift,
                                                        acc_shift, dp, q8, k8, v8);
        break;
      case kF16:
        amax3v_kernel<kF16><<<gv, 256, 0, stream>>>(rq, rk, rv, H, N, vshift, nvec, partials);
        quantize3v_kernel<kF16><<<gv, 256, 0, stream>>>(rq, rk, rv, H, N, D, vshift, nvec, partials, PV, sl, l_shift,
                                                        acc_shift, dp, q8, k8, v8);
        break;
      default:
        amax3v_kernel<kBF16><<<gv, 256, 0, stream>>>(rq, rk, rv, H, N, vshift, nvec, partials);
        quantize3v_kernel<kBF16><<<gv, 256, 0, stream>>>(rq, rk, rv, H, N, D, vshift, nvec, partials, PV, sl, l_shift,
                                                        acc_shift, dp, q8, k8, v8);
        break;
    }
  } else switch (dtype) {
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
    if (wb) {
      window_bias_kernel<<<bgrid, threads, 0, stream>>>(*wb, H, N, N4, brows, dp, bias);
    } else switch (mask_dtype) {
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
  const long long n = (long long)nrows * D;
  if (!o8) {
    OutSpec os;
    os.p = out;
    os.dtype = dtype;
    for (int i = 0; i < 4; ++i) os.strides[i] = out_strides ? out_strides[i] : st8[i];
    // on an error status the attention kernel writes the NaN output itself
    return attention_fwd(q8, k8, v8, nullptr, has_mask ? bias : nullptr, st8, st8, st8, nullptr,
                         has_mask ? bstr : nullptr, has_mask ? mask_z_period : 0, Z, H, N, D, 0, 0, 0, 0, 0, l_shift,
                         acc_shift, flags, dp, &os, stream);
  }
  int rc = attention_fwd(q8, k8, v8, o8, has_mask ? bias : nullptr, st8, st8, st8, st8, has_mask ? bstr : nullptr,
                         has_mask ? mask_z_period : 0, Z, H, N, D, 0, 0, 0, 0, 0, l_shift, acc_shift, flags, dp,
                         nullptr, stream);
  if (rc) return rc;
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
  if (!o8) return qfb::set_err(QFLASH_ERR_ARG, "null pointer");
  return qfb::fused_fwd(q, k, v, dtype, q_strides, k_strides, v_strides, mask, mask_dtype, mask_strides, mask_zb,
                        mask_hb, mask_z_period, q8, k8, v8, o8, out, nullptr, Z, H, N, D, scale_log2e, l_shift,
                        acc_shift, flags, workspace, workspace_bytes, stream);
}

extern "C" int qflash_fwd_fused_out(const void* q, const void* k, const void* v, int dtype,
                                    const int64_t q_strides[4], const int64_t k_strides[4],
                                    const int64_t v_strides[4], const void* mask, int mask_dtype,
                                    const int64_t mask_strides[4], int mask_zb, int mask_hb, int mask_z_period,
                                    int8_t* q8, int8_t* k8, int8_t* v8, void* out, const int64_t out_strides[4], int Z,
                                    int H, int N, int D, double scale_log2e, int32_t l_shift, int32_t acc_shift,
                                    uint32_t flags, void* workspace, size_t workspace_bytes, void* stream) {
  return qfb::fused_fwd(q, k, v, dtype, q_strides, k_strides, v_strides, mask, mask_dtype, mask_strides, mask_zb,
                        mask_hb, mask_z_period, q8, k8, v8, nullptr, out, out_strides, Z, H, N, D, scale_log2e,
                        l_shift, acc_shift, flags, workspace, workspace_bytes, stream);
}

extern "C" int qflash_fwd_fused_window(const void* q, const void* k, const void* v, int dtype,
                                       const int64_t q_strides[4], const int64_t k_strides[4],
                                       const int64_t v_strides[4], const void* table, int table_dtype,
                                       const int64_t table_strides[2], int table_rows, const int64_t* index,
                                       const void* window_mask, int window_mask_dtype, int num_windows, int8_t* q8,
                                       int8_t* k8, int8_t* v8, void* out, const int64_t out_strides[4], int Z, int H,
                                       int N, int D, double scale_log2e, int32_t l_shift, int32_t acc_shift,
                                       uint32_t flags, void* workspace, size_t workspace_bytes, void* stream) {
  if (!table_strides) return qfb::set_err(QFLASH_ERR_ARG, "null pointer");
  qfb::WindowBiasSpec wb;
  wb.table = table;
  wb.table_dtype = table_dtype;
  wb.table_strides[0] = table_strides[0];
  wb.table_strides[1] = table_strides[1];
  wb.table_rows = table_rows;
  wb.index = index;
  wb.mask = window_mask;
  wb.mask_dtype = window_mask_dtype;
  wb.num_windows = num_windows;
  return qfb::fused_fwd(q, k, v, dtype, q_strides, k_strides, v_strides, nullptr, -1, nullptr, 0, 0, 0, q8, k8, v8,
                        nullptr, out, out_strides, Z, H, N, D, scale_log2e, l_shift, acc_shift, flags, workspace,
                        workspace_bytes, stream, &wb);
}

extern "C" int qflash_fused_status(const void* workspace, void* stream, int64_t* status) {
  if (!workspace || !status) return qfb::set_err(QFLASH_ERR_ARG, "null pointer");
  // read through a pinned word of this thread (a copy into pageable memory is
  // staged by the driver); plain copy if pinned memory cannot be had
  static thread_local int64_t* pinned = nullptr;
  static thread_local bool tried = false;
  if (!tried) {
    tried = true;
    if (cudaHostAlloc((void**)&pinned, sizeof(int64_t), cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      pinned = nullptr;
    }
  }
  int64_t* dst = pinned ? pinned : status;
  cudaError_t e = cudaMemcpyAsync(dst, workspace, sizeof(int64_t), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return qfb::set_err(QFLASH_ERR_LAUNCH, "status read: %s", cudaGetErrorString(e));
  if (pinned) *status = *pinned;
  return QFLASH_OK;
}
