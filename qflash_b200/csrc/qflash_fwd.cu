// qflash_b200: integer-only attention forward for B200 (sm_100a).
//
// Computes, bit for bit, the int8 output of QFlash's Triton kernels
// qflash_kernel (qflash/kernel.py:85-180) and qflash_masked_kernel
// (qflash/kernel.py:183-272): S = Q K^T in int32, an integer online softmax
// over 32-key chunks taken in order (the chunk width is part of the
// arithmetic), P requantised to int8, acc = rescale(acc) + P V in int32,
// O = int8(int32(fp32(acc) / fp32(l))).
//
// Structure of one CTA (192 threads) -- a persistent loop over work items, an
// item being one 128-query-row tile of one (z, h) head, or two heads of <= 64
// rows packed in one tile:
//   warps 0-3  softmax: warp w owns TMEM lanes [32w, 32w+32) = query rows of
//              the tile; acc lives in TMEM (one row per lane, DV columns)
//   warp 4     TMA producer: Q tile, then K/V chunk stages (and bias chunks)
//   warp 5     TMEM allocator and tcgen05.mma issuer
// Per 32-key chunk g (counted over the CTA's whole item sequence):
//   MMA   S_g = Q K_g^T            -> TMEM S slot (g & 1), 32 columns
//   soft  read S_g, exp2/requant, write packed int8 P_g into the same slot;
//         acc = rescale(acc, alpha_g) in place once PV_{g-1} has landed
//   MMA   acc += P_g (TMEM) V_g
// The MMA warp issues S_{g+1} before PV_g, so the tensor core computes the
// next scores while the softmax warps work on the current chunk.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/qflash_b200.h"
#include "qfb_internal.h"
#include "sm100_ptx.cuh"

namespace qfb {

constexpr int kBM = 128;             // query rows per tile = TMEM lanes
constexpr int kBN = 32;              // keys per chunk (BLOCK_N of the reference)
constexpr int kNegInf = -(1 << 20);  // qflash/kernel.py:137
constexpr int kThreads = 192;
constexpr uint32_t kWaitHintNs = 100000;  // longest sleep of one try_wait (0.1 ms)

__device__ unsigned int g_err;       // set when a bounded wait gives up

// Error codes written to g_err (bit set per site).
enum : unsigned { kErrQEmpty = 1, kErrKvEmpty = 2, kErrQFull = 4, kErrKvFull = 8, kErrPFull = 16,
                  kErrPvEmpty = 32, kErrSFull = 64, kErrPvFull = 128, kErrPeer = 256, kErrSelftest = 1u << 31 };

struct KArgs {
  int Z, H, N, nch, ntiles, nitems, ZH;
  int rpi;                   // query rows per work item (one head per tile): 128, or 64 / 32 for small grids
  int bias_hb, bias_zb;      // 1 if the bias has a real H / Z dimension, 0 if broadcast
  int bias_zmod;             // > 0: the bias batch index is z mod bias_zmod (Swin window period)
  int v_col0;                // first output column handled (head dim 256 runs as two halves)
  int8_t* o;
  long long os_z, os_h, os_n;
  int o_vec16;               // O rows 16-byte aligned
  int rs, eM, rM;            // sm_rscale, exp_M, req_M
  long long lM, accM;
  int ls, as;                // L_SHIFT, ACC_SHIFT
  unsigned flags;
  int fast_exp;              // 1: 6-op exp2 form exact for every chunk; 2: exact while the row max < m_lim
  int m_lim;
  // When set, the fixed-point constants come from device memory (written by
  // the on-device parameter kernel): [0] status (non-zero: do nothing),
  // [1] sm_rscale [2] exp_M [3] req_M [4] l_M [5] acc_M [6] m_lim, [11] o_scale.
  const long long* dparams;
  // When set (with dparams), the epilogue writes int8(acc / l) * o_scale in
  // out_dtype at these element strides instead of int8 O.
  void* out;
  long long ou_z, ou_h, ou_n;
  int out_dtype, out_vec16;
  float o_scale;
  // int8 O rows are also stored at these byte offsets from their address in o:
  // the same tensor in other GPUs' memory (PeerSpec), written over NVLink
  int n_peer;
  long long o_peer_off[kMaxPeers];
  int o_bulk;                // a warp's O rows are contiguous: staged in shared memory, written by bulk copies
  // Gather barrier (when sig is set): the last CTA to finish stores `epoch`
  // into slot sig_rank of every rank's signal words and waits (bounded) until
  // all sig_world slots of its own hold it, so the kernel completes only once
  // every rank's rows are in every copy.  sig[kSigCount] counts finished CTAs.
  uint32_t* sig;
  uint32_t* sig_peer[kMaxPeers];
  int sig_rank, sig_world;
  uint32_t epoch;
};

// ------------------------------------------------------------------ integer primitives
// Arithmetic right shift with the reference's semantics for any shift amount:
// PTX shr.s32 clamps amounts above 32 (read as unsigned) to 32 -> sign fill.
__device__ __forceinline__ int shr_clamp(int a, int b) {
  int d;
  asm("shr.s32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// exp2_i32_shift / exp2_i32_idiv (qflash/kernel.py:40-51), int32 wrap-around.
__device__ __forceinline__ int exp2_generic(int x, int rs, int eM, bool idiv) {
  int q;
  if (!idiv) {
    q = (int)((unsigned)x * (unsigned)eM) >> 16;
  } else {
    q = (int)(0u - (unsigned)x) / rs;
  }
  const int r = (int)((unsigned)x + (unsigned)q * (unsigned)rs);
  const int h = (int)((unsigned)(r >> 1) + (unsigned)rs);
  return shr_clamp(h, q);
}

// exp2_i32_shift of x = s - m in 6 integer ops.  With cm1 = -m*exp_M + 2^16
// and c3 = rs - m:  t1 = x*exp_M + 2^16, q1 = t1 >> 16 = q + 1,
// r2 = q1*rs + x + rs = r + 2*rs, and r2 >> q1 = ((r >> 1) + rs) >> q.
// Exact whenever none of those int32 values wraps and q >= 0; the host
// establishes that (|exp_M| <= 1023, exp_M <= 0, |x| <= 2^21, rs < 2^26).
__device__ __forceinline__ int exp2_fast(int s, int eM, int cm1, int rs, int c3) {
  const int t1 = (int)((unsigned)s * (unsigned)eM + (unsigned)cm1);
  const int q1 = t1 >> 16;
  const int u = (int)((unsigned)s + (unsigned)c3);
  const int r2 = (int)((unsigned)q1 * (unsigned)rs + (unsigned)u);
  return shr_clamp(r2, q1);
}

// requantize (qflash/kernel.py:62-64): int8((p * req_M + 2^15) >> 16) is byte 2
// of the wrapped 32-bit value; pack four of them into one word (byte i = key 4c+i).
__device__ __forceinline__ uint32_t requant_pack4(int e0, int e1, int e2, int e3, int rM) {
  const uint32_t p0 = (unsigned)e0 * (unsigned)rM + 32768u;
  const uint32_t p1 = (unsigned)e1 * (unsigned)rM + 32768u;
  const uint32_t p2 = (unsigned)e2 * (unsigned)rM + 32768u;
  const uint32_t p3 = (unsigned)e3 * (unsigned)rM + 32768u;
  const uint32_t t01 = __byte_perm(p0, p1, 0x0062);
  const uint32_t t23 = __byte_perm(p2, p3, 0x0062);
  return __byte_perm(t01, t23, 0x5410);
}

// scale_release_shift (qflash/kernel.py:67-69) with A = alpha * M already
// formed: int32(((int64)x * A + 2^(S-1)) >> S), all wrap-around.
__device__ __forceinline__ int rel_shift64(int x, unsigned long long A, int S) {
  const unsigned long long v = (unsigned long long)(long long)x * A + (1ull << (S - 1));
  return (int)((long long)v >> S);
}
// scale_release_shift on the FP64 pipe.  With Cd = 1.5*2^(51+S) + 2^(S-1):
// (double)x is exact (2^52 + (x + 2^31), minus 2^52 + 2^31); x*A + Cd stays in
// the binade [2^(51+S), 2^(52+S)) (|x*A| < 2^62, S >= 13), where one ulp is
// 2^(S-1), so the FMA rounded down yields 1.5*2^52 + w in ulps with
// w = floor((x*A + 2^(S-1)) / 2^(S-1)); bits [1, 33) of its encoding are
// floor(w / 2) = rel(x) (mod 2^32).  Needs 0 <= A < 2^31.
__device__ __forceinline__ int rel_fp64(int x, double Ad, double Cd) {
  const double xd = __hiloint2double(0x43300000, x ^ (int)0x80000000) - 4503601774854144.0;  // 2^52 + 2^31
  const double y = __fma_rd(xd, Ad, Cd);
  return (int)__funnelshift_r((uint32_t)__double2loint(y), (uint32_t)__double2hiint(y), 1);
}
// scale_release_idiv (qflash/kernel.py:72-74): (x * alpha) // rs, int32 product.
__device__ __forceinline__ int rel_idiv(int x, int alpha, int rs) {
  return (int)((unsigned)x * (unsigned)alpha) / rs;
}

// Final division (qflash/kernel.py:176) with IEEE rounding, as the reference's
// interpreted run computes it: int32(fp32(acc) / fp32(l)); a NaN or
// out-of-range quotient becomes INT32_MIN (numpy's conversion on x86).
__device__ __forceinline__ int div_ieee_to_i32(int acc, int l) {
  const float qf = __fdiv_rn(__int2float_rn(acc), __int2float_rn(l));
  return (qf >= -2147483648.0f && qf < 2147483648.0f) ? __float2int_rz(qf) : (int)0x80000000;
}

// NE int8 values (packed four per word) times o_scale, rounded to the output
// dtype, stored at dst: o * o_scale as torch evaluates it (qflash/kernel.py:351),
// the product in fp32 and one rounding to the dtype.
template <int NE>
__device__ __forceinline__ void store_dequant(void* dst, const uint32_t (&res)[NE / 4], float os, int dtype,
                                              bool vec16) {
  float f[NE];
#pragma unroll
  for (int i = 0; i < NE; ++i) f[i] = (float)(int8_t)(res[i >> 2] >> (8 * (i & 3))) * os;
  if (dtype == kF32) {
    float* d = (float*)dst;
    if (vec16) {
#pragma unroll
      for (int i = 0; i < NE / 4; ++i)
        *(float4*)(d + 4 * i) = make_float4(f[4 * i], f[4 * i + 1], f[4 * i + 2], f[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < NE; ++i) d[i] = f[i];
    }
  } else {
    uint32_t w[NE / 2];
#pragma unroll
    for (int i = 0; i < NE / 2; ++i) {
      if (dtype == kF16) {
        const __half2 h2 = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *(const uint32_t*)&h2;
      } else {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *(const uint32_t*)&b2;
      }
    }
    if (vec16) {
#pragma unroll
      for (int i = 0; i < NE / 8; ++i)
        *(uint4*)((uint8_t*)dst + 16 * i) = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else {
      uint16_t* d = (uint16_t*)dst;
#pragma unroll
      for (int i = 0; i < NE / 2; ++i) {
        d[2 * i] = (uint16_t)w[i];
        d[2 * i + 1] = (uint16_t)(w[i] >> 16);
      }
    }
  }
}

// The constants could not be formed (where the reference raises): the
// dequantised output of this pass (columns [v_col0, v_col0 + DV)) is NaN, the
// input dtype's rounding of an fp32 quiet NaN.  Grid-stride over all rows.
template <int DV>
__device__ void fill_out_nan(const KArgs& a) {
  const float qnan = __int_as_float(0x7fc00000);
  const long long n = (long long)a.Z * a.H * a.N * DV;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    const long long r = i / DV, d = i - r * DV;
    const long long t = r / a.N, c = r - t * a.N;
    const long long z = t / a.H, h = t - z * a.H;
    const long long off = z * a.ou_z + h * a.ou_h + c * a.ou_n + a.v_col0 + d;
    if (a.out_dtype == kF32) {
      ((float*)a.out)[off] = qnan;
    } else if (a.out_dtype == kF16) {
      ((__half*)a.out)[off] = __float2half_rn(qnan);
    } else {
      ((__nv_bfloat16*)a.out)[off] = __float2bfloat16_rn(qnan);
    }
  }
}

// Bounded wait on an mbarrier phase: each try_wait may sleep up to kWaitHintNs
// (waking when the phase completes), so a waiting warp takes few issue slots
// from the others; the abort flag and the ~2 s limit are checked once per
// sleep.  On giving up it records `code` in the error word, raises the CTA's
// abort flag (so the other roles leave too) and returns false.  (Inline: an
// out-of-line slow path measured 20-40 % slower, through the register
// allocation a call imposes on every wait site.)
__device__ __forceinline__ bool bounded_wait(uint32_t bar, uint32_t parity, unsigned code, volatile int* abort_flag) {
  if (mbar_try_wait_hint(bar, parity, kWaitHintNs)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_hint(bar, parity, kWaitHintNs)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_err, code);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// ------------------------------------------------------------------ kernel
// SEGS = 2 packs two heads (of N <= 64 rows each) into one 128-row tile:
// rows [0, 64) belong to head 2*item, rows [64, 128) to head 2*item + 1.
template <int DQK, int DV, bool BIAS, int SEGS, bool GATHER = false>
struct Cfg {
  static constexpr int SEG_ROWS = kBM / SEGS;
  static constexpr int QA = DQK < 128 ? DQK : 128;  // bytes per row of one swizzle atom
  static constexpr int NQA = DQK / QA;              // atoms along the QK contraction
  static constexpr int VA = DV;                     // DV <= 128: one atom
  static constexpr int S_COLS = 32 * SEGS;          // one S slot: a 32-column region per segment
  // Paired accumulator (when it fits a 256-column TMEM allocation, so that two
  // CTAs share an SM): acc element i of a row sits in TMEM column 2i, biased by
  // 2^31, and column 2i + 1 holds the constant high word of 2^(52 + S), so the
  // column pair reads as the double 2^(52+S) + (acc + 2^31) * 2^S and the
  // fixed-point rescale is one FMA per element.  The PV MMA then multiplies by
  // V2, V with a zero byte after every element (built in shared memory).
  // (one head per tile only: with two heads of at most two chunks per tile
  // (Swin windows) an item rescales once, and the plain layout measured faster)
  static constexpr bool ILV = SEGS == 1 && 2 * S_COLS + 2 * DV <= 256;
  static constexpr int ACC_W = ILV ? 2 * DV : DV;   // TMEM columns of acc per segment
  static constexpr int V2A = 2 * DV;                // bytes per key row of V2 (one swizzle atom)
  static constexpr int KVS = BIAS ? 4 : 8;          // K/V chunk stages
  static constexpr int Q_BYTES = kBM * DQK;
  static constexpr int K_SEG = kBN * DQK;
  static constexpr int V_SEG = kBN * DV;
  static constexpr int V2_SEG = ILV ? kBN * V2A : 0;
  static constexpr int K_BYTES = SEGS * K_SEG;
  static constexpr int V_BYTES = SEGS * V_SEG;
  static constexpr int V2_BYTES = SEGS * V2_SEG;
  static constexpr int B_BYTES = BIAS ? kBM * kBN * 4 : 0;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KVS * K_BYTES;
  static constexpr int OFF_V2 = OFF_V + KVS * V_BYTES;
  static constexpr int OFF_B = OFF_V2 + KVS * V2_BYTES;
  // int8 O rows of each softmax warp, staged for bulk copies (gathered output)
  static constexpr int STG_BYTES = GATHER && DV <= 64 ? 2 * 4 * 32 * DV : 0;  // two buffers per warp
  static constexpr int OFF_STG = OFF_B + KVS * B_BYTES;
  static constexpr int OFF_BAR = OFF_STG + STG_BYTES;
  static constexpr int NBAR = 2 + 2 + KVS + KVS + 2 + 2 + 2;
  static constexpr int THREADS = kThreads;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr int ACC_OFF = 2 * S_COLS;         // TMEM column of acc (ACC_W columns per segment)
  static constexpr int TMEM_NEED = ACC_OFF + SEGS * ACC_W;
  static constexpr int TMEM_COLS = TMEM_NEED <= 128 ? 128 : (TMEM_NEED <= 256 ? 256 : 512);
  // resident CTAs the register budget is compiled for: what TMEM allows, at most
  // 2 (a third CTA per SM measured slower: the SM's shared units saturate first)
  static constexpr int MIN_CTAS = (512 / TMEM_COLS) < 2 ? (512 / TMEM_COLS) : 2;
  // registers per thread for MIN_CTAS CTAs of THREADS threads (multiple of 8);
  // the d = 64 one-head-per-tile kernels (ViT, DeiT) measured fastest under a
  // lower cap: 152 with the paired accumulator (0.4 % faster than 168; 136 is
  // 13 % slower), 144 with the plain one
  static constexpr int REGS_FIT = (65536 / (MIN_CTAS * THREADS)) / 8 * 8 > 255 ? 255 : (65536 / (MIN_CTAS * THREADS)) / 8 * 8;
  static constexpr int REGS_D64 = ILV ? 152 : 144;
  static constexpr int MAX_REGS = (DQK == 64 && DV == 64 && SEGS == 1 && REGS_FIT > REGS_D64) ? REGS_D64 : REGS_FIT;
  static constexpr uint32_t IDESC_S = idesc_i8(kBM, kBN, false);
  static constexpr uint32_t IDESC_PV = idesc_i8(kBM, ILV ? V2A : DV, true);
  static constexpr uint32_t SWQ = QA == 32 ? kSw32 : (QA == 64 ? kSw64 : kSw128);
  static constexpr uint32_t SWV = VA == 32 ? kSw32 : (VA == 64 ? kSw64 : kSw128);
  static constexpr uint32_t SWV2 = V2A == 64 ? kSw64 : kSw128;
};

// Position of 16-byte chunk c of row r in a tile of `w`-byte rows stored with
// the w-byte TMA / UMMA swizzle (w = 32, 64, 128; tile base aligned to 8 * w):
// the chunk index is XORed with bits [7, 7 + log2(w / 16)) of the row's offset.
__device__ __forceinline__ int swz_chunk(int r, int c, int w) { return c ^ (((r * w) >> 7) & (w / 16 - 1)); }

// MODE selects the arithmetic the kernel is compiled for:
//   kGen      every QFLASH_* form, chosen at run time
//   kFast     default arithmetic, 6-op exp2 proven exact for every chunk
//   kChecked  default arithmetic, 6-op exp2 while the row max < m_lim, else the general form
//   kPlain    default arithmetic, general exp2 (bias kernels: the score range is unknown)
// Flags other than DIV_FULL / DIV_IEEE must be 0 for every mode but kGen.
enum Mode : int { kGen = 0, kFast = 1, kChecked = 2, kPlain = 3 };

// GATHER compiles the gathered-output path (KArgs::n_peer, o_bulk, sig): the
// copies into other GPUs' memory and the barrier over the ranks.
template <int DQK, int DV, bool BIAS, int MODE, int SEGS, bool GATHER>
__global__ void __launch_bounds__(Cfg<DQK, DV, BIAS, SEGS, GATHER>::THREADS)
    __maxnreg__((Cfg<DQK, DV, BIAS, SEGS, GATHER>::MAX_REGS))
    qfa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmB,
                   const KArgs a_in) {
  using C = Cfg<DQK, DV, BIAS, SEGS, GATHER>;
  // arguments are read in place (parameter space); the fixed-point constants
  // may come from the device parameter block instead
  const KArgs& a = a_in;
  int k_rs = a.rs, k_eM = a.eM, k_rM = a.rM, k_mlim = a.m_lim;
  long long k_lM = a.lM, k_accM = a.accM;
  float k_os = a.o_scale;
  if (a_in.dparams) {
    const long long* dp = a_in.dparams;
    if (dp[0] != 0) {  // the constants could not be formed (reported by the parameter kernel)
      if (a_in.out) fill_out_nan<DV>(a_in);
      return;
    }
    k_rs = (int)dp[1];
    k_eM = (int)dp[2];
    k_rM = (int)dp[3];
    k_lM = dp[4];
    k_accM = dp[5];
    k_mlim = (int)dp[6];
    k_os = __int_as_float((int)dp[P_OS]);
  }
  // kChecked (no bias): every score is an int8 dot product, |s| < DQK * 2^14,
  // so when m_lim is at least that the 6-op exp2 holds for every chunk and the
  // per-chunk vote is not needed
  const bool k_fast_all = MODE == kChecked && k_mlim >= (DQK << 14);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto q_full = [&](int i) { return bar0 + 8u * i; };
  auto q_empty = [&](int i) { return bar0 + 8u * (2 + i); };
  auto kv_full = [&](int i) { return bar0 + 8u * (4 + i); };
  auto kv_empty = [&](int i) { return bar0 + 8u * (4 + C::KVS + i); };
  auto s_full = [&](int i) { return bar0 + 8u * (4 + 2 * C::KVS + i); };
  auto p_full = [&](int i) { return bar0 + 8u * (6 + 2 * C::KVS + i); };
  auto acc_full = [&](int i) { return bar0 + 8u * (8 + 2 * C::KVS + i); };
  uint32_t* tmem_slot = (uint32_t*)(smem + C::OFF_MISC);
  volatile int* abort_flag = (volatile int*)(smem + C::OFF_MISC + 4);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(q_full(i), 1);
      mbar_init(q_empty(i), 1);
      mbar_init(s_full(i), 1);
      mbar_init(p_full(i), 4);
      mbar_init(acc_full(i), 1);
    }
    for (int i = 0; i < C::KVS; ++i) {
      mbar_init(kv_full(i), 1);
      mbar_init(kv_empty(i), 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto wait = [abort_flag](uint32_t bar, uint32_t parity, unsigned code) -> bool {
    return bounded_wait(bar, parity, code, abort_flag);
  };

  const int nch = a.nch;
  // Work item of round k for this CTA.  Rounds alternate direction over the
  // CTAs (k*G + b, then k*G + G-1-b), so a CTA alternates between the tiles of
  // a head (the last tile of a head is often partial) while every round still
  // covers one contiguous range of items (the tiles of a head run together and
  // share K/V in L2).  A negative value ends the loop.
  auto item_of = [&](int k) -> int {
    const long long G = gridDim.x, b = blockIdx.x;
    const long long it = (long long)k * G + ((k & 1) ? G - 1 - b : b);
    return it < a.nitems ? (int)it : -1;
  };
  // head (z, h) and first query row of segment `sg` of work item `item`; false if the segment is empty
  auto decode = [&](int item, int sg, int& z, int& h, int& row0) -> bool {
    int zh;
    if (SEGS == 1) {
      zh = item / a.ntiles;
      row0 = (item - zh * a.ntiles) * a.rpi;
    } else {
      zh = item * SEGS + sg;
      row0 = 0;
    }
    z = zh / a.H;
    h = zh - z * a.H;
    return zh < a.ZH;
  };

  if (warp == 4) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      if (BIAS) tma_prefetch_desc(&tmB);
      uint32_t kv_it = 0;
      int qi = 0;
      bool ok = true;
      for (int k = 0, item = item_of(0); ok && item >= 0; item = item_of(++k), ++qi) {
        // per segment: head (z, h), first query row, bias batch index; -1 = empty
        int sz[SEGS], sh[SEGS], sr[SEGS], sbz[SEGS];
        int nseg = 0;
#pragma unroll
        for (int sg = 0; sg < SEGS; ++sg) {
          if (decode(item, sg, sz[sg], sh[sg], sr[sg])) {
            ++nseg;
            sbz[sg] = a.bias_zb ? (a.bias_zmod ? sz[sg] % a.bias_zmod : sz[sg]) : 0;
          } else {
            sz[sg] = -1;
          }
        }
        const int qb = qi & 1;
        if (!(ok = wait(q_empty(qb), ((qi >> 1) & 1) ^ 1, kErrQEmpty))) break;
        mbar_arrive_expect_tx(q_full(qb), nseg * C::SEG_ROWS * DQK);
#pragma unroll
        for (int sg = 0; sg < SEGS; ++sg) {
          if (sz[sg] < 0) continue;
#pragma unroll
          for (int at = 0; at < C::NQA; ++at)
            tma_load_4d(sbase + C::OFF_Q + qb * C::Q_BYTES + at * kBM * C::QA + sg * C::SEG_ROWS * C::QA, &tmQ,
                        q_full(qb), at * C::QA, sr[sg], sh[sg], sz[sg]);
        }
        for (int j = 0; j < nch; ++j, ++kv_it) {
          const int st = kv_it % C::KVS;
          if (!(ok = wait(kv_empty(st), ((kv_it / C::KVS) & 1) ^ 1, kErrKvEmpty))) break;
          mbar_arrive_expect_tx(kv_full(st), nseg * (C::K_SEG + C::V_SEG + C::B_BYTES / SEGS));
#pragma unroll
          for (int sg = 0; sg < SEGS; ++sg) {
            if (sz[sg] < 0) continue;
#pragma unroll
            for (int at = 0; at < C::NQA; ++at)
              tma_load_4d(sbase + C::OFF_K + st * C::K_BYTES + sg * C::K_SEG + at * kBN * C::QA, &tmK, kv_full(st),
                          at * C::QA, j * kBN, sh[sg], sz[sg]);
            tma_load_4d(sbase + C::OFF_V + st * C::V_BYTES + sg * C::V_SEG, &tmV, kv_full(st), a.v_col0, j * kBN,
                        sh[sg], sz[sg]);
            if (BIAS)
              tma_load_4d(sbase + C::OFF_B + st * C::B_BYTES + sg * C::SEG_ROWS * 128, &tmB, kv_full(st), j * kBN,
                          sr[sg], a.bias_hb ? sh[sg] : 0, sbz[sg]);
          }
        }
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    // Lane 0 issues the MMAs.  With the paired accumulator all 32 lanes also
    // build V2 of each chunk (V with a zero byte after every element) once its
    // S MMA and the previous chunk's PV MMA are issued, so the build is off the
    // softmax -> PV -> rescale path; PV of the chunk is issued one step later.
    uint32_t g = 0;
    int qi = 0;
    bool ok = true;
    // acc (+)= P_gg V_gg straight into the TMEM accumulator, once the softmax
    // warps have written P_gg and rescaled acc; `init` starts a new item (lane 0)
    auto issue_pv = [&](uint32_t gg, bool init) -> bool {
      const int slot = gg & 1;
      const int st = gg % C::KVS;
      if (!wait(p_full(slot), (gg >> 1) & 1, kErrPFull)) return false;
      tc_fence_after();
#pragma unroll
      for (int sg = 0; sg < SEGS; ++sg) {
        // the paired accumulator starts each item from the pattern the softmax
        // warps store, so its PV MMAs always accumulate
        const uint64_t bdesc =
            C::ILV ? smem_desc(sbase + C::OFF_V2 + st * C::V2_BYTES + sg * C::V2_SEG, kBN * C::V2A, 8 * C::V2A,
                               C::SWV2)
                   : smem_desc(sbase + C::OFF_V + st * C::V_BYTES + sg * C::V_SEG, kBN * C::VA, 8 * C::VA, C::SWV);
        mma_i8_ts(tmem + C::ACC_OFF + sg * C::ACC_W, tmem + slot * C::S_COLS, bdesc, C::IDESC_PV,
                  (C::ILV || !init) ? 1u : 0u);
      }
      tc_commit(acc_full(slot));
      tc_commit(kv_empty(st));
      return true;
    };
    // V2 of stage st: lane r turns key row r of V (swizzled rows of DV bytes)
    // into row r of V2 (swizzled rows of 2 DV bytes), then makes it visible to
    // the tensor core (async proxy)
    auto build_v2 = [&](int st) {
#pragma unroll
      for (int sg = 0; sg < SEGS; ++sg) {
        const uint32_t src = sbase + C::OFF_V + st * C::V_BYTES + sg * C::V_SEG + lane * DV;
        const uint32_t dst = sbase + C::OFF_V2 + st * C::V2_BYTES + sg * C::V2_SEG + lane * C::V2A;
#pragma unroll
        for (int c = 0; c < DV / 16; ++c) {
          const uint4 x = lds128(src + (swz_chunk(lane, c, DV) << 4));
          sts128(dst + (swz_chunk(lane, 2 * c, C::V2A) << 4),
                 make_uint4(__byte_perm(x.x, 0, 0x4140), __byte_perm(x.x, 0, 0x4342), __byte_perm(x.y, 0, 0x4140),
                            __byte_perm(x.y, 0, 0x4342)));
          sts128(dst + (swz_chunk(lane, 2 * c + 1, C::V2A) << 4),
                 make_uint4(__byte_perm(x.z, 0, 0x4140), __byte_perm(x.z, 0, 0x4342), __byte_perm(x.w, 0, 0x4140),
                            __byte_perm(x.w, 0, 0x4342)));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
    };
    for (int k = 0, item = item_of(0); ok && item >= 0; item = item_of(++k), ++qi) {
      const int qb = qi & 1;
      bool ok0 = true;
      if (lane == 0) ok0 = wait(q_full(qb), (qi >> 1) & 1, kErrQFull);
      if (!(ok = __shfl_sync(0xffffffffu, ok0, 0))) break;
      tc_fence_after();
      const uint32_t qaddr = sbase + C::OFF_Q + qb * C::Q_BYTES;
      for (int j = 0; j < nch; ++j, ++g) {
        const int st = g % C::KVS;
        // every lane that reads the chunk (V2 build) observes its arrival itself
        if (C::ILV || lane == 0) ok0 = wait(kv_full(st), (g / C::KVS) & 1, kErrKvFull);
        if (!(ok = __all_sync(0xffffffffu, ok0))) break;
        if (lane == 0) {
          tc_fence_after();
          const uint32_t kaddr = sbase + C::OFF_K + st * C::K_BYTES;
#pragma unroll
          for (int sg = 0; sg < SEGS; ++sg) {
            const uint32_t dS = tmem + (g & 1) * C::S_COLS + sg * 32;
#pragma unroll
            for (int kk = 0; kk < DQK / 32; ++kk) {
              const int at = (kk * 32) / C::QA, off = (kk * 32) % C::QA;
              const uint64_t ad = smem_desc(qaddr + at * kBM * C::QA + off, 16, 8 * C::QA, C::SWQ);
              const uint64_t bd = smem_desc(kaddr + sg * C::K_SEG + at * kBN * C::QA + off, 16, 8 * C::QA, C::SWQ);
              mma_i8_ss(dS, ad, bd, C::IDESC_S, kk > 0 ? 1u : 0u);
            }
          }
          tc_commit(s_full(g & 1));
          if (j == nch - 1) tc_commit(q_empty(qb));
          if (j > 0) ok0 = issue_pv(g - 1, j == 1);
        }
        if (!(ok = __shfl_sync(0xffffffffu, ok0, 0))) break;
        if (C::ILV) build_v2(st);
      }
      if (ok) {
        if (lane == 0) ok0 = issue_pv(g - 1, nch == 1);
        ok = __shfl_sync(0xffffffffu, ok0, 0);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax warps
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    constexpr bool GEN = MODE == kGen;
    const bool exp_idiv = GEN && (a.flags & QFLASH_FLAG_EXP_IDIV);
    const bool l_idiv = GEN && (a.flags & QFLASH_FLAG_L_IDIV);
    const bool acc_idiv = GEN && (a.flags & QFLASH_FLAG_ACC_IDIV);
    const bool div_full = !(a.flags & QFLASH_FLAG_DIV_IEEE);

    const int rs = k_rs, eM = k_eM, rM = k_rM;
    const int S = a.as;
    // rescaling by alpha == rs is the identity while |acc| * |delta0| < 2^(S-1)
    const long long delta0 = (long long)rs * k_accM - (1ll << S);
    const float ident_lim = (float)(1ull << (S - 1)) * 0.999f / (float)(delta0 < 0 ? -delta0 : (delta0 ? delta0 : 1));
    const float two_mS = __int_as_float((127 - S) << 23);  // 2^-S
    const bool nch_launch_ok = a.nch <= 500;
    const int ident_lim_i = ident_lim >= 2.0e9f ? 0x7fffffff : (int)ident_lim;
    const float accM_ru = __ll2float_ru(k_accM < 0 ? -k_accM : k_accM);
    // paired-accumulator constants (see rescale): H, the high word of 2^(52+S);
    // 2^-S; 2^(52+S) + 2^(31+S); 2^(S-1); the range of A = alpha * acc_M for which
    // the one-FMA rescale is exact (empty unless 1 <= S <= 32)
    const uint32_t acc_hi = (uint32_t)(1075 + S) << 20;
    const double two_mSd = __longlong_as_double((1023ll - S) << 52);
    const double acc_anchor = __longlong_as_double(((1075ll + S) << 52) | (1ll << 31));
    const double acc_half = __longlong_as_double((1022ll + S) << 52);
    const bool s_pair = S >= 1 && S <= 32;
    const long long acc_a_lo = s_pair ? (S > 20 ? (1ll << (S - 20)) : 1ll) : (1ll << 62);
    const long long acc_a_hi = s_pair ? (2ll << S) - (S > 19 ? (1ll << (S - 19)) : 1ll) : 0ll;
    const bool accM32 = k_accM >= 1 && k_accM < (1ll << 31) && s_pair;
    const double accM_sd = (double)k_accM * two_mSd;                  // acc_M * 2^-S, exact
    const double cK = -4503601774854144.0 * (double)k_accM;           // -(2^52 + 2^31) acc_M, exact
    const float accM_f = (float)k_accM;
    const int alpha_lo = accM32 ? (int)((acc_a_lo + k_accM - 1) / k_accM) : 1;
    const int alpha_hi = accM32 ? (int)min((acc_a_hi - 1) / k_accM, (long long)0x7fffffff) : 0;
    const bool pair_range = accM32 && alpha_hi >= alpha_lo;
    // l takes the same one-FMA scale_release when its constants are acc's
    const bool l_pair = !l_idiv && s_pair && k_lM == k_accM && a.ls == S;
    // Bound on |acc| of a row for the kernels without a bias: while no P byte of
    // the row has been negative and every alpha is in [0, rs],
    //   |acc_j| <= 128 * (l_j + j + 1)  after chunk j.
    // Each step: |rel(x)| <= |x| A / 2^S + 1/2 and rel(l) >= l A / 2^S - 1/2, so
    // |acc_j| <= 128 (l_j - sum P_j) + K A / 2^S + 64.5 + |PV_j| with
    // |PV_j| <= 128 sum P_j; with A / 2^S <= rs acc_M / 2^S <= 1 + 2^-10 the
    // slack K grows by at most 128 per chunk for up to 500 chunks.
    const bool lb_launch = !BIAS && !GEN && s_pair && S >= 10 && nch_launch_ok &&
                           (long long)rs * k_accM - (1ll << S) <= (1ll << (S - 10));
    uint32_t g = 0;
    int stg_buf = 0;  // staging buffer of the next gathered-output epilogue
    bool ok = true;
    for (int k = 0, item = item_of(0); ok && item >= 0; item = item_of(++k)) {
      // warp -> segment (head) and its 32-row slice
      const int sg = SEGS == 1 ? 0 : warp / (4 / SEGS);
      int z, h, rbase;
      const bool seg_ok = decode(item, sg, z, h, rbase);
      const int row0 = rbase + (SEGS == 1 ? warp : warp % (4 / SEGS)) * 32;
      // an item of fewer than 128 rows leaves the warps past them idle (their
      // lanes hold the next item's rows, computed by another CTA)
      const bool active = seg_ok && row0 < a.N && (SEGS != 1 || warp * 32 < a.rpi);
      const int row = row0 + lane;
      const bool row_ok = row < a.N;
      int m = kNegInf, l = 1;
      // upper bound on max |acc| of this row, kept in fp32 with round-up margins
      float abound = 0.f;
      bool lb = lb_launch;  // the l-based bound on |acc| holds for this row
      // that bound after chunk jj - 1 (INT_MAX when it does not hold)
      auto acc_bound = [&](int jj) -> int {
        return (lb && (unsigned)(l + jj) < (1u << 23)) ? (l + jj) << 7 : 0x7fffffff;
      };
      // acc lives in TMEM (this warp's lanes, ACC_W columns); PV MMAs accumulate into it
      const uint32_t acc_base = tmem + lane_base + C::ACC_OFF + sg * C::ACC_W;
      if (C::ILV && active) {
        // paired accumulator: every item starts from acc = 0, i.e. (2^31, H) pairs;
        // the stores complete (tcgen05.wait::st of the P store) before this
        // warp releases the item's first P to the MMA warp.  The PV MMAs write
        // all 128 lanes, so the previous item's last PV must have landed first:
        // a warp with no rows in that item (past N) never waited for it.
        if (g > 0) {
          if (!(ok = wait(acc_full((g - 1) & 1), ((g - 1) >> 1) & 1, kErrPvFull))) break;
          tc_fence_after();
        }
        int pat[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) pat[i] = (i & 1) ? (int)acc_hi : (int)0x80000000u;
#pragma unroll
        for (int part = 0; part < C::ACC_W / 32; ++part) tmem_st32(acc_base + part * 32, pat);
      }

      // acc = rel(acc, alpha) in place, once PV_gg (the previous chunk's) has landed
      auto rescale = [&](uint32_t gg, int alpha, long long A, double Ad, double Cd, bool pair_ok) -> bool {
        if (!wait(acc_full(gg & 1), (gg >> 1) & 1, kErrPvFull)) return false;
        tc_fence_after();
        if constexpr (C::ILV) {
          // Paired accumulator: column pair (u, H) with u = x + 2^31 reads as the
          // double X = 2^(52+S) + u * 2^S.  With Ad = A * 2^-S and
          // Cd = 2^(52+S) + 2^(31+S) + 2^(S-1) - (2^52 + 2^31) * A,
          // X * Ad + Cd = x*A + 2^(S-1) + 2^(31+S) + 2^(52+S) exactly, which lies in
          // [2^(52+S), 2^(53+S)) (ulp 2^S) while |rel(x)| < 2^31; one FMA rounded
          // down therefore gives 2^(52+S) + 2^S * (2^31 + rel(x)): its low word is
          // the biased new acc and its high word is H again.  Ad is exact; Cd is
          // exact (a multiple of 2^(S-1) below 2^(52+S) in magnitude) for A in
          // [acc_a_lo, acc_a_hi); the first step forms Cd - 2^(S-1) exactly with an
          // FMA ((2^21 + 1) (2^S - A) 2^31, a 53-bit multiple of 2^31).  A = 0
          // (alpha = 0: the row max jumped far) makes every rel(x) 0: Ad = 0 and
          // Cd = 2^(52+S) + 2^(31+S) give exactly that.
          if (__all_sync(0xffffffffu, pair_ok || !row_ok)) {
#pragma unroll
            for (int part = 0; part < C::ACC_W / 32; ++part) {
              int v[32];
              tmem_ld32(acc_base + part * 32, v);
#pragma unroll
              for (int d = 0; d < 16; ++d) {
                const double y = __fma_rd(__hiloint2double(v[2 * d + 1], v[2 * d]), Ad, Cd);
                v[2 * d] = __double2loint(y);
                v[2 * d + 1] = __double2hiint(y);
              }
              tmem_st32(acc_base + part * 32, v);
            }
          } else {
            // the general forms (64-bit product, idiv, shifts outside [1, 32]) are
            // rare: a compact loop over the pairs that takes v[0] and rotates
#pragma unroll 1
            for (int part = 0; part < C::ACC_W / 32; ++part) {
              int v[32];
              tmem_ld32(acc_base + part * 32, v);
#pragma unroll 1
              for (int d = 0; d < 16; ++d) {
                const int x = v[0] ^ (int)0x80000000u;
                const int r = acc_idiv ? rel_idiv(x, alpha, rs) : rel_shift64(x, (unsigned long long)A, S);
#pragma unroll
                for (int i = 0; i < 30; ++i) v[i] = v[i + 2];
                v[30] = r ^ (int)0x80000000u;
                v[31] = (int)acc_hi;
              }
              tmem_st32(acc_base + part * 32, v);
            }
          }
        } else {
          const bool fast = !acc_idiv && S >= 13 && A >= 0 && A < (1ll << 31);
          if (__all_sync(0xffffffffu, fast || !row_ok)) {
            // int32((x * A + 2^(S-1)) >> S) on the FP64 pipe (rel_fp64)
            const double Ad = (double)A;
            const double Cd = __longlong_as_double(((1023ll + 51 + S) << 52) | (1ll << 51) | 1ll);
#pragma unroll
            for (int part = 0; part < DV / 32; ++part) {
              int v[32];
              tmem_ld32(acc_base + part * 32, v);
#pragma unroll
              for (int d = 0; d < 32; ++d) v[d] = rel_fp64(v[d], Ad, Cd);
              tmem_st32(acc_base + part * 32, v);
            }
          } else {
            // the general forms (64-bit product, idiv) are rare: a compact loop
            // that takes v[0] and rotates the array
#pragma unroll 1
            for (int part = 0; part < DV / 32; ++part) {
              int v[32];
              tmem_ld32(acc_base + part * 32, v);
#pragma unroll 1
              for (int d = 0; d < 32; ++d) {
                const int r = acc_idiv ? rel_idiv(v[0], alpha, rs) : rel_shift64(v[0], (unsigned long long)A, S);
#pragma unroll
                for (int i = 0; i < 31; ++i) v[i] = v[i + 1];
                v[31] = r;
              }
              tmem_st32(acc_base + part * 32, v);
            }
          }
        }
        tmem_wait_st();
        return true;
      };

      for (int j = 0; j < nch; ++j, ++g) {
        const int slot = g & 1;
        if (!(ok = wait(s_full(slot), (g >> 1) & 1, kErrSFull))) break;
        tc_fence_after();
        int alpha = 0, m_new = m;
        long long A = 0;
        bool pairA = false;
        double Ad = 0.0, Cd = 0.0;
        uint32_t pw[8];
        if (active) {
          int s[32];
          tmem_ld32(tmem + lane_base + slot * C::S_COLS + sg * 32, s);
          if (BIAS) {
            const uint8_t* brow = smem + C::OFF_B + (g % C::KVS) * C::B_BYTES + (warp * 32 + lane) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int4 b = *(const int4*)(brow + ((c ^ (lane & 7)) << 4));
              s[4 * c + 0] = (int)((unsigned)s[4 * c + 0] + (unsigned)b.x);
              s[4 * c + 1] = (int)((unsigned)s[4 * c + 1] + (unsigned)b.y);
              s[4 * c + 2] = (int)((unsigned)s[4 * c + 2] + (unsigned)b.z);
              s[4 * c + 3] = (int)((unsigned)s[4 * c + 3] + (unsigned)b.w);
            }
          }
          const int nvalid = a.N - j * kBN;  // < 32 only in a ragged last chunk
          if (nvalid < kBN) {
#pragma unroll
            for (int c = 0; c < 32; ++c) s[c] = c < nvalid ? s[c] : kNegInf;
          }
          // row max (with the running max m) as a tree of three-input maxima
          int t3[11];
#pragma unroll
          for (int c = 0; c < 10; ++c) t3[c] = __vimax3_s32(s[3 * c], s[3 * c + 1], s[3 * c + 2]);
          t3[10] = max(s[30], s[31]);
          m_new = max(__vimax3_s32(__vimax3_s32(t3[0], t3[1], t3[2]), __vimax3_s32(t3[3], t3[4], t3[5]),
                                   __vimax3_s32(t3[6], t3[7], t3[8])),
                      __vimax3_s32(t3[9], t3[10], m));
          bool use_fast = MODE == kFast;
          if (MODE == kChecked) use_fast = k_fast_all || __all_sync(0xffffffffu, m_new < k_mlim);
          // In a ragged last chunk every padded column holds NEG_INF, so all of
          // them share one P value: groups of four columns past the last valid
          // one (whole eighths of the chunk) take it without recomputation.
          const int nq = nvalid >= kBN ? 4 : (nvalid + 7) >> 3;  // eighths-pairs with a valid column
          if (use_fast && nvalid >= kBN) {
            // a full chunk: the 32 exp2 / requantise chains in one block
            const int cm1 = (int)((0u - (unsigned)m_new) * (unsigned)eM + 65536u);
            const int c3 = (int)((unsigned)rs - (unsigned)m_new);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int e0 = exp2_fast(s[4 * c + 0], eM, cm1, rs, c3);
              const int e1 = exp2_fast(s[4 * c + 1], eM, cm1, rs, c3);
              const int e2 = exp2_fast(s[4 * c + 2], eM, cm1, rs, c3);
              const int e3 = exp2_fast(s[4 * c + 3], eM, cm1, rs, c3);
              pw[c] = requant_pack4(e0, e1, e2, e3, rM);
            }
          } else if (use_fast) {
            // ragged last chunk (static indices throughout: pw stays in registers)
            const int cm1 = (int)((0u - (unsigned)m_new) * (unsigned)eM + 65536u);
            const int c3 = (int)((unsigned)rs - (unsigned)m_new);
            const int ep = exp2_fast(kNegInf, eM, cm1, rs, c3);
            const uint32_t pp = requant_pack4(ep, ep, ep, ep, rM);
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
              if (qd == 0 || qd < nq) {
#pragma unroll
                for (int c = 2 * qd; c < 2 * qd + 2; ++c) {
                  const int e0 = exp2_fast(s[4 * c + 0], eM, cm1, rs, c3);
                  const int e1 = exp2_fast(s[4 * c + 1], eM, cm1, rs, c3);
                  const int e2 = exp2_fast(s[4 * c + 2], eM, cm1, rs, c3);
                  const int e3 = exp2_fast(s[4 * c + 3], eM, cm1, rs, c3);
                  pw[c] = requant_pack4(e0, e1, e2, e3, rM);
                }
              } else {
                pw[2 * qd] = pp;
                pw[2 * qd + 1] = pp;
              }
            }
          } else if (MODE == kChecked) {
            // rare fallback of the range-checked kernel: compact, rotating s and pw
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
              const int e0 = exp2_generic((int)((unsigned)s[0] - (unsigned)m_new), rs, eM, false);
              const int e1 = exp2_generic((int)((unsigned)s[1] - (unsigned)m_new), rs, eM, false);
              const int e2 = exp2_generic((int)((unsigned)s[2] - (unsigned)m_new), rs, eM, false);
              const int e3 = exp2_generic((int)((unsigned)s[3] - (unsigned)m_new), rs, eM, false);
              const uint32_t w = requant_pack4(e0, e1, e2, e3, rM);
#pragma unroll
              for (int i = 0; i < 28; ++i) s[i] = s[i + 4];
#pragma unroll
              for (int i = 0; i < 7; ++i) pw[i] = pw[i + 1];
              pw[7] = w;
            }
          } else if (MODE != kFast) {
            const int ep = exp2_generic((int)((unsigned)kNegInf - (unsigned)m_new), rs, eM, exp_idiv);
            const uint32_t pp = requant_pack4(ep, ep, ep, ep, rM);
#pragma unroll
            for (int qd = 0; qd < 4; ++qd) {
              if (qd > 0 && qd >= nq) {
                pw[2 * qd] = pp;
                pw[2 * qd + 1] = pp;
                continue;
              }
#pragma unroll
              for (int c = 2 * qd; c < 2 * qd + 2; ++c) {
                const int e0 = exp2_generic((int)((unsigned)s[4 * c + 0] - (unsigned)m_new), rs, eM, exp_idiv);
                const int e1 = exp2_generic((int)((unsigned)s[4 * c + 1] - (unsigned)m_new), rs, eM, exp_idiv);
                const int e2 = exp2_generic((int)((unsigned)s[4 * c + 2] - (unsigned)m_new), rs, eM, exp_idiv);
                const int e3 = exp2_generic((int)((unsigned)s[4 * c + 3] - (unsigned)m_new), rs, eM, exp_idiv);
                pw[c] = requant_pack4(e0, e1, e2, e3, rM);
              }
            }
          }
          alpha = exp2_generic((int)((unsigned)m - (unsigned)m_new), rs, eM, exp_idiv);
          tmem_st8(tmem + lane_base + slot * C::S_COLS, pw);
          // the fixed-point constants of this chunk's scale_release (acc and l):
          // A = alpha * acc_M and the one-FMA form's Ad, Cd (see rescale)
          A = (long long)((unsigned long long)(long long)alpha * (unsigned long long)k_accM);
          // A in [acc_a_lo, acc_a_hi) or 0 <=> alpha in [alpha_lo, alpha_hi] or 0 (acc_M < 2^31);
          // Cd - 2^(S-1) = 2^(52+S) + 2^(31+S) + alpha * cK exactly, and for alpha = 0
          // adding 2^(S-1) (half an ulp) rounds to even, back to 2^(52+S) + 2^(31+S)
          pairA = pair_range && (alpha == 0 || (unsigned)(alpha - alpha_lo) <= (unsigned)(alpha_hi - alpha_lo));
          const double alpha_d = (double)alpha;
          Ad = alpha_d * accM_sd;
          Cd = __fma_rn(alpha_d, cK, acc_anchor) + acc_half;
          // acc = rel(acc, alpha) before PV of this chunk is added (first chunk: acc
          // starts from PV alone).  Skipped when it is the identity for every row
          // of the warp: alpha == rs and |acc| * |rs * acc_M - 2^S| < 2^(S-1).
          if (j > 0) {
            bool ident, pair_ok;
            if (BIAS) {
              ident = !acc_idiv && alpha == rs && abound < ident_lim;
              pair_ok = !acc_idiv && pairA && abound * (float)alpha * accM_f * two_mS < 2.0e9f;
            } else {
              const int bnd = acc_bound(j);  // bounds acc after chunk j - 1
              ident = !acc_idiv && alpha == rs && bnd < ident_lim_i;
              pair_ok = !acc_idiv && pairA && bnd < (1 << 29);
            }
            if (!__all_sync(0xffffffffu, ident || !row_ok) && !(ok = rescale(g - 1, alpha, A, Ad, Cd, pair_ok)))
              break;
          }
        }
        // P and acc are ready: release the MMA warp before the bookkeeping below,
        // which only later chunks need
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(slot));
        if (active) {
          // l_j = sum of the 32 int8 P values, two independent dot-product chains
          int ls0 = 0, ls1 = 0;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            ls0 = __dp4a((int)pw[2 * c], 0x01010101, ls0);
            ls1 = __dp4a((int)pw[2 * c + 1], 0x01010101, ls1);
          }
          int lr;
          if (l_pair && pairA && (unsigned)(l + (1 << 29)) < (1u << 30)) {
            // the acc constants, one FMA (|l| < 2^29 keeps |rel(l)| < 2^31)
            const double y = __fma_rd(__hiloint2double((int)acc_hi, l ^ (int)0x80000000u), Ad, Cd);
            lr = __double2loint(y) ^ (int)0x80000000u;
          } else {
            lr = l_idiv ? rel_idiv(l, alpha, rs)
                        : rel_shift64(l, (unsigned long long)(long long)alpha * (unsigned long long)k_lM, a.ls);
          }
          l = (int)((unsigned)lr + (unsigned)ls0 + (unsigned)ls1);
          m = m_new;
          const uint32_t neg = ((pw[0] | pw[1] | pw[2] | pw[3]) | (pw[4] | pw[5] | pw[6] | pw[7])) & 0x80808080u;
          if (!BIAS) {
            lb = lb && !neg && (j == 0 || (unsigned)alpha <= (unsigned)rs);  // chunk 0: acc is PV alone
          } else if (j > 0) {
            // |rel(x)| <= |x| * |A| / 2^S + 1 (the idiv form: <= |x| * |alpha| / rs + 1),
            // |A| = |alpha| * acc_M taken in float with round-up; no bound when the
            // 64-bit product could wrap, or in the idiv form
            const float aAbs = __fmul_ru(__uint2float_ru(alpha < 0 ? 0u - (unsigned)alpha : (unsigned)alpha), accM_ru);
            abound = (acc_idiv || S > 31 || abound * aAbs >= 4.6e18f)
                         ? __int_as_float(0x7f800000)
                         : __fmaf_ru(abound, aAbs * two_mS * 1.0001f, 2.f);
          }
          // |PV| <= 128 * sum|P|; sum|P| = ls0 + ls1 unless some P byte is negative
          if (BIAS) abound = __fadd_ru(abound, neg ? 524288.f : (float)((ls0 + ls1) << 7));
        }
      }
      if (!ok) break;

      // epilogue: O row = int8(int32(fp32(acc) / fp32(l))), once the last PV has landed
      if (active) {
        if (!(ok = wait(acc_full((g - 1) & 1), ((g - 1) >> 1) & 1, kErrPvFull))) break;
        tc_fence_after();
        int8_t* orow = a.o + (long long)z * a.os_z + (long long)h * a.os_h + (long long)row * a.os_n + a.v_col0;
        constexpr int EPP = C::ILV ? 16 : 32;  // acc elements per 32-column TMEM load
        constexpr int STEP = C::ILV ? 2 : 1;   // register stride of the elements
        // Default rounding: the reference's compiled sequence itself -- the int32
        // to fp32 conversion, div.full.f32 and the truncating, saturating
        // conversion back (cvt.rzi.s32.f32) -- for every element.
        // IEEE rounding (QFLASH_FLAG_DIV_IEEE): for |acc| < 2^23 and 0 < l < 2^24,
        // trunc(RN_f32(acc / l)) equals the truncated integer quotient (rounding up
        // to an integer n >= 2 needs l >= 2^24 / n, i.e. |acc| >= 2^23), which is
        // trunc(RZ(fp32(acc) * RU(1/l))): RU(1/l) - 1/l < 2^-23 / l, so
        // |acc| * RU(1/l) lies in [|acc| / l, |acc| / l + 1/l), below the next
        // integer, and rounding toward zero cannot drop below the integer part.
        const float lf = __int2float_rn(l);
        const bool fast_ieee =
            __all_sync(0xffffffffu, (l > 0 && l < (1 << 24) && (BIAS ? abound < 8388607.f : acc_bound(nch) < 8388607)) ||
                                        !row_ok);
        const float rcp = __frcp_ru(lf);
        // gathered output: the warp's rows go through its staging rows in shared
        // memory and leave as one bulk copy per destination
        const bool bulk = GATHER && C::STG_BYTES > 0 && a.o_bulk;
        // two staging buffers per warp, alternating by item: the copies of the
        // previous item may still be reading the other one
        const uint32_t stg = sbase + C::OFF_STG + (stg_buf * 4 + warp) * 32 * DV;
        if (bulk) {
          if (lane == 0) bulk_wait_read_but_last();  // the copies of two items ago have read this buffer
          __syncwarp();
          stg_buf ^= 1;
        }
#pragma unroll
        for (int part = 0; part < C::ACC_W / 32; ++part) {
          int v[32];
          tmem_ld32(acc_base + part * 32, v);
          if (C::ILV) {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[2 * i] ^= (int)0x80000000u;  // unbias
          }
          uint32_t res[EPP / 4];
          bool part_fast = div_full || fast_ieee;
          if (!part_fast) {
            // IEEE rounding without a bound for the row (e.g. a negative P byte
            // stopped the l-based bound): the fast form still holds for this
            // part if its own values have |acc| < 2^23
            bool in_range = l > 0 && l < (1 << 24);
#pragma unroll
            for (int i = 0; i < EPP; ++i) in_range = in_range && (unsigned)(v[STEP * i] + 8388607) <= 16777214u;
            part_fast = __all_sync(0xffffffffu, in_range || !row_ok);
          }
          if (part_fast) {
            int r[EPP];
#pragma unroll
            for (int i = 0; i < EPP; ++i) {
              const float xf = __int2float_rn(v[STEP * i]);
              float qf;
              if (div_full) {
                asm("div.full.f32 %0, %1, %2;" : "=f"(qf) : "f"(xf), "f"(lf));
              } else {
                qf = __fmul_rz(xf, rcp);
              }
              r[i] = __float2int_rz(qf);
            }
#pragma unroll
            for (int w4 = 0; w4 < EPP / 4; ++w4)
              res[w4] = __byte_perm(__byte_perm(r[4 * w4], r[4 * w4 + 1], 0x0040),
                                    __byte_perm(r[4 * w4 + 2], r[4 * w4 + 3], 0x0040), 0x5410);
          } else {
            // rare: the IEEE fp32 division, compact (4 elements per step, rotating)
#pragma unroll 1
            for (int w4 = 0; w4 < EPP / 4; ++w4) {
              int r4[4];
#pragma unroll
              for (int b = 0; b < 4; ++b) r4[b] = div_ieee_to_i32(v[STEP * b], l);
#pragma unroll
              for (int i = 0; i < 32 - 4 * STEP; ++i) v[i] = v[i + 4 * STEP];
#pragma unroll
              for (int i = 0; i < EPP / 4 - 1; ++i) res[i] = res[i + 1];
              res[EPP / 4 - 1] =
                  __byte_perm(__byte_perm(r4[0], r4[1], 0x0040), __byte_perm(r4[2], r4[3], 0x0040), 0x5410);
            }
          }
          if (row_ok && a.out) {
            const int esz = a.out_dtype == kF32 ? 4 : 2;
            uint8_t* drow = (uint8_t*)a.out +
                            ((long long)z * a.ou_z + (long long)h * a.ou_h + (long long)row * a.ou_n + a.v_col0 +
                             part * EPP) * esz;
            store_dequant<EPP>(drow, res, k_os, a.out_dtype, a.out_vec16);
          } else if (row_ok && bulk) {
#pragma unroll
            for (int q4 = 0; q4 < EPP / 16; ++q4)
              sts128(stg + lane * DV + part * EPP + 16 * q4,
                     make_uint4(res[4 * q4], res[4 * q4 + 1], res[4 * q4 + 2], res[4 * q4 + 3]));
          } else if (row_ok) {
            int8_t* dst = orow + part * EPP;
            if (a.o_vec16) {
#pragma unroll
              for (int q4 = 0; q4 < EPP / 16; ++q4) {
                const int4 val = make_int4((int)res[4 * q4], (int)res[4 * q4 + 1], (int)res[4 * q4 + 2],
                                           (int)res[4 * q4 + 3]);
                *(int4*)(dst + 16 * q4) = val;
                if (GATHER) {
#pragma unroll 1
                  for (int pi = 0; pi < a.n_peer; ++pi) *(int4*)(dst + a.o_peer_off[pi] + 16 * q4) = val;
                }
              }
            } else {
#pragma unroll
              for (int b = 0; b < EPP; ++b) dst[b] = (int8_t)(res[b >> 2] >> (8 * (b & 3)));
#pragma unroll 1
              for (int pi = 0; pi < (GATHER ? a.n_peer : 0); ++pi)
#pragma unroll
                for (int b = 0; b < EPP; ++b) dst[a.o_peer_off[pi] + b] = (int8_t)(res[b >> 2] >> (8 * (b & 3)));
            }
          }
        }
        if (bulk) {
          fence_proxy_async_smem();  // the staged rows are visible to the bulk copies
          __syncwarp();
          if (lane == 0) {
            // the warp's rows [row0, row0 + nrows) are contiguous (row stride DV, checked on the host)
            const uint32_t bytes = (uint32_t)min(32, a.N - row0) * DV;
            int8_t* gdst = a.o + (long long)z * a.os_z + (long long)h * a.os_h + (long long)row0 * a.os_n;
            bulk_store(gdst, stg, bytes);
            // the peers in an order that differs by CTA and warp, so that the
            // GPU's copies spread over every destination instead of all SMs
            // (of every rank) writing to the same peer at once
            int pi = (int)((blockIdx.x * 4u + (unsigned)warp) % (unsigned)a.n_peer);
#pragma unroll 1
            for (int c = 0; c < a.n_peer; ++c, pi = pi + 1 == a.n_peer ? 0 : pi + 1)
              bulk_store(gdst + a.o_peer_off[pi], stg, bytes);
            bulk_commit();
          }
        }
      }
    }
    if (GATHER && C::STG_BYTES > 0 && a.o_bulk && lane == 0) {
      bulk_wait_all();  // the bulk copies' global writes have completed
      fence_proxy_async_global();
    }
    // the peer copies' rows are performed system-wide before this CTA reports
    // itself finished (gather barrier below) or the kernel completes
    if (GATHER && a.n_peer > 0) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (GATHER && a.sig && threadIdx.x == 0) {
    // gather barrier (KArgs::sig): the last CTA to finish announces this rank's
    // rows to every rank and waits, bounded, until every rank has announced
    // this launch (flags only grow, so a rank already at the next launch counts)
    __threadfence_system();
    if (atomicAdd(a.sig + kSigCount, 1u) == gridDim.x - 1) {
      a.sig[kSigCount] = 0;  // ready for the next launch
      __threadfence_system();
#pragma unroll 1
      for (int pi = 0; pi < a.sig_world - 1; ++pi) st_release_sys(a.sig_peer[pi] + a.sig_rank, a.epoch);
      st_release_sys(a.sig + a.sig_rank, a.epoch);
      const long long t0 = clock64();
#pragma unroll 1
      for (int r = 0; r < a.sig_world; ++r) {
        while ((int)(ld_acquire_sys(a.sig + r) - a.epoch) < 0) {
          if (clock64() - t0 > kWaitCycles) {
            atomicOr(&g_err, kErrPeer);
            r = a.sig_world;
            break;
          }
          __nanosleep(256);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static thread_local std::string t_err;
static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_last_grid{0};

int set_err(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

static CUtensorMapSwizzle tma_swizzle(int atom_bytes) {
  return atom_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                          : (atom_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}

// 4-D map over a [Z, H, rows, cols] tensor (cols contiguous); strides in bytes.
static int make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t cols, uint64_t rows,
                    uint64_t H, uint64_t Z, uint64_t s_row, uint64_t s_h, uint64_t s_z, uint32_t box_cols,
                    uint32_t box_rows, int atom_bytes) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return set_err(QFLASH_ERR_DEVICE, "cuTensorMapEncodeTiled entry point unavailable");
  if (((uintptr_t)base & 15) || (s_row & 15) || (s_h & 15) || (s_z & 15))
    return set_err(QFLASH_ERR_ALIGN, "TMA needs 16-byte aligned base and strides (base %p, strides %llu %llu %llu)",
                   base, (unsigned long long)s_row, (unsigned long long)s_h, (unsigned long long)s_z);
  // The encoding is a function of these arguments alone, so recent ones are
  // reused: repeated calls on the same buffers (a caching allocator hands the
  // same addresses back) skip the driver call.
  struct Key {
    const void* base;
    uint64_t v[7];
    uint32_t box_cols, box_rows;
    int dt, atom;
  };
  Key key;
  memset(&key, 0, sizeof(Key));  // padding bytes take part in the comparison
  key.base = base;
  const uint64_t kv[7] = {cols, rows, H, Z, s_row, s_h, s_z};
  memcpy(key.v, kv, sizeof(kv));
  key.box_cols = box_cols;
  key.box_rows = box_rows;
  key.dt = (int)dt;
  key.atom = atom_bytes;
  constexpr int kSlots = 16;
  static thread_local Key keys[kSlots];
  static thread_local CUtensorMap maps[kSlots];
  static thread_local int used = 0, next = 0;
  for (int i = 0; i < used; ++i) {
    if (memcmp(&keys[i], &key, sizeof(Key)) == 0) {
      *m = maps[i];
      return QFLASH_OK;
    }
  }
  cuuint64_t dims[4] = {cols, rows, H, Z};
  cuuint64_t strides[3] = {s_row, s_h, s_z};
  cuuint32_t box[4] = {box_cols, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   tma_swizzle(atom_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_err(QFLASH_ERR_TMA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  memcpy(&keys[next], &key, sizeof(Key));
  maps[next] = *m;
  next = (next + 1) % kSlots;
  if (used < kSlots) ++used;
  return QFLASH_OK;
}

constexpr int kMaxDevices = 64;

int sm_count(int dev) {
  static int n[kMaxDevices] = {0};
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev];
}

template <int DQK, int DV, bool BIAS, int MODE, int SEGS, bool GATHER>
static int launch(int dev, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                  const CUtensorMap& mb, const KArgs& ka, cudaStream_t stream) {
  using C = Cfg<DQK, DV, BIAS, SEGS, GATHER>;
  auto kern = qfa_fwd_kernel<DQK, DV, BIAS, MODE, SEGS, GATHER>;
  static int per_sm[kMaxDevices] = {0};
  static std::mutex mu;
  int ctas;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (per_sm[dev] == 0) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
        return set_err(QFLASH_ERR_LAUNCH, "cudaFuncSetAttribute: %s", cudaGetErrorString(cudaGetLastError()));
      // the whole unified L1 as shared memory, so that the CTAs the other
      // limits allow are resident at once (the default carveout can hold fewer)
      if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
          cudaSuccess)
        return set_err(QFLASH_ERR_LAUNCH, "cudaFuncSetAttribute (carveout): %s", cudaGetErrorString(cudaGetLastError()));
      // resident CTAs per SM: registers, shared memory and TMEM columns
      cudaFuncAttributes fa;
      int regs = 255;
      if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess) regs = fa.numRegs;
      int smem_sm = 0;
      cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
      const int warp_regs = ((regs * 32 + 255) / 256) * 256;
      const int by_regs = 65536 / (warp_regs * (C::THREADS / 32));
      const int by_smem = smem_sm / (C::SMEM + 1024);
      const int by_tmem = 512 / C::TMEM_COLS;
      int v = by_regs < by_smem ? by_regs : by_smem;
      v = v < by_tmem ? v : by_tmem;
      if (const char* e = getenv("QFLASH_CTAS_PER_SM")) v = atoi(e);
      per_sm[dev] = v < 1 ? 1 : v;
    }
    ctas = per_sm[dev];
  }
  int grid = sm_count(dev) * ctas;
  // A grid that would leave CTA slots empty takes smaller work items: 64 or
  // 32 query rows of a head (the CTA still loads and multiplies a 128-row Q
  // box; warps past the item's rows idle), as many as one resident wave holds.
  // QFLASH_ROWS_PER_ITEM (32, 64 or 128) forces the choice.
  KArgs kb = ka;
  if (SEGS == 1) {
    auto items_for = [&](int rpi) { return (long long)ka.ZH * ((ka.N + rpi - 1) / rpi); };
    int rpi = kBM;
    if (const char* e = getenv("QFLASH_ROWS_PER_ITEM")) {
      const int f = atoi(e);
      if (f == 32 || f == 64 || f == 128) rpi = f;
    } else {
      while (rpi > 32 && items_for(rpi / 2) <= grid) rpi /= 2;
    }
    if (items_for(rpi) > 0x7fffffffLL) rpi = kBM;
    kb.rpi = rpi;
    kb.ntiles = (ka.N + rpi - 1) / rpi;
    kb.nitems = (int)items_for(rpi);
  }
  if (grid > kb.nitems) grid = kb.nitems;
  kern<<<grid, C::THREADS, C::SMEM, stream>>>(mq, mk, mv, mb, kb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_err(QFLASH_ERR_LAUNCH, "launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  g_last_grid.store(grid, std::memory_order_relaxed);
  return QFLASH_OK;
}

// Make the device that owns `p` current for this library's runtime (its
// current-device state is separate from the caller's).
int select_device(const void* p, int* dev) {
  cudaPointerAttributes pa;
  if (cudaPointerGetAttributes(&pa, p) != cudaSuccess) {
    cudaGetLastError();
    return set_err(QFLASH_ERR_ARG, "pointer %p is not known to CUDA", p);
  }
  if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged)
    return set_err(QFLASH_ERR_ARG, "pointer %p is not device memory", p);
  if (pa.device < 0 || pa.device >= kMaxDevices) return set_err(QFLASH_ERR_DEVICE, "device %d", pa.device);
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != pa.device && cudaSetDevice(pa.device) != cudaSuccess)
    return set_err(QFLASH_ERR_DEVICE, "cudaSetDevice(%d) failed", pa.device);
  static int checked[kMaxDevices] = {0};
  if (!checked[pa.device]) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, pa.device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, pa.device);
    if (major != 10 || minor != 0)
      return set_err(QFLASH_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", pa.device, major,
                     minor);
    checked[pa.device] = 1;
  }
  *dev = pa.device;
  return QFLASH_OK;
}

}  // namespace qfb

using namespace qfb;

namespace qfb {

int attention_fwd(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                  const int64_t q_strides[4], const int64_t k_strides[4], const int64_t v_strides[4],
                  const int64_t o_strides[4], const int64_t bias_strides[4], int bias_z_period, int Z, int H, int N,
                  int D, int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M, int64_t acc_M, int32_t l_shift,
                  int32_t acc_shift, uint32_t flags, const long long* dparams, const OutSpec* out, void* stream_,
                  const PeerSpec* peers) {
  cudaStream_t stream = (cudaStream_t)stream_;
  if (Z < 0 || H < 0 || N < 0) return set_err(QFLASH_ERR_ARG, "negative shape");
  if (!(D == 32 || D == 64 || D == 128 || D == 256)) return set_err(QFLASH_ERR_ARG, "head dim %d not in {32,64,128,256}", D);
  if (Z == 0 || H == 0 || N == 0) return QFLASH_OK;
  const bool fused_out = out != nullptr;
  if (fused_out && (!dparams || !out->p || out->dtype < kF32 || out->dtype > kBF16 || out->strides[3] != 1))
    return set_err(QFLASH_ERR_ARG, "dequantised output needs device constants, a float dtype and a contiguous head dim");
  if (!q || !k || !v || !q_strides || !k_strides || !v_strides || (!fused_out && (!o || !o_strides)))
    return set_err(QFLASH_ERR_ARG, "null pointer");
  if (q_strides[3] != 1 || k_strides[3] != 1 || v_strides[3] != 1 || (!fused_out && o_strides[3] != 1))
    return set_err(QFLASH_ERR_ARG, "innermost (head-dim) stride must be 1");
  if (!dparams && sm_rscale <= 0) return set_err(QFLASH_ERR_ARG, "sm_rscale must be positive");
  if (l_shift < 1 || l_shift > 62 || acc_shift < 1 || acc_shift > 62) return set_err(QFLASH_ERR_ARG, "shift out of [1, 62]");
  if (bias && !bias_strides) return set_err(QFLASH_ERR_ARG, "bias without strides");
  if ((flags & QFLASH_FLAG_DIV_FULL) && (flags & QFLASH_FLAG_DIV_IEEE))
    return set_err(QFLASH_ERR_ARG, "QFLASH_FLAG_DIV_FULL and QFLASH_FLAG_DIV_IEEE are exclusive");
  if (flags & ~(QFLASH_FLAG_EXP_IDIV | QFLASH_FLAG_L_IDIV | QFLASH_FLAG_ACC_IDIV | QFLASH_FLAG_DIV_FULL |
                QFLASH_FLAG_DIV_IEEE))
    return set_err(QFLASH_ERR_ARG, "unknown flag bits 0x%x", flags);
  DeviceGuard keep_device;  // the caller's current device is restored on return
  int dev = 0;
  if (int rc0 = select_device(q, &dev)) return rc0;

  KArgs ka;
  memset(&ka, 0, sizeof(ka));
  ka.Z = Z;
  ka.H = H;
  ka.N = N;
  ka.nch = (N + kBN - 1) / kBN;
  // two heads per 128-row tile when a head has at most 64 query rows
  const int segs = (N <= kBM / 2 && (D == 32 || D == 64)) ? 2 : 1;
  ka.rpi = kBM;
  ka.ntiles = segs == 2 ? 1 : (N + kBM - 1) / kBM;
  const long long zh_total = (long long)Z * H;
  if (zh_total > 0x7fffffffLL) return set_err(QFLASH_ERR_ARG, "too many heads");
  ka.ZH = (int)zh_total;
  const long long items = segs == 2 ? (zh_total + 1) / 2 : zh_total * ka.ntiles;
  if (bias_z_period < 0) return set_err(QFLASH_ERR_ARG, "negative bias_z_period");
  ka.bias_zmod = bias_z_period;
  if (items > 0x7fffffffLL) return set_err(QFLASH_ERR_ARG, "too many tiles");
  ka.nitems = (int)items;
  if (fused_out) {
    const int esz = out->dtype == kF32 ? 4 : 2;
    ka.out = out->p;
    ka.out_dtype = out->dtype;
    ka.ou_z = out->strides[0];
    ka.ou_h = out->strides[1];
    ka.ou_n = out->strides[2];
    ka.out_vec16 = (((uintptr_t)out->p & 15) == 0) && (out->strides[0] * esz % 16 == 0) &&
                   (out->strides[1] * esz % 16 == 0) && (out->strides[2] * esz % 16 == 0);
  } else {
    ka.o = o;
    ka.os_z = o_strides[0];
    ka.os_h = o_strides[1];
    ka.os_n = o_strides[2];
    ka.o_vec16 = (((uintptr_t)o & 15) == 0) && (o_strides[0] % 16 == 0) && (o_strides[1] % 16 == 0) &&
                 (o_strides[2] % 16 == 0);
  }
  if (peers && peers->n > 0) {
    if (fused_out) return set_err(QFLASH_ERR_UNSUPPORTED, "peer copies take the int8 output only");
    if (peers->n > kMaxPeers) return set_err(QFLASH_ERR_ARG, "%d peer copies (at most %d)", peers->n, kMaxPeers);
    for (int i = 0; i < peers->n; ++i) {
      const int8_t* po = peers->o[i];
      if (!po) return set_err(QFLASH_ERR_ARG, "peer copy %d is null", i);
      // same 16-byte phase as o, so the vector stores stay aligned in every copy
      if (((uintptr_t)po & 15) != ((uintptr_t)o & 15))
        return set_err(QFLASH_ERR_ALIGN, "peer copy %d (%p) and o (%p) differ in 16-byte alignment", i, po, o);
      cudaPointerAttributes pa;
      if (cudaPointerGetAttributes(&pa, po) != cudaSuccess || pa.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        return set_err(QFLASH_ERR_ARG, "peer copy %d (%p) is not device memory known to CUDA", i, po);
      }
      ka.o_peer_off[i] = (long long)((intptr_t)po - (intptr_t)o);
    }
    ka.n_peer = peers->n;
    // a warp's 32 rows are one contiguous block when the rows are dense
    ka.o_bulk = ka.o_vec16 && D <= 64 && o_strides[2] == D;
  }
  if (peers && peers->sig) {
    if (fused_out) return set_err(QFLASH_ERR_UNSUPPORTED, "the gather barrier takes the int8 output only");
    if (peers->rank < 0 || peers->rank > peers->n || peers->epoch == 0)
      return set_err(QFLASH_ERR_ARG, "gather barrier: rank %d of %d, epoch %u", peers->rank, peers->n + 1,
                     peers->epoch);
    if ((uintptr_t)peers->sig & 3) return set_err(QFLASH_ERR_ALIGN, "signal words must be 4-byte aligned");
    for (int i = 0; i < peers->n; ++i)
      if (!peers->sig_peer[i] || ((uintptr_t)peers->sig_peer[i] & 3))
        return set_err(QFLASH_ERR_ARG, "peer signal words %d are null or unaligned", i);
    ka.sig = peers->sig;
    for (int i = 0; i < peers->n; ++i) ka.sig_peer[i] = peers->sig_peer[i];
    ka.sig_rank = peers->rank;
    ka.sig_world = peers->n + 1;
    ka.epoch = peers->epoch;
  }
  ka.rs = sm_rscale;
  ka.eM = exp_M;
  ka.rM = req_M;
  ka.lM = l_M;
  ka.accM = acc_M;
  ka.ls = l_shift;
  ka.as = acc_shift;
  ka.flags = flags;
  // The 6-op exp2 form (exp2_fast) is exact when none of its int32 values
  // wraps.  Without a bias a score is an int8 dot product, |s| <= D*2^14, or
  // NEG_INF = -2^20, so with S0 = max(D*2^14, 2^20) every x = s - m_new is in
  // [-(S0 + m_new), 0].  x*exp_M + 2^16 fits int32 for |x| <= X1 and
  // r2 = x + (q+2)*rs fits for |x| <= X2, so rows with m_new <= min(X1, X2) - S0
  // are safe; if that holds for the largest possible m_new (D*2^14) it always holds.
  if (dparams) {
    // constants are produced on the device: the range check runs per chunk (m_lim from the device)
    ka.dparams = dparams;
    ka.fast_exp = bias ? 0 : 2;
  } else {
    const long long S0 = ((long long)D << 14) > (1ll << 20) ? ((long long)D << 14) : (1ll << 20);
    const long long aem = -(long long)exp_M;
    const long long lim31 = (1ll << 31) - 1;
    long long X = aem > 0 ? (lim31 - 65536) / aem : lim31;
    const long long X2 = ((lim31 - 2ll * sm_rscale - 2) * 65536) / (aem * sm_rscale + 65536);
    X = X < X2 ? X : X2;
    const long long mlim = X - S0;
    if (bias || exp_M > 0 || mlim <= -(1ll << 20)) {
      ka.fast_exp = 0;
    } else if (mlim >= ((long long)D << 14)) {
      ka.fast_exp = 1;
    } else {
      ka.fast_exp = 2;
    }
    ka.m_lim = (int)(mlim > lim31 ? lim31 : mlim);
  }

  const int DV = D == 256 ? 128 : D;
  const int qa = D < 128 ? D : 128;
  CUtensorMap mq, mk, mv, mb;
  memset(&mb, 0, sizeof(mb));
  int rc;
  if ((rc = make_map(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, q, D, N, H, Z, q_strides[2], q_strides[1], q_strides[0], qa,
                     kBM / segs, qa)))
    return rc;
  if ((rc = make_map(&mk, CU_TENSOR_MAP_DATA_TYPE_UINT8, k, D, N, H, Z, k_strides[2], k_strides[1], k_strides[0], qa,
                     kBN, qa)))
    return rc;
  if ((rc = make_map(&mv, CU_TENSOR_MAP_DATA_TYPE_UINT8, v, D, N, H, Z, v_strides[2], v_strides[1], v_strides[0], DV,
                     kBN, DV)))
    return rc;
  if (bias) {
    const int64_t bz = bias_strides[0], bh = bias_strides[1], br = bias_strides[2], bc = bias_strides[3];
    if (bc != 1) return set_err(QFLASH_ERR_ARG, "bias innermost stride must be 1");
    ka.bias_zb = bz != 0;
    ka.bias_hb = bh != 0;
    if (bias_z_period > 0 && !bz) return set_err(QFLASH_ERR_ARG, "bias_z_period needs a batch dimension in the bias");
    const int zb = bz ? (bias_z_period > 0 ? bias_z_period : Z) : 1;
    const uint64_t row_b = (uint64_t)br * 4;
    const uint64_t h_b = bh ? (uint64_t)bh * 4 : row_b * N;
    const uint64_t z_b = bz ? (uint64_t)bz * 4 : h_b * (bh ? H : 1);
    if ((rc = make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_INT32, bias, N, N, bh ? H : 1, zb, row_b, h_b, z_b, kBN,
                       kBM / segs, 128)))
      return rc;
  }
  const int passes = D == 256 ? 2 : 1;
  const bool gather = ka.n_peer > 0 || ka.sig;
  uint32_t* const sig = ka.sig;
  for (int p = 0; p < passes; ++p) {
    ka.v_col0 = p * DV;
    // the barrier closes the last pass only (a peer's flag then implies both of its passes)
    ka.sig = p == passes - 1 ? sig : nullptr;
    // the compact default-arithmetic kernels unless a QFLASH_* form needs the general one
    const bool gen = flags & (QFLASH_FLAG_EXP_IDIV | QFLASH_FLAG_L_IDIV | QFLASH_FLAG_ACC_IDIV);
    const int mode = gen ? kGen : (bias ? kPlain : (ka.fast_exp == 1 ? kFast : (ka.fast_exp == 2 ? kChecked : kGen)));
#define QFB_G(DQ, DVV, B, M, S)                                                   \
  (gather ? launch<DQ, DVV, B, M, S, true>(dev, mq, mk, mv, mb, ka, stream)       \
          : launch<DQ, DVV, B, M, S, false>(dev, mq, mk, mv, mb, ka, stream))
#define QFB_LAUNCH(DQ, DVV, B, M) \
  (segs == 2 ? QFB_G(DQ, DVV, B, M, 2) : QFB_G(DQ, DVV, B, M, 1))
#define QFB_LAUNCH1(DQ, DVV, B, M) QFB_G(DQ, DVV, B, M, 1)
#define QFB_CASE(DQ, DVV, L)                                                      \
  if (bias)                                                                       \
    rc = mode == kGen ? L(DQ, DVV, true, kGen) : L(DQ, DVV, true, kPlain);        \
  else if (mode == kFast)                                                         \
    rc = L(DQ, DVV, false, kFast);                                                \
  else if (mode == kChecked)                                                      \
    rc = L(DQ, DVV, false, kChecked);                                             \
  else                                                                            \
    rc = L(DQ, DVV, false, kGen);
    switch (D) {
      case 32: QFB_CASE(32, 32, QFB_LAUNCH) break;
      case 64: QFB_CASE(64, 64, QFB_LAUNCH) break;
      case 128: QFB_CASE(128, 128, QFB_LAUNCH1) break;
      default: QFB_CASE(256, 128, QFB_LAUNCH1) break;
    }
#undef QFB_G
#undef QFB_LAUNCH
#undef QFB_LAUNCH1
#undef QFB_CASE
    if (rc) return rc;
  }
  return QFLASH_OK;
}

}  // namespace qfb

extern "C" int qflash_i8_fwd_ex(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                                const int64_t q_strides[4], const int64_t k_strides[4], const int64_t v_strides[4],
                                const int64_t o_strides[4], const int64_t bias_strides[4], int bias_z_period, int Z,
                                int H, int N, int D, int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M,
                                int64_t acc_M, int32_t l_shift, int32_t acc_shift, uint32_t flags, void* stream) {
  return qfb::attention_fwd(q, k, v, o, bias, q_strides, k_strides, v_strides, o_strides, bias_strides,
                            bias_z_period, Z, H, N, D, sm_rscale, exp_M, req_M, l_M, acc_M, l_shift, acc_shift, flags,
                            nullptr, nullptr, stream);
}

extern "C" int qflash_i8_fwd_gather(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                                    const int64_t q_strides[4], const int64_t k_strides[4],
                                    const int64_t v_strides[4], const int64_t o_strides[4],
                                    const int64_t bias_strides[4], int bias_z_period, int Z, int H, int N, int D,
                                    int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M, int64_t acc_M,
                                    int32_t l_shift, int32_t acc_shift, uint32_t flags, int8_t* const* o_peers,
                                    int n_peers, uint32_t* sig, uint32_t* const* sig_peers, int rank,
                                    uint32_t epoch, void* stream) {
  if (n_peers < 0 || n_peers > qfb::kMaxPeers || (n_peers > 0 && !o_peers))
    return qfb::set_err(QFLASH_ERR_ARG, "n_peers %d (0..%d, with a pointer array)", n_peers, qfb::kMaxPeers);
  if (sig && n_peers > 0 && !sig_peers) return qfb::set_err(QFLASH_ERR_ARG, "signal words without the peers'");
  qfb::PeerSpec ps;
  memset(&ps, 0, sizeof(ps));
  ps.n = n_peers;
  for (int i = 0; i < n_peers; ++i) ps.o[i] = o_peers[i];
  ps.sig = sig;
  if (sig)
    for (int i = 0; i < n_peers; ++i) ps.sig_peer[i] = sig_peers[i];
  ps.rank = rank;
  ps.epoch = epoch;
  return qfb::attention_fwd(q, k, v, o, bias, q_strides, k_strides, v_strides, o_strides, bias_strides,
                            bias_z_period, Z, H, N, D, sm_rscale, exp_M, req_M, l_M, acc_M, l_shift, acc_shift, flags,
                            nullptr, nullptr, stream, &ps);
}

extern "C" int qflash_i8_fwd(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                             const int64_t q_strides[4], const int64_t k_strides[4], const int64_t v_strides[4],
                             const int64_t o_strides[4], const int64_t bias_strides[4], int Z, int H, int N, int D,
                             int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M, int64_t acc_M,
                             int32_t l_shift, int32_t acc_shift, uint32_t flags, void* stream) {
  return qflash_i8_fwd_ex(q, k, v, o, bias, q_strides, k_strides, v_strides, o_strides, bias_strides, 0, Z, H, N, D,
                          sm_rscale, exp_M, req_M, l_M, acc_M, l_shift, acc_shift, flags, stream);
}

extern "C" int qflash_device_error(void* stream, uint32_t* out) {
  if (!out) return set_err(QFLASH_ERR_ARG, "null out");
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return set_err(QFLASH_ERR_LAUNCH, "sync: %s", cudaGetErrorString(e));
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_err, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_err, &zero, sizeof(zero)) != cudaSuccess)
    return set_err(QFLASH_ERR_LAUNCH, "error word: %s", cudaGetErrorString(cudaGetLastError()));
  *out = v;
  return QFLASH_OK;
}

namespace qfb {
// The bounded wait of the attention kernel on an mbarrier that nothing ever
// arrives at: gives up after max_cycles SM clocks and records kErrSelftest in
// the error word, as a real timeout would record its site.
__global__ void wait_selftest_kernel(long long max_cycles) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_u32(&bar);
  mbar_init(b, 1);
  fence_mbar_init();
  const long long t0 = clock64();
  while (!mbar_try_wait_hint(b, 0, 1000)) {
    if (clock64() - t0 > max_cycles) {
      atomicOr(&g_err, kErrSelftest);
      return;
    }
  }
}
}  // namespace qfb

extern "C" int qflash_selftest_wait_timeout(void* stream, long long max_cycles) {
  if (max_cycles < 0 || max_cycles > 4000000000LL) return set_err(QFLASH_ERR_ARG, "max_cycles out of range");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_err(QFLASH_ERR_DEVICE, "no device");
  qfb::wait_selftest_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(max_cycles);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_err(QFLASH_ERR_LAUNCH, "selftest launch: %s", cudaGetErrorString(e));
  return QFLASH_OK;
}

namespace qfb {
// Max-reduction of up to 4 floats over the ranks through their signal words
// (qflash_peer_max).  Word layout after the gather barrier's: flags at
// kXFlag + r, values at kXVal + 4 * (8 * (epoch & 1) + r) -- two buffers by
// epoch parity, so a rank already at the next exchange writes the other one.
constexpr int kXFlag = 16, kXVal = 64;
struct PeerMaxArgs {
  const float* in;
  float* out;
  uint32_t* sig;
  uint32_t* sig_peer[kMaxPeers];
  int n, rank, world;
  uint32_t epoch;
};

// max that keeps a NaN (torch's amax propagates it)
__device__ __forceinline__ float max_nan(float a, float b) { return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b); }

__global__ void peer_max_kernel(const __grid_constant__ PeerMaxArgs a) {
  // thread p < world serves rank p (p == world - 1: this rank's own words):
  // it writes this rank's values and flag there, then waits for rank p's flag
  // here, so the remote stores and the waits run side by side
  __shared__ int failed;
  const int par = 8 * (a.epoch & 1);
  const int p = threadIdx.x;
  if (p == 0) failed = 0;
  __syncthreads();
  if (p < a.world) {
    uint32_t* w = p == a.world - 1 ? a.sig : a.sig_peer[p];
    volatile float* slot = (volatile float*)(w + kXVal + 4 * (par + a.rank));
#pragma unroll
    for (int i = 0; i < 4; ++i) slot[i] = i < a.n ? a.in[i] : 0.f;
    __threadfence_system();
    st_release_sys(w + kXFlag + a.rank, a.epoch);
    const long long t0 = clock64();
    while ((int)(ld_acquire_sys(a.sig + kXFlag + p) - a.epoch) < 0) {
      if (clock64() - t0 > kWaitCycles) {
        atomicOr(&g_err, kErrPeer);
        failed = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (p < a.n) {
    float m = __int_as_float(0x7fc00000);
    if (!failed) {
      m = ((volatile float*)(a.sig + kXVal + 4 * par))[p];
      for (int r = 1; r < a.world; ++r) m = max_nan(m, ((volatile float*)(a.sig + kXVal + 4 * (par + r)))[p]);
    }
    a.out[p] = m;
  }
}
}  // namespace qfb

extern "C" int qflash_peer_max(const float* in, int n, float* out, uint32_t* sig, uint32_t* const* sig_peers,
                               int n_peers, int rank, uint32_t epoch, void* stream) {
  if (!in || !out || !sig || n < 1 || n > 4 || n_peers < 0 || n_peers > qfb::kMaxPeers || rank < 0 ||
      rank > n_peers || epoch == 0 || (n_peers > 0 && !sig_peers) || ((uintptr_t)sig & 15))
    return set_err(QFLASH_ERR_ARG, "peer_max: n %d, n_peers %d, rank %d, epoch %u", n, n_peers, rank, epoch);
  qfb::PeerMaxArgs pa;
  memset(&pa, 0, sizeof(pa));
  pa.in = in;
  pa.out = out;
  pa.sig = sig;
  for (int i = 0; i < n_peers; ++i) {
    if (!sig_peers[i] || ((uintptr_t)sig_peers[i] & 15))
      return set_err(QFLASH_ERR_ARG, "peer signal words %d are null or unaligned", i);
    pa.sig_peer[i] = sig_peers[i];
  }
  pa.n = n;
  pa.rank = rank;
  pa.world = n_peers + 1;
  pa.epoch = epoch;
  DeviceGuard keep_device;
  int dev = 0;
  if (int rc = select_device(sig, &dev)) return rc;
  qfb::peer_max_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(pa);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_err(QFLASH_ERR_LAUNCH, "peer_max launch: %s", cudaGetErrorString(e));
  return QFLASH_OK;
}

extern "C" uint64_t qflash_launch_count(void) { return g_launches.load(); }
extern "C" int qflash_last_grid(void) { return g_last_grid.load(); }
extern "C" const char* qflash_version(void) { return "qflash_b200 0.1.0 (sm_100a)"; }
extern "C" const char* qflash_last_error(void) { return t_err.c_str(); }
