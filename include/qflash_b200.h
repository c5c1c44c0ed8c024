/*
 * qflash_b200 -- C ABI of the B200 (sm_100a) integer-only attention forward.
 *
 * The functions below are what a host binding (Python ctypes, a C/C++
 * caller, a cgo/JNI stub) calls.  Buffers are plain device pointers owned by
 * the caller; the library allocates no device memory.  Calls are asynchronous
 * on the given CUDA stream and return a status code (0 = launched).
 *
 * Reference: EfficientCompLab/qflash, qflash/kernel.py.
 */
#ifndef QFLASH_B200_H_
#define QFLASH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define QFLASH_OK 0
#define QFLASH_ERR_ARG (-1)         /* bad shape, head dim, null pointer, parameter */
#define QFLASH_ERR_ALIGN (-2)       /* pointer or stride alignment the TMA path cannot take */
#define QFLASH_ERR_TMA (-3)         /* tensor-map encoding failed */
#define QFLASH_ERR_LAUNCH (-4)      /* kernel launch failed */
#define QFLASH_ERR_DEVICE (-5)      /* no sm_100 device / driver entry point missing */
#define QFLASH_ERR_UNSUPPORTED (-6) /* combination not implemented */

/* flags: the reference's QFLASH_* arithmetic switches (qflash/kernel.py:30-36)
 * and the final-division rounding. 0 = the reference defaults, with the final
 * division acc / l (kernel.py:176) rounded as the reference's compiled Triton
 * kernel rounds it on B200: Triton lowers the int32 / int32 division to the
 * approximate fp32 divide div.full.f32. */
#define QFLASH_FLAG_EXP_IDIV 1u  /* QFLASH_EXP_USE_SHIFT=0: exp2_i32_idiv (kernel.py:47-51) */
#define QFLASH_FLAG_L_IDIV 2u    /* QFLASH_L_USE_SHIFT=0: scale_release_idiv for l (kernel.py:72-74) */
#define QFLASH_FLAG_ACC_IDIV 4u  /* QFLASH_ACC_USE_SHIFT=0: scale_release_idiv for acc */
#define QFLASH_FLAG_DIV_FULL 8u  /* final division as div.full.f32 (the default; accepted for explicitness) */
#define QFLASH_FLAG_DIV_IEEE 16u /* final division IEEE round-to-nearest: the reference's algorithm as its
                                    interpreted (TRITON_INTERPRET=1, numpy) run computes it */

/*
 * Integer attention forward: O = int8(acc / l) of the chunked integer online
 * softmax over int8 Q, K, V.
 *
 * Replaces the Triton launches qflash_kernel[grid](...) (qflash/kernel.py:319-326)
 * and qflash_masked_kernel[grid](...) (qflash/kernel.py:339-346); the
 * arguments are those launches' arguments:
 *   q, k, v, o      int8 [Z, H, N, D]; strides in elements, innermost (D) stride must be 1
 *   bias            int32 additive bias broadcastable to [Z, H, N, N] (NULL = unmasked
 *                   kernel); bias_strides in elements, 0 for a broadcast dimension, and
 *                   its row stride must be a multiple of 4 elements (16 bytes)
 *   D               32, 64, 128 or 256
 *   sm_rscale, exp_M, req_M, l_M, acc_M   the host-derived fixed-point constants
 *                   (kernel.py:302-307)
 *   l_shift, acc_shift   QFLASH_L_SHIFT / QFLASH_ACC_SHIFT (1..62)
 *   flags           QFLASH_FLAG_*
 *   stream          cudaStream_t (NULL = legacy default stream)
 * Pointers and the q/k/v/bias strides of the three outer dimensions must be 16-byte aligned.
 * Every entry point makes the device that owns q current for its launches and
 * restores the calling thread's current device before it returns.
 */
int qflash_i8_fwd(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                  const int64_t q_strides[4], const int64_t k_strides[4], const int64_t v_strides[4],
                  const int64_t o_strides[4], const int64_t bias_strides[4], int Z, int H, int N, int D,
                  int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M, int64_t acc_M, int32_t l_shift,
                  int32_t acc_shift, uint32_t flags, void* stream);

/*
 * qflash_i8_fwd with one more argument, bias_z_period: when > 0, batch index z
 * reads bias batch entry z % bias_z_period (the bias then has bias_z_period
 * entries in its batch dimension).  Swin's shifted-window bias depends on the
 * window index only, so a [num_windows, H, N, N] bias serves a batch of
 * num_images * num_windows windows without being expanded (the reference
 * materialises the expanded [Z, H, N, N] bias, qflash/kernel.py:336).
 * bias_z_period = 0 is qflash_i8_fwd.
 */
int qflash_i8_fwd_ex(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                     const int64_t q_strides[4], const int64_t k_strides[4], const int64_t v_strides[4],
                     const int64_t o_strides[4], const int64_t bias_strides[4], int bias_z_period, int Z, int H,
                     int N, int D, int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M, int64_t acc_M,
                     int32_t l_shift, int32_t acc_shift, uint32_t flags, void* stream);

/*
 * qflash_i8_fwd_ex for a batch shard whose int8 output is wanted on every GPU
 * of a job (the all_gather of the shards, fused into the attention epilogue;
 * no counterpart in the reference, whose multi-GPU use is data parallel over
 * batches).  o points at this shard's rows inside a gathered [Z_total, H, N, D]
 * buffer; o_peers[i] points at the same rows of another GPU's copy of that
 * buffer, mapped into this process (qflash_ipc_open), with o's strides and
 * o's 16-byte alignment.  Every O row is stored into o and into each peer copy
 * (P2P stores over NVLink, bulk copies of whole warps' rows when the rows are
 * dense and D <= 64; nothing is read from peer memory).  0 <= n_peers <= 7;
 * n_peers = 0 is qflash_i8_fwd_ex.
 * With sig set, the kernel also completes only once every rank's rows are in
 * every copy: sig points at this rank's QFLASH_SIG_WORDS signal words (uint32,
 * zero-initialised, in memory the peers map), sig_peers[i] at the signal words
 * of the rank that owns o_peers[i], rank is this rank's index in [0, n_peers],
 * and epoch is a non-zero launch counter, equal on every rank for the same
 * launch and growing from one launch to the next.  The last CTA to finish
 * writes epoch into every rank's flag `rank` and waits (bounded, ~2 s; a
 * timeout sets bit 256 of the device error word) until its own flags all
 * reach epoch.  Launches of one rank must not overlap on its GPU.  With
 * sig == NULL the caller orders the stores itself (a collective enqueued
 * after this call on every rank, e.g. an all_reduce of one element).
 */
#define QFLASH_SIG_WORDS 128
int qflash_i8_fwd_gather(const int8_t* q, const int8_t* k, const int8_t* v, int8_t* o, const int32_t* bias,
                         const int64_t q_strides[4], const int64_t k_strides[4], const int64_t v_strides[4],
                         const int64_t o_strides[4], const int64_t bias_strides[4], int bias_z_period, int Z, int H,
                         int N, int D, int32_t sm_rscale, int32_t exp_M, int32_t req_M, int64_t l_M, int64_t acc_M,
                         int32_t l_shift, int32_t acc_shift, uint32_t flags, int8_t* const* o_peers, int n_peers,
                         uint32_t* sig, uint32_t* const* sig_peers, int rank, uint32_t epoch, void* stream);

/*
 * CUDA IPC for the gathered output: qflash_ipc_alloc allocates `bytes` of
 * zeroed device memory on the current device and writes its 64-byte IPC handle;
 * another process opens it with qflash_ipc_open (on its current device, peer
 * access enabled) and unmaps it with qflash_ipc_close; the owner frees it with
 * qflash_ipc_free once every peer has closed it.
 */
#define QFLASH_IPC_HANDLE_BYTES 64

/*
 * Max over the ranks of n <= 4 floats (device pointers in / out), through the
 * same signal words as qflash_i8_fwd_gather's barrier (16-byte aligned): each
 * rank writes its values and a flag into every rank's words and waits,
 * bounded (~2 s; a timeout sets bit 256 of the device error word and writes
 * NaN), for all flags of this epoch.  NaN wins, as in torch's amax.  Used for
 * the global quantisation scales of a sharded forward (one launch of one
 * warp instead of a library all_reduce).  epoch as for the gather barrier,
 * counted separately from it.
 */
int qflash_peer_max(const float* in, int n, float* out, uint32_t* sig, uint32_t* const* sig_peers, int n_peers,
                    int rank, uint32_t epoch, void* stream);
int qflash_ipc_alloc(size_t bytes, void** ptr, void* handle);
int qflash_ipc_open(const void* handle, void** ptr);
int qflash_ipc_close(void* ptr);
int qflash_ipc_free(void* ptr);

/*
 * The whole forward of qflash.forward on the device, without the reference's
 * host synchronisation (the `.item()` at qflash/kernel.py:297): per-tensor
 * scales (kernel.py:294-296), the fixed-point constants (kernel.py:298-307,
 * Python double arithmetic), int8 quantisation (kernel.py:309-311), bias
 * quantisation (kernel.py:328-336), the attention kernel and the dequantised
 * output o * o_scale (kernel.py:351) -- each step as torch evaluates it on a
 * CUDA device, so the output equals the reference's bit for bit.
 *   q, k, v        float [Z, H, N, D], dtype 0 = f32, 1 = f16, 2 = bf16; strides in
 *                  elements with the head dim contiguous
 *   mask           optional additive float mask (mask_dtype 0/1/2) or bool mask (3),
 *                  broadcast to [Z, H, N, N] through mask_strides (0 on broadcast
 *                  dims); mask_zb / mask_hb its batch / head extents (1, Z or
 *                  mask_z_period; 1 or H); mask_z_period as in qflash_i8_fwd_ex
 *   q8, k8, v8, o8 int8 [Z, H, N, D] contiguous: the quantised tensors and the int8 output
 *   out            [Z, H, N, D] contiguous, dtype of q (all NaN if the constants
 *                  cannot be formed -- where the reference raises, e.g. q or k all zero)
 *   scale_log2e    the softmax scale times 1.44269504 (kernel.py:290-292)
 *   workspace      device memory, 256-byte aligned, >= qflash_fused_workspace_bytes()
 * Asynchronous on `stream`; qflash_fused_status() reports the constants' status.
 */
int qflash_fwd_fused(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
                     const int64_t k_strides[4], const int64_t v_strides[4], const void* mask, int mask_dtype,
                     const int64_t mask_strides[4], int mask_zb, int mask_hb, int mask_z_period, int8_t* q8,
                     int8_t* k8, int8_t* v8, int8_t* o8, void* out, int Z, int H, int N, int D, double scale_log2e,
                     int32_t l_shift, int32_t acc_shift, uint32_t flags, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * qflash_fwd_fused without the int8 output buffer: the attention epilogue
 * writes int8(acc / l) * o_scale straight into `out` (the input dtype) at the
 * element strides `out_strides` (NULL: contiguous [Z, H, N, D]; the head-dim
 * stride must be 1), e.g. the [Z, N, H, D] layout QAttention reshapes to
 * (qflash/attention.py:26) without a copy.  Replaces kernel.py:347-351 (the
 * int8 O tensor and o * o_scale).  On a status other than 0 `out` is all NaN.
 */
int qflash_fwd_fused_out(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
                         const int64_t k_strides[4], const int64_t v_strides[4], const void* mask, int mask_dtype,
                         const int64_t mask_strides[4], int mask_zb, int mask_hb, int mask_z_period, int8_t* q8,
                         int8_t* k8, int8_t* v8, void* out, const int64_t out_strides[4], int Z, int H, int N, int D,
                         double scale_log2e, int32_t l_shift, int32_t acc_shift, uint32_t flags, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * qflash_fwd_fused_out for Swin window attention with the bias built on the
 * device from its parts instead of a dense float mask: entry (w, h, i, j) of
 * the mask is table[index[i * N + j], h] plus window_mask[w, i, j] (added in
 * the promoted dtype of the two, as QWindowAttention does at
 * qflash/attention.py:68-72), then quantised as kernel.py:332-336 does.  The
 * reference expands that mask to [Z, H, N, N] (118 MB of int32 bias for Swin-T
 * stage 1); here it exists once per window and head, and batch z uses window
 * z % num_windows.  table: [table_rows, H] of table_dtype at element strides
 * table_strides; index: int64 [N * N] contiguous; window_mask: [num_windows, N,
 * N] contiguous of window_mask_dtype, or NULL (bias only; num_windows ignored).
 * Workspace: qflash_fused_workspace_bytes(window_mask ? num_windows : 1, H, N).
 * An index outside the table gives status 3 (and a NaN output).
 */
int qflash_fwd_fused_window(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
                            const int64_t k_strides[4], const int64_t v_strides[4], const void* table,
                            int table_dtype, const int64_t table_strides[2], int table_rows, const int64_t* index,
                            const void* window_mask, int window_mask_dtype, int num_windows, int8_t* q8, int8_t* k8,
                            int8_t* v8, void* out, const int64_t out_strides[4], int Z, int H, int N, int D,
                            double scale_log2e, int32_t l_shift, int32_t acc_shift, uint32_t flags, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Workspace bytes qflash_fwd_fused needs (mask_zb = mask_hb = 0 without a mask). */
size_t qflash_fused_workspace_bytes(int mask_zb, int mask_hb, int N);

/* Synchronises the stream and reads the status the fused forward recorded in its
 * workspace: 0 ok, 1 division by zero (the reference raises ZeroDivisionError),
 * 2 constants not representable (NaN/inf scales, or beyond int32), 3 a window
 * bias index outside its table. */
int qflash_fused_status(const void* workspace, void* stream, int64_t* status);

/*
 * qflash_fwd_fused for callers that cannot allocate device memory -- their
 * memory is owned by a pool or runtime they cannot extend, or cudaMalloc /
 * cudaFree (which may synchronise the whole device) are not allowed on their
 * path -- and so cannot pass a workspace.  No counterpart in the reference.
 * Same arguments and result as qflash_fwd_fused without workspace /
 * workspace_bytes; allocates nothing.  Its scratch is a fixed 4 MiB array in
 * the library (every GPU that loads the library holds it until exit), enough
 * for the constants plus an int32 bias of a mask up to about 4 MiB at
 * [mask_zb, mask_hb, N, N rounded up to 4] int32; larger masks are rejected
 * with QFLASH_ERR_UNSUPPORTED.  The array's device address is looked up
 * (cudaGetSymbolAddress) on every call made outside a stream capture, so a
 * device's first call must come before any capture.  Every call shares the one array: calls whose
 * work overlaps on the GPU (other streams, other threads) race and corrupt
 * each other; serialise them.  Nothing in the array needs to start at zero --
 * each call writes every byte it later reads -- so stale contents from an
 * earlier call are harmless.
 */
int qflash_fwd_fused_noalloc(const void* q, const void* k, const void* v, int dtype, const int64_t q_strides[4],
                             const int64_t k_strides[4], const int64_t v_strides[4], const void* mask,
                             int mask_dtype, const int64_t mask_strides[4], int mask_zb, int mask_hb,
                             int mask_z_period, int8_t* q8, int8_t* k8, int8_t* v8, int8_t* o8, void* out, int Z,
                             int H, int N, int D, double scale_log2e, int32_t l_shift, int32_t acc_shift,
                             uint32_t flags, void* stream);

/*
 * Status of the last qflash_fwd_fused_noalloc call on the device that owns q
 * (the same codes as qflash_fused_status; no counterpart in the reference):
 * the no-alloc caller has no workspace pointer to hand qflash_fused_status, so
 * this reads the library's scratch array of that device.  Synchronises the
 * stream.  The scratch keeps the most recent call's status, whichever stream
 * made it.
 */
int qflash_fused_noalloc_status(const void* q, void* stream, int64_t* status);

/* Reads and clears the device-side error word the kernels set when a bounded
 * wait gives up (0 = none).  Synchronises the stream. */
int qflash_device_error(void* stream, uint32_t* out);

/* Self-test of the timeout path: one thread waits, with the attention kernel's
 * bounded wait, on an mbarrier that nothing arrives at; after max_cycles SM
 * clocks (at most 4e9) it gives up and sets bit 31 of the device error word
 * (read it with qflash_device_error).  Asynchronous on `stream`, on the
 * current device.  No counterpart in the reference. */
int qflash_selftest_wait_timeout(void* stream, long long max_cycles);

/* Measured dense int8 tensor-core throughput, the denominator of the benchmark's
 * tensor roofline: ctas_per_sm (1 or 2) CTAs per SM each issue `iters`
 * back-to-back tcgen05.mma kind::i8 of M = 128, N = 256, K = 32 (2 * 128 * 256 *
 * 32 integer ops each) from shared memory into TMEM and wait for them.  The
 * caller times the launch on `stream` (CUDA events) and divides
 * SMs * ctas_per_sm * iters * 2097152 ops by the elapsed time.  No counterpart
 * in the reference (its contractions are the Triton tl.dot calls at
 * qflash/kernel.py:153,171). */
int qflash_i8_mma_peak(int ctas_per_sm, int iters, void* stream);
/* Synchronises the stream; *out = 1 if a peak-kernel wait gave up, else 0 (read and clear). */
int qflash_i8_mma_peak_status(void* stream, uint32_t* out);

/* Number of kernel launches issued by this library since load (for accounting). */
uint64_t qflash_launch_count(void);

/* Grid size (CTAs) of the most recent kernel launch (for accounting). */
int qflash_last_grid(void);

/* Library version string. */
const char* qflash_version(void);

/* Human-readable text of the last error on the calling thread. */
const char* qflash_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* QFLASH_B200_H_ */
