/* qrb200 -- B200-native batched square QR factorization, C ABI.
 *
 * Drop-in replacement for the reference entry point
 *     custom_kernel(data) -> (H, tau)        reflection_no_reflectors.py:181-196
 * (johnzfitch/qr-contest).  Output contract = torch.geqrf / LAPACK compact layout:
 * R in the upper triangle of H (including the diagonal), unit-lower Householder tails
 * strictly below it, tau_k = 2 / (v_k^T v_k) in [1, 2].  All pointers are DEVICE
 * pointers of the current CUDA device; everything is enqueued on `stream`
 * (a cudaStream_t passed as void*, NULL = legacy default stream).
 *
 * Nothing in this header depends on PyTorch or on the CUDA headers.
 */
#ifndef QRB200_H
#define QRB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes returned by every entry point */
#define QRB200_OK 0
#define QRB200_ERR_INVALID_ARG 1   /* null pointer, negative batch, bad dtype */
#define QRB200_ERR_UNSUPPORTED_N 2 /* n outside [0, qrb200_max_n()] */
#define QRB200_ERR_WORKSPACE 3     /* workspace given but smaller than required */
#define QRB200_ERR_CUDA 4          /* a CUDA runtime call or kernel launch failed */
#define QRB200_ERR_SCRATCH_LIMIT 5 /* allocation-free entry point: one matrix of this order
                                      needs more than QRB200_NOALLOC_SCRATCH_BYTES */

/* element types of A / H / tau (the factors are always computed in float32) */
#define QRB200_F32 0
#define QRB200_BF16 1
#define QRB200_F16 2

/* per-matrix info bits written to info[b] (0 = clean) */
#define QRB200_INFO_NONFINITE_INPUT 1 /* NaN/Inf met in the LU stage */
#define QRB200_INFO_CHOL1_NOT_PD 2    /* 1st CholeskyQR Gram not positive definite after jitter */
#define QRB200_INFO_CHOL2_NOT_PD 4    /* 2nd pass */
#define QRB200_INFO_LU_ZERO_PIVOT 8   /* exactly singular column met (informational) */
#define QRB200_INFO_DEVICE_TIMEOUT 16 /* a bounded in-kernel wait expired (never expected) */
#define QRB200_INFO_BOUNDS 32         /* bounds-check build (libqrb200_checked.so) only: a row
                                         index read from the LU's pivot maps was out of range;
                                         the access was redirected inside the buffer */

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int qrb200_version(void);

/* Human-readable text for a status code (static storage). */
const char* qrb200_status_string(int status);

/* Largest supported order n. */
int32_t qrb200_max_n(void);

/* Bytes of device workspace qrb200_geqrf_batched needs for (batch, n).
 * Replaces nothing in the reference (torch allocates internally); callers that manage
 * memory themselves size the buffer with this. */
int qrb200_workspace_bytes(int64_t batch, int32_t n, size_t* bytes);

/* Batched QR of `batch` row-major n x n matrices.
 *   A     [batch][n][n]  input, element type `dtype`, not modified
 *   H     [batch][n][n]  output, element type `dtype`
 *   tau   [batch][n]     output, element type `dtype`
 *   info  [batch]        output, QRB200_INFO_* bits (int32)
 *   workspace            device buffer of >= qrb200_workspace_bytes() bytes, or NULL to let
 *                        the library allocate it stream-ordered (cudaMallocAsync) per call
 * Replaces custom_kernel (reflection_no_reflectors.py:181-196): the frame
 * (_frame :55-81 -- torch.linalg.lu, two CholeskyQR passes), the closure
 * R = triu(Q^T A) (:186), the chart (_chart :86-176) and the assembly (:192-196).
 * Asynchronous with respect to the host; returns QRB200_OK once all work is enqueued. */
int qrb200_geqrf_batched(const void* A, void* H, void* tau, int32_t* info, int64_t batch,
                         int32_t n, int32_t dtype, void* workspace, size_t workspace_bytes,
                         void* stream);

/* qrb200_geqrf_batched plus the explicit orthogonal factor
 *   Q     [batch][n][n]  output, element type `dtype`: Q = householder_product(H, tau)
 * Replaces the consumer-side reconstruction torch.linalg.householder_product(H, tau) (LAPACK
 * orgqr, the use the reference documents in README.md:125-127): the chart factors
 * I - Q_frame S = Y (T Y^T) (reflection_no_reflectors.py:86-176), so the product of the
 * reflectors is the frame (:81) with column k scaled by the sign s_k, and it is written
 * straight from the frame the pipeline already holds (n^2 work instead of O(n^3)).
 * Same workspace, status codes and info bits as qrb200_geqrf_batched; Q may not be NULL. */
int qrb200_geqrf_batched_q(const void* A, void* H, void* tau, void* Q, int32_t* info,
                           int64_t batch, int32_t n, int32_t dtype, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Batched QR of `batch` tall row-major m x n matrices (m >= n; m == n is the square call).
 *   A     [batch][m][n]  input, element type `dtype`
 *   H     [batch][m][n]  output: s_i R_ij on and above the diagonal of the top n x n block,
 *                        the n reflector tails below it (torch.geqrf's layout for m x n)
 *   tau   [batch][n]     output;  info [batch] as for qrb200_geqrf_batched (the
 *                        informational QRB200_INFO_LU_ZERO_PIVOT bit is not reported)
 * Replaces the reference's rectangular chart modlu_rect (irregular/exp1_irregular.py:106-122:
 * the unpivoted sign-rule elimination over the n columns of an m x n frame), here applied to
 * the frame of reflection_no_reflectors.py:55-81 computed from the tall A itself.  Every
 * stage is column-nested, so the square kernels run on [A | 0] (m x m) with the CholeskyQR
 * jitter averaged over the first n diagonal entries, and the first n columns are returned:
 * the cost is that of an m x m factorization.  Padded buffers are allocated stream-ordered
 * (cudaMallocAsync) per call. */
int qrb200_geqrf_batched_rect(const void* A, void* H, void* tau, int32_t* info, int64_t batch,
                              int32_t m, int32_t n, int32_t dtype, void* stream);

/* Same computation as qrb200_geqrf_batched, with every kernel launch bracketed by CUDA
 * events on `stream`; blocks until the stream is idle and writes the summed device time
 * (milliseconds) of each kernel family into family_ms[0 .. qrb200_num_families()-1].
 * Replaces the reference's CUDA-event stage timing (common/bench.py:12-21,
 * kan_metric/prof_cluster.py) for the benchmark's roofline figures. */
int qrb200_geqrf_batched_timed(const void* A, void* H, void* tau, int32_t* info,
                               int64_t batch, int32_t n, int32_t dtype, void* workspace,
                               size_t workspace_bytes, void* stream, float* family_ms);

/* Number of kernel families reported by qrb200_geqrf_batched_timed, and their names
 * ("lu_panel", "lu_trail", "gram", "chol_panel", "chol_trail", "q_apply", "chart_panel",
 * "chart_trail", "closure", "small_fused" -- the one-kernel path for n <= 128).  No reference counterpart (the stage list of
 * reflection_no_reflectors.py:55-196 as this library splits it into kernels). */
int32_t qrb200_num_families(void);
const char* qrb200_family_name(int32_t family);

/* Total number of CUDA kernels this process has launched through the library.
 * No reference counterpart; used to report launches inside a timed region. */
long long qrb200_launch_count(void);

/* Process-wide tuning options (no reference counterpart).
 *   QRB200_OPT_GEMM_PATH: 0 = automatic (tcgen05 3xTF32 tiles when n % 4 == 0 and n >= 128,
 *   SIMT float32 tiles otherwise), 1 = SIMT tiles only, 2 = tcgen05 tiles whenever n % 4 == 0.
 * Returns QRB200_ERR_INVALID_ARG for an unknown key or value. */
#define QRB200_OPT_GEMM_PATH 1
/*   QRB200_OPT_SMALL_N: largest n (0..128, default 64) factored by the fused kernel that keeps
 *   the whole pipeline of one matrix in one CTA's shared memory (no workspace); larger n use
 *   the staged kernels.  Changing it also changes qrb200_workspace_bytes. */
#define QRB200_OPT_SMALL_N 2
/*   QRB200_OPT_CHOL_BLOCK: column block of the two-level Cholesky elimination of the
 *   CholeskyQR passes (0 = one level: every 32-wide panel updates the whole trailing matrix;
 *   64, 128 (default) or 256: the panels update only their block and the rest of the trailing
 *   matrix takes one K = block update per block).  Used when the tcgen05 path is active and
 *   n > block.  qrb200_workspace_bytes reflects the value set when it is called. */
#define QRB200_OPT_CHOL_BLOCK 3
/*   QRB200_OPT_LANES: number of internal streams (1..4, default 2) a chunk of the batch is
 *   split over; they fork from and join back to the caller's stream, so the call keeps its
 *   stream semantics.  1 = everything on the caller's stream. */
#define QRB200_OPT_LANES 4
/*   QRB200_OPT_CHART_BLOCK: column block of the two-level chart elimination (0 = one level;
 *   64, 128 (default) or 256): its 32-wide panels update only the block's columns and rows,
 *   the rest of the trailing matrix takes one float32 K = block update per block.  Used when
 *   n % 4 == 0 and n > block.  qrb200_workspace_bytes reflects the value set when it is called. */
#define QRB200_OPT_CHART_BLOCK 5
/*   QRB200_OPT_PANEL_LOOP: column loop of the register-resident panels (panels of at most 512
 *   rows): 0 = automatic (default; LU and chart panels of at most 128 rows then run two rows
 *   per thread of 64 threads, all panels of 129-256 rows two rows per thread of 128), 1 = fully unrolled, 2 = rotating registers (one column step of code, smaller
 *   than the instruction cache).  Modes 1 and 2 give bit-identical results. */
#define QRB200_OPT_PANEL_LOOP 6
/*   QRB200_OPT_CLOSURE_DUAL_N: largest n (0..512, default 256) whose closure GEMM runs two CTAs
 *   per SM; larger n use the one-CTA tile shape (which adds its float32 partial sums every
 *   256 k, so the two shapes agree to float32 rounding, not bit for bit). */
#define QRB200_OPT_CLOSURE_DUAL_N 7
int qrb200_set_option(int32_t key, int64_t value);

/* Text of the last CUDA runtime error that made an entry point of this thread return
 * QRB200_ERR_CUDA ("no error" if none).  No reference counterpart (torch raises with the
 * CUDA message). */
const char* qrb200_last_cuda_error(void);

/* Size of the built-in device scratch of qrb200_geqrf_batched_noalloc (64 MiB). */
#define QRB200_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)

/* Allocation-free variant of qrb200_geqrf_batched.  No counterpart in the reference: it is
 * for callers that cannot allocate device memory when they factor (host callbacks and
 * allocator hooks where cudaMalloc would re-enter or deadlock, embedders with fully
 * pre-partitioned memory).  The working buffers live in a file-scope device array of
 * QRB200_NOALLOC_SCRATCH_BYTES that every GPU loading this library holds until exit; the
 * batch is factored in chunks that fit it.  The function calls no cudaMalloc, cudaFree or
 * allocating library routine.
 *  - Same arguments, results and info bits as qrb200_geqrf_batched (no workspace).
 *  - Returns QRB200_ERR_SCRATCH_LIMIT, before it touches the buffers or the device, when the
 *    working set of a single n x n problem does not fit the scratch.  With the default options
 *    that is n above 1792 for n % 4 == 0 (32-wide panels) and above 1826 otherwise (16-wide
 *    panels); the bound moves with QRB200_OPT_CHOL_BLOCK / QRB200_OPT_CHART_BLOCK, which size
 *    the panel buffers.
 *  - The first call in each CUDA context of a device (with that device current) looks up the
 *    array's device address; make it before any stream capture.  A device reset creates a
 *    new context and the next call looks the address up again.
 *  - All calls share the array: calls that overlap on the GPU (other streams or threads)
 *    race and must be serialized by the caller. */
int qrb200_geqrf_batched_noalloc(const void* A, void* H, void* tau, int32_t* info,
                                 int64_t batch, int32_t n, int32_t dtype, void* stream);

/* Host-buffer variant: A, H, tau and info are HOST pointers (page-locked memory gives
 * overlapped copies; pageable memory works without the overlap).  Replaces the reference's
 * `custom_kernel(data)` called on a CPU tensor (reflection_no_reflectors.py:181-196), whose
 * results come back in host memory when the call returns.  The batch is cut into sub-batches
 * of `sub_batch` matrices (0 = automatic) that rotate over three streams: upload, factor and
 * download of neighbouring sub-batches overlap.  Device buffers are allocated on first use,
 * cached per device and grown as needed (qrb200_release_host_staging frees them).  The
 * sub-batches wait for work already queued on `stream`; the call blocks until every result
 * is in host memory.  Same results, status codes and info bits as qrb200_geqrf_batched. */
int qrb200_geqrf_batched_host(const void* A, void* H, void* tau, int32_t* info, int64_t batch,
                              int32_t n, int32_t dtype, int64_t sub_batch, void* stream);

/* Frees the current device's cached buffers of qrb200_geqrf_batched_host. */
int qrb200_release_host_staging(void);

#ifdef __cplusplus
}
#endif

#endif /* QRB200_H */
