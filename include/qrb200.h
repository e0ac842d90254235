/*
 * qrb200.h -- C ABI of the B200-native batched Householder QR library (libqrb200.so).
 *
 * Drop-in boundary for the reference's submission entry point
 *   custom_kernel(data: Tensor[batch, n, n] f32 cuda) -> (H, tau)
 * (submission.py:913-921; contract in reference_repo/task.yml:12-27 and
 * reference_repo/task.py:4-5) and for the Q formation its checker performs with
 * torch.linalg.householder_product (reference_repo/reference.py:144).
 *
 * Conventions for every entry point:
 *   - Matrices are dense, row-major, contiguous (batch, n, n) fp32 in device memory,
 *     exactly the layout reference.generate_input returns (reference.py:87).
 *   - (H, tau) follow torch.geqrf / LAPACK SGEQRF compact form: R in the upper
 *     triangle of H, unit-leading Householder vectors strictly below the diagonal,
 *     tau[batch, n]; reflector convention of submissions/v1.py:9-38
 *     (beta = -sign(alpha)*||x||, sign(0) = +1).
 *   - All work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) and is asynchronous with respect to the host.  The library never
 *     allocates device memory on these paths; scratch comes from the caller's
 *     `workspace` of at least qrb_workspace_size() bytes (256-byte aligned).
 *   - Return value is a qrb_status.  Errors never throw; a per-thread message is
 *     available from qrb_last_error().  Calls on distinct streams are independent;
 *     one workspace must not be shared by calls that may run concurrently.
 *   - A may alias H (in-place factorisation).  Q must not alias A, H or tau.
 */
#ifndef QRB200_H
#define QRB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QRB_API __attribute__((visibility("default")))
#else
#define QRB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum qrb_status {
  QRB_OK = 0,
  QRB_ERR_INVALID_ARG = 1,   /* null pointer, n < 1, batch < 0, misaligned pointer */
  QRB_ERR_UNSUPPORTED = 2,   /* n above QRB_MAX_N, batch above 2^31, or (allocation-free
                                entry point) a batch larger than its static scratch holds */
  QRB_ERR_WORKSPACE = 3,     /* workspace missing or smaller than qrb_workspace_size() */
  QRB_ERR_CUDA = 4,          /* a CUDA runtime call or kernel launch failed */
  QRB_ERR_DEVICE = 5         /* current device is not an sm_100 (B200-class) GPU */
};

#define QRB_MAX_N 8192

/* Library version, major*10000 + minor*100 + patch. */
QRB_API int qrb_version(void);

/* Static description of a status code. */
QRB_API const char* qrb_status_string(int status);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len).  Returns the status of the last failing call on this thread
 * (QRB_OK if none). */
QRB_API int qrb_last_error(char* buf, size_t len);

/* Bytes of device workspace the calls below need for (batch, n).  0 is a valid
 * answer (small n needs none).  Same value for geqrf, orgqr and qr. */
QRB_API size_t qrb_workspace_size(int64_t batch, int n);

/* Batched Householder QR in compact form:  (H, tau) = geqrf(A).
 * Replaces custom_kernel (submission.py:913-921) / ref_kernel's torch.geqrf
 * (reference_repo/reference.py:90-92).  A is not modified unless A == H. */
QRB_API int qrb_geqrf_f32(const float* A, float* H, float* tau, int64_t batch, int n,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Q = H_0 H_1 ... H_{n-1} from compact (H, tau) (the full n x n orthogonal factor).
 * Replaces torch.linalg.householder_product(H, tau) (reference_repo/reference.py:144). */
QRB_API int qrb_orgqr_f32(const float* H, const float* tau, float* Q, int64_t batch, int n,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Fused full QR: (H, tau) = geqrf(A) and Q = householder_product(H, tau) in one call,
 * reusing the block reflector factors between the two phases.  R = triu(H).
 * The north-star path: torch.linalg.qr(A) with Q and R both available. */
QRB_API int qrb_qr_f32(const float* A, float* H, float* tau, float* Q, int64_t batch, int n,
               void* workspace, size_t workspace_bytes, void* stream);

/* Returns, and clears, the first error code that a library kernel recorded on the
 * current device when one of its bounded waits on tensor-core or bulk-copy completion
 * ran out (0 = none).  Such a kernel stops issuing copies, MMAs and stores, waits
 * (bounded) for the ones it already has in flight, releases its tensor memory and
 * exits, so its output is invalid.  Synchronises with the device.  No counterpart in the reference
 * (its kernels have no device-side waits). */
QRB_API int qrb_device_error(void);

/* Test hook for the device-side bounded waits: launches one CTA on `stream` whose two
 * roles wait on mbarriers that nothing arrives on, with no copy or MMA in flight.  The
 * first wait runs out after `limit` polls (1 .. 2^20), records error code 90 (read it
 * with qrb_device_error) and stops the CTA, the other role's wait gives up at once, and
 * the kernel exits.  Returns a qrb_status.  No counterpart in the reference. */
QRB_API int qrb_selftest_bounded_wait(unsigned limit, void* stream);

/* Number of kernels one qrb_qr_f32 (with_q != 0) or qrb_geqrf_f32 (with_q == 0) call
 * enqueues for (batch, n): 1 for n <= 64, otherwise one panel per 32 columns plus two or
 * three per block update (three when the W^T reduction is split over row chunks; one on
 * the SIMT path, n % 4 != 0).  0 for an empty batch or an unsupported n.  For graph
 * builders and launch accounting; no counterpart in the reference. */
QRB_API int64_t qrb_kernel_launches(int64_t batch, int n, int with_q);

/* Per-launch kernel timing, off by default.  While enabled, every kernel the library
 * launches is bracketed by two CUDA events on its launching stream.  The report
 * waits for the logged events, writes one line per kernel name,
 *   "<name> <launches> <total ms> <algorithmic bytes> <flops>\n",
 * into buf (NUL-terminated, truncated to len), clears the log and returns the length
 * the full report needs (including the NUL).  With buf == NULL it only returns that
 * length and keeps the log.  For profilers and benchmarks; no
 * counterpart in the reference (its bench scripts time whole calls). */
QRB_API void qrb_kernel_timing(int enable);
QRB_API size_t qrb_kernel_timing_report(char* buf, size_t len);

/* (H, tau) = geqrf(A) without any caller workspace, for callers that cannot
 * allocate device memory (a plugin host that passes only raw input/output pointers,
 * or a path that must not enter the allocator).  No counterpart in the reference.
 * Scratch lives in an 8 MiB static device array that every GPU loading the library
 * keeps until exit; for n > 64 the batch is limited to 2048 (QRB_ERR_UNSUPPORTED
 * beyond).  All calls share that array: calls that may overlap on the GPU race.
 * The first call on a device looks the array up and should come before any
 * stream capture; the looked-up address is kept for the life of the process, so the
 * entry point must not be used across a device reset.  Returns a qrb_status and, on
 * failure, sets the qrb_last_error message. */
QRB_API int qrb_geqrf_f32_noalloc(const float* A, float* H, float* tau, int64_t batch, int n,
                                  void* stream);

/* Device workspace, in bytes, of qrb_qr_f32_host for this batch (with_q != 0: Q is
 * formed too); 0 for invalid sizes or an empty batch. */
QRB_API size_t qrb_host_workspace_size(int64_t batch, int n, int with_q);

/* The same QR with HOST buffers: A (batch x n x n) is read from host memory and H,
 * tau and, when Q is not NULL, Q are written to host memory.  The batch is cut into
 * chunks whose copy-in, factorisation and copy-out overlap on internal streams;
 * `stream` orders the whole call (it waits for the caller's earlier work on it and
 * the caller's later work on it waits for the last copy).  Host buffers should be
 * page-locked (cudaHostAlloc / cudaHostRegister) for the copies to overlap; A may
 * alias H.  `device_workspace` is device memory of qrb_host_workspace_size bytes,
 * 256-byte aligned.  Results are identical to qrb_qr_f32 / qrb_geqrf_f32.  No
 * counterpart in the reference, whose harness keeps inputs and outputs on the device
 * (reference_repo/eval.py:128-131); this serves callers whose batch lives in host
 * memory. */
QRB_API int qrb_qr_f32_host(const float* A, float* H, float* tau, float* Q, int64_t batch, int n,
                            void* device_workspace, size_t device_workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QRB200_H */
