// qrb_geqrf_f32_noalloc: the compact QR factorisation for callers that cannot
// allocate device memory.
//
// Some callers cannot call cudaMalloc at the point where they need a
// factorisation: a plugin host or foreign runtime that hands the library only raw
// input and output pointers and owns no device allocator, or a latency-critical
// path that must not enter the allocator (cudaMalloc can synchronise the device)
// and works within a memory budget reserved up front.  The regular entry point
// needs a caller workspace for the per-panel T factors of the blocked path
// (n > 64).  This variant keeps that scratch in a file-scope __device__ array
// instead, so the caller passes only A, H and tau.
//
// Limits and sharing rules:
//   * The scratch holds ONE panel's T factors for every matrix of the batch
//     (32 x 32 fp32 = 4 KiB per matrix), so for n > 64 the batch may be at most
//     kNoAllocScratchBytes / 4 KiB = 2048 matrices.  n <= 64 needs no scratch
//     and has no batch limit.  Larger batches are rejected (QRB_ERR_UNSUPPORTED).
//   * For n > 64 the trailing updates run on the SIMT fp32 kernel (qrb_apply.cu):
//     the tensor-core path needs workspace for its split operands.  Results agree
//     with the regular entry point to fp32 rounding, not bit for bit.
//   * Every GPU that loads the library holds the 8 MiB array until process exit.
//   * Every call shares the one array.  Each panel writes its T block in full
//     before the trailing update reads it, so nothing has to be cleared between
//     calls, but calls that may overlap on the GPU (different streams, or
//     different host threads without ordering) race on the scratch.
//   * The device address of the array is looked up once per device by the first
//     call made with that device current (cudaGetSymbolAddress); make that first
//     call before any stream capture begins.  The cached address belongs to the
//     device's primary context: do not use this entry point across a device reset
//     (cudaDeviceReset), which would leave the cached address stale.
#include <atomic>
#include <mutex>

#include "../../include/qrb200.h"
#include "qrb_internal.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB
constexpr size_t kTBytes = size_t(qrb::kNB) * qrb::kNB * sizeof(float);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_ptr[kMaxDevices];
std::mutex g_setup_mutex;

// Device address of g_noalloc_scratch on the current device (looked up once).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  void* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return e;
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return cudaSuccess;
}

}  // namespace

extern "C" QRB_API int qrb_geqrf_f32_noalloc(const float* A, float* H, float* tau, int64_t batch,
                                             int n, void* stream) {
  // Argument checks mirror qrb_geqrf_f32; the workspace is internal.  Failures set the
  // thread's qrb_last_error message like every other entry point.
  using qrb::set_error;
  if (batch < 0) return set_error(QRB_ERR_INVALID_ARG, "batch must be >= 0");
  if (n < 1) return set_error(QRB_ERR_INVALID_ARG, "n must be >= 1");
  if (n > QRB_MAX_N) return set_error(QRB_ERR_UNSUPPORTED, "n exceeds QRB_MAX_N");
  if (batch > (int64_t)1 << 31) return set_error(QRB_ERR_UNSUPPORTED, "batch exceeds 2^31");
  if (batch == 0) return QRB_OK;
  // Compared by division so that no product can wrap.
  if (n > qrb::kSmallMaxN && batch > (int64_t)(kNoAllocScratchBytes / kTBytes))
    return set_error(QRB_ERR_UNSUPPORTED,
                     "batch exceeds the 2048 matrices the static scratch holds for n > 64");
  if (A == nullptr || H == nullptr || tau == nullptr)
    return set_error(QRB_ERR_INVALID_ARG, "A, H and tau must not be null");
  if ((reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(H) & 15u) ||
      (reinterpret_cast<uintptr_t>(tau) & 3u))
    return set_error(QRB_ERR_INVALID_ARG, "A and H must be 16-byte aligned, tau 4-byte aligned");
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return set_error(QRB_ERR_CUDA, "could not query the current device");
  if (major != 10) return set_error(QRB_ERR_DEVICE, "the current device is not sm_100");

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n <= qrb::kSmallMaxN)
    return qrb::launch_small(A, H, tau, nullptr, batch, n, 1, s) == cudaSuccess
               ? QRB_OK
               : set_error(QRB_ERR_CUDA, "small-n kernel launch failed");

  void* scratch = nullptr;
  if (scratch_address(&scratch) != cudaSuccess)
    return set_error(QRB_ERR_CUDA, "cudaGetSymbolAddress of the scratch array failed");
  float* T = static_cast<float*>(scratch);
  // Same right-looking blocked algorithm as qrb_geqrf_f32, with one T slot reused
  // by every panel (stream order keeps panel p+1 from overwriting it early).
  for (int k = 0; k < n; k += qrb::kNB) {
    const int b = n - k < qrb::kNB ? n - k : qrb::kNB;
    const float* src = k == 0 ? A : H;
    if (qrb::launch_panel(src, H, tau, T, batch, n, k, b, s) != cudaSuccess)
      return set_error(QRB_ERR_CUDA, "panel kernel launch failed");
    if (k + b < n &&
        qrb::launch_apply(H, T, src, H, batch, n, k, b, k + b, n, 1, 0, nullptr, s) != cudaSuccess)
      return set_error(QRB_ERR_CUDA, "trailing update launch failed");
  }
  return QRB_OK;
}
