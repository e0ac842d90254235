// Internal declarations shared by the libqrb200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qrb {

// Panel (block reflector) width of the blocked path.  Every panel is factored
// by one lane-per-column kernel, so the width is the warp size.
constexpr int kNB = 32;

// Matrices with n <= kSmallMaxN are factored (and Q formed) by one CTA each,
// entirely on chip.
constexpr int kSmallMaxN = 64;

// Wide blocks (qrb_wide.cu): for n % 4 == 0 and n >= kWideMinN the trailing update and
// Q formation apply kWideNB reflectors at a time (four panels of kNB).
constexpr int kWideNB = 128;
constexpr int kWideMinN = 256;       // smallest n the workspace is sized for
constexpr int kWideDefaultN = 512;   // smallest n dispatched there by default (measured: n = 256 and
                                     // 352 are faster on the 32-wide path)

// Reflector convention of submissions/v1.py:9-38: |v0| below this is replaced by 1.
constexpr float kEpsV0 = 1e-30f;

// ---- device helpers --------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Householder reflector from alpha = x[0] and tail2 = ||x[1:]||^2, following
// submissions/v1.py:17-29: beta = -sign(alpha)*||x|| (sign(0) = +1),
// v0 = alpha - beta, tau = 2 v0^2 / (v0^2 + tail2) (0 if that is 0),
// u = x[1:] * (1 / v0) with |v0| < 1e-30 -> v0 := 1.
struct Reflector {
  float beta, tau, inv_v0, v0;   // v0: the (guarded) pivot of the unscaled vector
};

__device__ __forceinline__ Reflector make_reflector(float alpha, float tail2, bool trivial) {
  Reflector r;
  if (trivial) {  // m == 1: H = I (v1.py:14-16)
    r.beta = alpha;
    r.tau = 0.f;
    r.inv_v0 = 1.f;
    r.v0 = 1.f;
    return r;
  }
  float norm = sqrtf(alpha * alpha + tail2);
  float beta = alpha >= 0.f ? -norm : norm;
  float v0 = alpha - beta;
  float vn2 = v0 * v0 + tail2;
  r.beta = beta;
  r.tau = vn2 > 0.f ? __fdividef(2.f * v0 * v0, vn2) : 0.f;   // short-latency division on the serial path
  r.v0 = fabsf(v0) < kEpsV0 ? 1.f : v0;
  r.inv_v0 = __fdividef(1.f, r.v0);
  return r;
}

// ---- host helpers -----------------------------------------------------------
// Records `msg` as the calling thread's last error (qrb_last_error) and returns status.
int set_error(int status, const char* msg);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

// Brackets one kernel launch with CUDA events on its stream while kernel timing is
// enabled (qrb_kernel_timing); `bytes` / `flops` are the launch's algorithmic traffic
// and arithmetic, summed per kernel name in the report.  No-op when timing is off.
class LaunchTimer {
 public:
  LaunchTimer(const char* name, cudaStream_t s, double bytes = 0, double flops = 0);
  ~LaunchTimer();
  LaunchTimer(const LaunchTimer&) = delete;
  LaunchTimer& operator=(const LaunchTimer&) = delete;

 private:
  const char* name_;
  cudaStream_t s_;
  double bytes_, flops_;
  cudaEvent_t e0_ = nullptr, e1_ = nullptr;
};

// ---- launchers (return cudaError_t of the launch) ---------------------------
// Small-n fused kernel: geqrf and/or orgqr of n <= 64 matrices, one CTA each.
// mode bit 0: factor A -> (H, tau); bit 1: form Q from (H, tau).
cudaError_t launch_small(const float* A, float* H, float* tau, float* Q,
                         int64_t batch, int n, int mode, cudaStream_t s);

// Panel factorisation of H[:, k:, k:k+b] (b <= 32) with T factor:
// reads the panel from `src` (A on the first panel, otherwise H), writes the
// factored panel to H, tau[:, k:k+b] and T[batch][32][32] (upper triangular,
// I - V T V^T = H_k ... H_{k+b-1}).
cudaError_t launch_panel(const float* src, float* H, float* tau, float* T,
                         int64_t batch, int n, int k, int b, cudaStream_t s);

// Block reflector application  C[:, k:, c0:c1] -= V op(T) (V^T C[:, k:, c0:c1])
// with V = unit-lower reflectors H[:, k:, k:k+b].  trans_t = 1 applies T^T
// (Q_k^T, the geqrf trailing update), 0 applies T (Q_k, orgqr).  `src` is read
// (it may equal C).  If identity_fill, entries of C with row < k+b or column < k+b
// are taken as the identity instead of being read (orgqr without a Q init).
// `tcws` (nullable): workspace of tc_ws_floats(batch, n) floats for the tensor-core
// path (tf32 pieces of V and of W2, and the W^T partials); without it, or for
// n % 4 != 0, the SIMT kernel runs.
cudaError_t launch_apply(const float* H, const float* T, const float* src, float* C,
                         int64_t batch, int n, int k, int b, int c0, int c1, int trans_t,
                         int identity_fill, float* tcws, cudaStream_t s);
size_t tc_ws_floats(int64_t batch, int n);

// The two implementations launch_apply dispatches to (SIMT fp32 for any n).
cudaError_t launch_apply_simt(const float* H, const float* T, const float* src, float* C,
                              int64_t batch, int n, int k, int b, int c0, int c1, int trans_t,
                              int identity_fill, cudaStream_t s);
// Tensor-core (tcgen05, 3xTF32) variant of launch_apply; needs n % 4 == 0.
bool apply_tc_supported(int n);
cudaError_t launch_apply_tc(const float* H, const float* T, const float* src, float* C,
                            int64_t batch, int n, int k, int b, int c0, int c1, int trans_t,
                            int identity_fill, float* tcws, cudaStream_t s);
// Kernels one launch_apply_tc enqueues: wpart, w2 (only with a split W^T reduction), update.
int tc_update_launches(int64_t batch, int n, int k, int c0, int c1);

// ---- wide blocks (qrb_wide.cu) ----
bool wide_supported(int n);
// Workspace floats of the wide path (block T factors, V and W2 pieces, Y partials).
size_t wide_ws_floats(int64_t batch, int n);
// Kernels one wide block call enqueues.
int wide_block_launches(int64_t batch, int n, int K, bool update, bool tfactor, bool orgqr);
// geqrf, block at column K of width bw (its panels already factored, their T factors at
// t32blk = [panel][batch][32][32]): forms the block's 128 x 128 T factor (want_t) and,
// when `update`, applies the block to columns [K + bw, n) of H (read from src).
cudaError_t wide_geqrf_block(const float* src, float* H, const float* t32blk, float* ws, int64_t batch, int n,
                             int K, int bw, bool want_t, bool update, cudaStream_t s);
// orgqr: Q[K:, K:] = (I - V T V^T) Q[K:, K:] with the identity generated where Q is not
// formed yet, using the block T factor stored by wide_geqrf_block.
cudaError_t wide_orgqr_block(const float* H, float* Q, float* ws, int64_t batch, int n, int K, int bw,
                             cudaStream_t s);

// First error code recorded by a kernel whose bounded wait ran out (0 = none); clears it.
int take_device_error();
// Device address of that error flag on the current device (looked up once per device).
// Kernels outside the translation unit that defines the flag record through it: without
// relocatable device code every translation unit is its own device module, so an
// `extern __device__` declaration elsewhere would not name the same variable.
int* device_error_flag();

// T factors of all panels from (H, tau), for orgqr without a preceding geqrf.
cudaError_t launch_larft(const float* H, const float* tau, float* T_all,
                         int64_t batch, int n, cudaStream_t s);

}  // namespace qrb
