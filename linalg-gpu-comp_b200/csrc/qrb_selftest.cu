// Test hook for the device-side bounded waits (qrb_selftest_bounded_wait).
//
// One CTA of two warps whose roles wait on mbarriers that nothing ever arrives on, with
// no TMA copy or MMA in flight: warp 0 waits with a short caller-given limit, warp 1
// with the production limit.  Warp 0's wait runs out, records code 90 in the device
// error flag and raises the CTA's stop flag; warp 1's wait sees the flag and gives up
// without recording anything; the kernel exits.  This exercises the same wait routine
// (mbar_wait_abort) that the tensor-core kernels use.
#include "../../include/qrb200.h"
#include "qrb_internal.cuh"
#include "qrb_sm100.cuh"

namespace qrb {
namespace {

__global__ void __launch_bounds__(64) selftest_wait_kernel(unsigned limit, int* err) {
  __shared__ uint64_t bar[2];
  __shared__ int stop;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar[0], 1);
    sm100::mbar_init(&bar[1], 1);
    stop = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (lane == 0) {
    if (warp == 0)
      sm100::mbar_wait_abort(&bar[0], 0, &stop, err, 90, limit);
    else
      sm100::mbar_wait_abort(&bar[1], 0, &stop, err, 91);
  }
  __syncthreads();
}

}  // namespace
}  // namespace qrb

extern "C" QRB_API int qrb_selftest_bounded_wait(unsigned limit, void* stream) {
  if (limit == 0 || limit > (1u << 20)) return qrb::set_error(QRB_ERR_INVALID_ARG, "limit must be in [1, 2^20]");
  int* err = qrb::device_error_flag();
  if (err == nullptr) return qrb::set_error(QRB_ERR_CUDA, "could not look up the device error flag");
  qrb::selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(limit, err);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QRB_OK : qrb::set_error(QRB_ERR_CUDA, cudaGetErrorString(e));
}
