// Compiled call path of the torch ops: geqrf (custom_kernel) and the fused qr, each one
// C++ call -- ATen allocation of the outputs and workspace, torch's current stream of
// the input's device, and the C ABI of libqrb200 (include/qrb200.h).  The ctypes path
// costs a Python-level argument conversion per pointer and a Python allocation per
// output; here a call is a kernel launch plus a few microseconds, which is what the
// reference harness times for small batches (eval.py times each custom_kernel call).
//
// Inputs arrive already checked and contiguous (ops._check_batch), so the errors a user
// sees keep their Python types; a failing library status raises RuntimeError with the
// library's message, like _lib.check.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include "qrb200.h"

namespace {

void check_status(int status) {
  if (status != QRB_OK) {
    char buf[512];
    qrb_last_error(buf, sizeof buf);
    TORCH_CHECK(false, "libqrb200 error ", status, ": ", buf);
  }
}

struct Call {
  int64_t batch;
  int n;
  at::Tensor ws;
  void* wp = nullptr;
  size_t wb = 0;
  explicit Call(const at::Tensor& A) : batch(A.size(0)), n(static_cast<int>(A.size(1))) {
    wb = qrb_workspace_size(batch, n);
    if (wb > 0) {
      ws = at::empty({static_cast<int64_t>(wb)}, A.options().dtype(at::kByte));
      wp = ws.data_ptr();
    }
  }
};

std::tuple<at::Tensor, at::Tensor> geqrf(const at::Tensor& A) {
  c10::cuda::CUDAGuard guard(A.device());
  Call c(A);
  at::Tensor H = at::empty_like(A);
  at::Tensor tau = at::empty({c.batch, c.n}, A.options());
  check_status(qrb_geqrf_f32(A.data_ptr<float>(), H.data_ptr<float>(), tau.data_ptr<float>(), c.batch, c.n,
                             c.wp, c.wb, c10::cuda::getCurrentCUDAStream(A.get_device()).stream()));
  return {H, tau};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> qr(const at::Tensor& A) {
  c10::cuda::CUDAGuard guard(A.device());
  Call c(A);
  at::Tensor H = at::empty_like(A);
  at::Tensor tau = at::empty({c.batch, c.n}, A.options());
  at::Tensor Q = at::empty_like(A);
  check_status(qrb_qr_f32(A.data_ptr<float>(), H.data_ptr<float>(), tau.data_ptr<float>(), Q.data_ptr<float>(),
                          c.batch, c.n, c.wp, c.wb, c10::cuda::getCurrentCUDAStream(A.get_device()).stream()));
  return {H, tau, Q};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("geqrf", &geqrf, "(H, tau) = geqrf(A) for a checked, contiguous (batch, n, n) float32 CUDA tensor");
  m.def("qr", &qr, "(H, tau, Q) for a checked, contiguous (batch, n, n) float32 CUDA tensor");
}
