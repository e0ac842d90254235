// T factors of every panel from compact (H, tau), for orgqr called without a
// preceding geqrf in the same call (the fused qr path reuses the T factors the
// panel kernel produced).  Restates submissions/v1.py:41-56 (_build_wy):
// G = V^T V, T[j][j] = tau_j, T[:j, j] = -tau_j T[:j, :j] G[:j, j].
#include "qrb_internal.cuh"

namespace qrb {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
larft_kernel(const float* __restrict__ H, const float* __restrict__ tau, float* __restrict__ T_all,
             int64_t batch, int n) {
  __shared__ float Vs[32][33];
  __shared__ float G[32][33];
  __shared__ float Ts[32][33];
  const int npan = (n + kNB - 1) / kNB;
  const int p = blockIdx.x % npan;       // panel
  const int64_t mat = blockIdx.x / npan;
  const int k = p * kNB, b = min(kNB, n - k), m = n - k;
  const size_t moff = (size_t)mat * n * n;
  const int tid = threadIdx.x;
  const int gi = tid >> 3, gj = 4 * (tid & 7);
  float g[4] = {0.f, 0.f, 0.f, 0.f};
  for (int r0 = 0; r0 < m; r0 += 32) {
    __syncthreads();
    for (int idx = tid; idx < 32 * 32; idx += kThreads) {
      int r = idx >> 5, i = idx & 31, rr = r0 + r;
      float v = 0.f;
      if (i < b && rr < m) v = rr > i ? __ldg(H + moff + (size_t)(k + rr) * n + k + i) : (rr == i ? 1.f : 0.f);
      Vs[r][i] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < 32; ++r) {
      const float a = Vs[r][gi];
#pragma unroll
      for (int q = 0; q < 4; ++q) g[q] = fmaf(a, Vs[r][gj + q], g[q]);
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) G[gi][gj + q] = g[q];
  __syncthreads();
  if (tid < 32) {
    const int i = tid;
    for (int j = 0; j < 32; ++j) {
      const float tj = j < b ? __ldg(tau + (size_t)mat * n + k + j) : 0.f;
      float t = 0.f;
      for (int c = 0; c < j; ++c) t = fmaf(Ts[i][c], G[c][j], t);
      Ts[i][j] = i < j ? -tj * t : (i == j ? tj : 0.f);
    }
    float* T = T_all + ((size_t)p * batch + mat) * kNB * kNB;
    for (int r = 0; r < 32; ++r) T[r * 32 + i] = Ts[r][i];
  }
}

}  // namespace

cudaError_t launch_larft(const float* H, const float* tau, float* T_all, int64_t batch, int n,
                         cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  dim3 grid((unsigned)((int64_t)((n + kNB - 1) / kNB) * batch));
  LaunchTimer timer("larft_kernel", s, (double)batch * 2.0 * n * n);
  larft_kernel<<<grid, kThreads, 0, s>>>(H, tau, T_all, batch, n);
  return cudaGetLastError();
}

}  // namespace qrb
