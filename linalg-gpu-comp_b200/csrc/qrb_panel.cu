// Panel factorisation (geqr2 on an m x b panel, b <= 32) fused with the compact-WY
// T factor (larft), for the blocked path (n > 64).
//
// Replaces the reference's panel kernels -- Triton _panel_qr_kernel
// (submission.py:95-167), the nvrtc CUDA panel_qr (submission.py:198-296) and the
// cuSOLVER geqrf panels of the large-n path (submission.py:858) -- plus its
// Gram/solve T^{-1} construction (submission.py:434-448).
//
// Layout.  Lane c of every warp owns panel column c; warp w and register i give
// CTA-local row w + W*i, so a CTA of W warps holds W*RPT rows in registers and a
// cluster of CL CTAs (rank q) holds rows [q*W*RPT, (q+1)*W*RPT).  Step j:
//   1. every lane fetches column j of its rows with one shuffle per row and forms
//      partial ||x||^2 / alpha (identical in all lanes of a warp);
//   2. the per-warp partials are combined across warps (and, for CL > 1, across
//      the cluster through distributed shared memory) -- every CTA sums the same
//      values in the same order, so all agree bit-for-bit on beta and tau;
//   3. each lane forms its partial w_c = v^T a_c; reduced the same way;
//   4. lanes c > j apply a_c -= tau w_c v; lane j stores beta / v.
// For c < j the reduced w_c equals (V^T V)[c, j], so the Gram matrix of the T
// recurrence T[:j, j] = -tau_j T[:j, :j] G[:j, j] (submissions/v1.py:48-56) falls out
// of the same pass; warp 0 evaluates the recurrence row-parallel after the loop.
#include <atomic>
#include <cooperative_groups.h>

#include "qrb_internal.cuh"
#include "qrb_sm100.cuh"

namespace cg = cooperative_groups;

namespace qrb {
namespace {


template <int RPT, int CL, int W>
__global__ void __launch_bounds__(W * 32)
panel_kernel(const float* __restrict__ src, float* __restrict__ H, float* __restrict__ tau,
             float* __restrict__ Tout, int n, int k, int b, int* err) {
  constexpr int kPanelWarps = W;
  constexpr int kRowsCta = W * RPT;
  __shared__ float2 red_n[2][W];                  // per-warp (tail^2, alpha) partials
  __shared__ float red_w[2][W][32];               // per-warp d_c partials
  __shared__ float rowj[2][32];                   // row j of the panel (rank 0)
  __shared__ float2 cred_n[2][CL];                // per-CTA partials (CL > 1)
  __shared__ float cred_w[2][CL][32];
  __shared__ float crowj[2][32];
  __shared__ float Ts[32][33];                    // T factor (rank 0 only)
  __shared__ float Gt[32][32];                    // Gt[j][c] = (V^T V)[c][j], c < j (rank 0)
  __shared__ float taus[32];
  __shared__ uint64_t cbar[2];                    // per step parity: the cluster's partials landed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int rank = 0;
  if constexpr (CL > 1) rank = (int)cg::this_cluster().block_rank();
  const int64_t mat = blockIdx.x / CL;
  const int m = n - k;
  const size_t moff = (size_t)mat * n * n;
  const int row0 = rank * kRowsCta + warp;        // panel row of register 0

  if constexpr (CL > 1) {
    if (threadIdx.x == 0) {
      sm100::mbar_init(&cbar[0], 1);
      sm100::mbar_init(&cbar[1], 1);
      sm100::fence_mbar_init();
    }
    cg::this_cluster().sync();   // every CTA's barriers exist before anything is pushed to them
  }
  // Bytes each CTA receives per step: every CTA's 32 dot partials and (tail, alpha), and
  // row j of the panel from rank 0.
  constexpr uint32_t kStepBytes = CL * (32 * 4 + 8) + 32 * 4;
  bool ok = true;

  float a[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int pr = row0 + W * i;
    a[i] = (pr < m && lane < b) ? __ldg(src + moff + (size_t)(k + pr) * n + k + lane) : 0.f;
  }

  // Reflectors are applied unscaled: u_j = (0.., v0, x_{j+1}, ..) and H_j = I - s u u^T
  // with s = tau / v0^2, so no lane rescales its rows per step; lane c keeps its raw
  // column and divides it by v0_c once at the end.  Only registers i < kTop can hold
  // a row <= 31 (rank 0); every other row is below any pivot of the panel and needs no
  // row predicate.
  constexpr int kTop = 32 / W;
  float my_inv = 1.f, my_beta = 0.f;   // this lane's column reflector (set at step j == lane)
  for (int j = 0; j < b; ++j) {
    const int par = j & 1;
    // ---- 1. column j of my rows: partial ||x||^2 and alpha, and for every column c
    //         d_c = sum over rows r > j of x_r a_rc, which does not depend on the
    //         reflector: u^T a_c = v0 a_jc + d_c.  So one reduction round per step.
    float u[RPT];
    float tail = 0.f, tail2 = 0.f, alpha = 0.f, d0 = 0.f, d1 = 0.f, ajc = 0.f;
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int pr = row0 + W * i;
      const float x = __shfl_sync(0xffffffffu, a[i], j);
      u[i] = x;
      if (i < kTop) {
        const float xt = pr > j ? x : 0.f;
        tail = fmaf(xt, xt, tail);
        alpha += pr == j ? x : 0.f;
        ajc += pr == j ? a[i] : 0.f;
        d0 = fmaf(xt, a[i], d0);
      } else if (i & 1) {
        tail2 = fmaf(x, x, tail2);
        d1 = fmaf(x, a[i], d1);
      } else {
        tail = fmaf(x, x, tail);
        d0 = fmaf(x, a[i], d0);
      }
    }
    tail += tail2;
    // ---- 2. one reduction round (double-buffered: one barrier per step suffices) ----
    if (lane == 0) red_n[par][warp] = make_float2(tail, alpha);
    red_w[par][warp][lane] = d0 + d1;
    if (rank == 0 && warp == (j & (kPanelWarps - 1))) rowj[par][lane] = ajc;   // row j: warp j % W
    __syncthreads();
    float2 nsum = make_float2(0.f, 0.f);
    float dsum = 0.f, aj;
    if constexpr (CL == 1) {
#pragma unroll
      for (int q = 0; q < kPanelWarps; ++q) {
        const float2 t = red_n[par][q];
        nsum.x += t.x;
        nsum.y += t.y;
        dsum += red_w[par][q][lane];
      }
      aj = rowj[par][lane];
    } else {
      // CTA sums first; warp 0 pushes them into every rank's receive buffers with
      // st.async, each store completing its bytes on the receiver's mbarrier, and every
      // CTA waits on its own barrier only (no cluster-wide barrier per step).  Each CTA
      // then adds the CL sums in rank order (bit-identical beta / tau everywhere).  The
      // buffers alternate by step parity: a CTA sends step j + 2 only after it has
      // received every CTA's step j + 1, which each sends after reading its step-j buffer.
      if (threadIdx.x == 0) sm100::mbar_arrive_expect_tx(&cbar[par], kStepBytes);
      if (warp == 0) {
        float2 p = make_float2(0.f, 0.f);
        float sw = 0.f;
#pragma unroll
        for (int q = 0; q < kPanelWarps; ++q) {
          const float2 t = red_n[par][q];
          p.x += t.x;
          p.y += t.y;
          sw += red_w[par][q][lane];
        }
        const float rj = rowj[par][lane];
#pragma unroll
        for (int q = 0; q < CL; ++q) {
          const uint32_t bar = sm100::mapa_shared(sm100::smem_u32(&cbar[par]), q);
          sm100::st_async_f32(sm100::mapa_shared(sm100::smem_u32(&cred_w[par][rank][lane]), q), sw, bar);
          if (lane == 0) sm100::st_async_f32x2(sm100::mapa_shared(sm100::smem_u32(&cred_n[par][rank]), q), p, bar);
          if (rank == 0) sm100::st_async_f32(sm100::mapa_shared(sm100::smem_u32(&crowj[par][lane]), q), rj, bar);
        }
      }
      if (ok && !sm100::mbar_wait(&cbar[par], (j >> 1) & 1)) {
        ok = false;
        atomicCAS(err, 0, 70);
      }
#pragma unroll
      for (int q = 0; q < CL; ++q) {
        const float2 t = cred_n[par][q];
        nsum.x += t.x;
        nsum.y += t.y;
        dsum += cred_w[par][q][lane];
      }
      aj = crowj[par][lane];
    }
    const Reflector f = make_reflector(nsum.y, nsum.x, j == m - 1);
    const float w = fmaf(f.v0, aj, dsum);   // u^T a_c with u = (0.., v0, x_{j+1}, ..)
#pragma unroll
    for (int i = 0; i < kTop && i < RPT; ++i) {
      const int pr = row0 + W * i;
      u[i] = pr > j ? u[i] : (pr == j ? f.v0 : 0.f);
    }

    // ---- 4. apply to columns > j (lane j keeps its raw column) -------------------
    const float coef = lane > j ? f.tau * f.inv_v0 * f.inv_v0 * w : 0.f;
#pragma unroll
    for (int i = 0; i < RPT; ++i) a[i] = fmaf(-coef, u[i], a[i]);
    if (lane == j) {
      my_inv = f.inv_v0;
      my_beta = f.beta;
    }
    // ---- record G[:j, j] = (V^T V)[c, j] and tau_j (warp 0 of rank 0) ----------
    // Lane c < j holds raw column c, so w = v0_j v0_c G[c][j].
    if (warp == 0 && rank == 0) {
      if (lane < j) Gt[j][lane] = w * f.inv_v0 * my_inv;
      if (lane == 0) {
        taus[j] = f.tau;
        tau[(size_t)mat * n + k + j] = f.tau;
      }
    }
  }

  // ---- T factor after the column loop: lane i builds row i of T in registers -----
  // T[i][j] = -tau_j * sum_{c<j} T[i][c] G[c][j] (j > i; T[i][c] = 0 for c < i),
  // T[i][i] = tau_i: rows are independent, so the 32 recurrences run side by side; with
  // the loops unrolled the row stays in registers and G[:, j] is a broadcast read.
  if (warp == 0 && rank == 0) {
    __syncwarp();
    const int i = lane;
    float t[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int c = 0; c + 3 < j; c += 4) {
        s0 = fmaf(t[c], Gt[j][c], s0);
        s1 = fmaf(t[c + 1], Gt[j][c + 1], s1);
        s2 = fmaf(t[c + 2], Gt[j][c + 2], s2);
        s3 = fmaf(t[c + 3], Gt[j][c + 3], s3);
      }
#pragma unroll
      for (int c = j & ~3; c < j; ++c) s0 = fmaf(t[c], Gt[j][c], s0);
      const float v = -taus[j] * ((s0 + s1) + (s2 + s3));
      t[j] = (j < i || j >= b) ? 0.f : (j == i ? taus[j] : v);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) Ts[i][j] = t[j];
  }

  // ---- write back panel (v = raw / v0 below, beta on the diagonal) and T ------
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int pr = row0 + W * i;
    float h = a[i] * my_inv;
    if (i < kTop) h = pr > lane ? h : (pr == lane ? my_beta : a[i]);
    if (pr < m && lane < b) H[moff + (size_t)(k + pr) * n + k + lane] = h;
  }
  if (warp == 0 && rank == 0) {
    __syncwarp();
    float* T = Tout + (size_t)mat * 32 * 32;
#pragma unroll 4
    for (int r = 0; r < 32; ++r) T[r * 32 + lane] = Ts[r][lane];
  }
  if constexpr (CL > 1) cg::this_cluster().sync();   // no CTA exits while peers may still write to it
}

template <int RPT, int CL, int W = 8>
cudaError_t launch_panel_t(const float* src, float* H, float* tau, float* T, int64_t batch,
                           int n, int k, int b, cudaStream_t s) {
  const double m = n - k;
  LaunchTimer timer("panel_kernel", s, (double)batch * (8.0 * m * b + 4.0 * b + 4096.0),
                    (double)batch * 4.0 * m * b * b);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(batch * CL));
  cfg.blockDim = dim3(W * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if constexpr (CL > 8) {   // 16-CTA clusters exceed the portable size: opt in once per device
    static std::atomic<unsigned long long> done{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
    const unsigned long long bit = 1ull << (dev & 63);
    if ((done.load(std::memory_order_acquire) & bit) == 0) {
      const cudaError_t e =
          cudaFuncSetAttribute(panel_kernel<RPT, CL, W>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      done.fetch_or(bit, std::memory_order_acq_rel);
    }
  }
  int* err = device_error_flag();
  if (err == nullptr) return cudaErrorInvalidValue;
  return cudaLaunchKernelEx(&cfg, panel_kernel<RPT, CL, W>, src, H, tau, T, n, k, b, err);
}

}  // namespace

cudaError_t launch_panel(const float* src, float* H, float* tau, float* T, int64_t batch,
                         int n, int k, int b, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  const int m = n - k;
  // Single CTA while the panel fits 8 warps x 64 rows; clusters of 256-row CTAs
  // (512-row for m > 2048, 16 of them for m > 4096) beyond that.
  // Short panels: with many matrices in flight (throughput-bound) fewer warps with more
  // rows each cost less per column (fewer partials, cheaper barrier); a small batch is
  // latency-bound and does better spread over 8 warps.  Measured on one B200: b512_n256
  // 1.54 vs 1.59 ms, b40_n176 0.218 vs 0.210 ms.
  const bool wide = batch >= 256;
  if (m <= 64) return wide ? launch_panel_t<32, 1, 2>(src, H, tau, T, batch, n, k, b, s)
                           : launch_panel_t<8, 1>(src, H, tau, T, batch, n, k, b, s);
  if (m <= 128) return wide ? launch_panel_t<32, 1, 4>(src, H, tau, T, batch, n, k, b, s)
                            : launch_panel_t<16, 1>(src, H, tau, T, batch, n, k, b, s);
  if (m <= 256) return launch_panel_t<32, 1>(src, H, tau, T, batch, n, k, b, s);
  if (m <= 512) return launch_panel_t<64, 1>(src, H, tau, T, batch, n, k, b, s);
  if (m <= 1024) return launch_panel_t<32, 4>(src, H, tau, T, batch, n, k, b, s);
  // 1024 < m <= 2048: with 16+ matrices the GPU is full either way, and 4-CTA clusters of
  // 512 rows cost less per column than 8-CTA clusters of 256 (cheaper exchange; measured
  // b32_n2048 panels 2.70 vs 2.90 ms); a small batch keeps the 8-CTA spread (b8_n2048
  // 6.14 vs 6.27 ms, b2_n4096 13.99 vs 14.13 ms).
  if (m <= 2048) return batch >= 16 ? launch_panel_t<64, 4>(src, H, tau, T, batch, n, k, b, s)
                                    : launch_panel_t<32, 8>(src, H, tau, T, batch, n, k, b, s);
  if (m <= 4096) return launch_panel_t<64, 8>(src, H, tau, T, batch, n, k, b, s);
  return launch_panel_t<64, 16>(src, H, tau, T, batch, n, k, b, s);   // up to 8192 rows
}

}  // namespace qrb
