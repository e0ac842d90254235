// Block reflector application  C[k:, c0:c1] -= V op(T) (V^T C[k:, c0:c1])  (SIMT fp32).
// Used for n % 4 != 0, where TMA cannot describe the rows; other n take the
// tensor-core kernel in qrb_apply_tc.cu.
//
// Replaces the reference's trailing update (_wy_trailing_trisolve,
// submission.py:434-460: bmm, solve_triangular, baddbmm; and the cublasLt
// BF16x9 pair of the large-n path, submission.py:875-884) and serves orgqr's
// backward accumulation.  V = unit lower trapezoidal reflectors H[k:, k:k+b].
//
// One CTA owns one matrix and a 64-column strip of C over all m = n - k rows:
//   phase 1  W = V^T C          (32 x 64, split over 4 row groups, reduced in smem)
//   phase 2  W = op(T) W        (T^T for geqrf, T for orgqr)
//   phase 3  C -= V W           (64-row chunks, 4x4 register tiles)
// The strip is read twice (phase 1 and 3); the second read is served by L2.
#include <atomic>

#include "qrb_internal.cuh"

namespace qrb {
namespace {

constexpr int kTN = 64;          // strip width
constexpr int kThreads = 256;
constexpr int kRC1 = 32;         // rows per phase-1 chunk
constexpr int kRC3 = 64;         // rows per phase-3 chunk

struct ApplySmem {
  float Vs[kRC1][kNB + 4];        // phase 1 V chunk [row][refl]
  float Cs[kRC1][kTN + 4];        // phase 1 C chunk
  float Wred[4][kNB][kTN];        // phase 1 partials per row group
  float Ts[kNB][kNB + 1];
  float W2[kNB][kTN + 4];         // op(T) W
  float VT[kNB][kRC3 + 4];        // phase 3 V chunk, transposed [refl][row]
};

__device__ __forceinline__ float vload(const float* __restrict__ H, size_t moff, int n, int k,
                                       int b, int r, int i, int m) {
  // Unit lower trapezoidal V[r][i], r relative to row k.
  if (i >= b || r >= m) return 0.f;
  if (r > i) return __ldg(H + moff + (size_t)(k + r) * n + k + i);
  return r == i ? 1.f : 0.f;
}

__device__ __forceinline__ float cload(const float* __restrict__ src, size_t moff, int n, int R,
                                       int Cc, int kb, bool ident) {
  if (Cc >= n) return 0.f;
  if (ident && (R < kb || Cc < kb)) return R == Cc ? 1.f : 0.f;
  return src[moff + (size_t)R * n + Cc];
}

__global__ void __launch_bounds__(kThreads)
apply_kernel(const float* __restrict__ H, const float* __restrict__ Tg, const float* src,
             float* C, int n, int k, int b, int c0, int c1, int trans_t, int ident) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ApplySmem& sm = *reinterpret_cast<ApplySmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int nstrips = (c1 - c0 + kTN - 1) / kTN;
  const int64_t mat = blockIdx.x / nstrips;
  const int cs = c0 + (int)(blockIdx.x % nstrips) * kTN;   // first column of the strip
  const int m = n - k;
  const int kb = k + b;
  const size_t moff = (size_t)mat * n * n;

  // T (or T^T) into shared memory.
  const float* T = Tg + (size_t)mat * kNB * kNB;
  for (int idx = tid; idx < kNB * kNB; idx += kThreads) {
    int r = idx / kNB, c = idx % kNB;
    float t = T[idx];
    if (trans_t) sm.Ts[c][r] = t; else sm.Ts[r][c] = t;
  }

  // ---- phase 1: W = V^T C ------------------------------------------------------
  const int kg = tid >> 6, t64 = tid & 63;
  const int i0 = 4 * (t64 >> 3);             // 4 reflectors
  const int cA = 4 * (t64 & 7);              // columns cA..cA+3 and cA+32..cA+35
  float acc[4][8];
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int y = 0; y < 8; ++y) acc[x][y] = 0.f;

  for (int r0 = 0; r0 < m; r0 += kRC1) {
    __syncthreads();
    for (int idx = tid; idx < kRC1 * kNB; idx += kThreads) {
      int r = idx / kNB, i = idx % kNB;
      sm.Vs[r][i] = vload(H, moff, n, k, b, r0 + r, i, m);
    }
    for (int idx = tid; idx < kRC1 * kTN; idx += kThreads) {
      int r = idx / kTN, c = idx % kTN;
      sm.Cs[r][c] = (r0 + r < m && cs + c < c1) ? cload(src, moff, n, k + r0 + r, cs + c, kb, ident) : 0.f;
    }
    __syncthreads();
#pragma unroll 2
    for (int rr = kg; rr < kRC1; rr += 4) {
      float4 vv = *reinterpret_cast<const float4*>(&sm.Vs[rr][i0]);
      float4 ca = *reinterpret_cast<const float4*>(&sm.Cs[rr][cA]);
      float4 cb = *reinterpret_cast<const float4*>(&sm.Cs[rr][cA + 32]);
      const float vx[4] = {vv.x, vv.y, vv.z, vv.w};
      const float cx[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 8; ++y) acc[x][y] = fmaf(vx[x], cx[y], acc[x][y]);
    }
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    *reinterpret_cast<float4*>(&sm.Wred[kg][i0 + x][cA]) =
        make_float4(acc[x][0], acc[x][1], acc[x][2], acc[x][3]);
    *reinterpret_cast<float4*>(&sm.Wred[kg][i0 + x][cA + 32]) =
        make_float4(acc[x][4], acc[x][5], acc[x][6], acc[x][7]);
  }
  __syncthreads();
  // Reduce the 4 row groups in place into Wred[0].
  for (int idx = tid; idx < kNB * kTN; idx += kThreads) {
    int i = idx / kTN, c = idx % kTN;
    sm.Wred[0][i][c] = (sm.Wred[0][i][c] + sm.Wred[1][i][c]) + (sm.Wred[2][i][c] + sm.Wred[3][i][c]);
  }
  __syncthreads();

  // ---- phase 2: W2 = op(T) W ----------------------------------------------------
  {
    const int i = tid >> 3, cc = 8 * (tid & 7);
    float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int l = 0; l < kNB; ++l) {
      const float t = sm.Ts[i][l];
      float4 wa = *reinterpret_cast<const float4*>(&sm.Wred[0][l][cc]);
      float4 wb = *reinterpret_cast<const float4*>(&sm.Wred[0][l][cc + 4]);
      o[0] = fmaf(t, wa.x, o[0]); o[1] = fmaf(t, wa.y, o[1]);
      o[2] = fmaf(t, wa.z, o[2]); o[3] = fmaf(t, wa.w, o[3]);
      o[4] = fmaf(t, wb.x, o[4]); o[5] = fmaf(t, wb.y, o[5]);
      o[6] = fmaf(t, wb.z, o[6]); o[7] = fmaf(t, wb.w, o[7]);
    }
    *reinterpret_cast<float4*>(&sm.W2[i][cc]) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(&sm.W2[i][cc + 4]) = make_float4(o[4], o[5], o[6], o[7]);
  }

  // ---- phase 3: C -= V W2 --------------------------------------------------------
  const int tr = 4 * (tid >> 4), tc = 4 * (tid & 15);
  for (int r0 = 0; r0 < m; r0 += kRC3) {
    __syncthreads();
    for (int idx = tid; idx < kRC3 * kNB; idx += kThreads) {
      int r = idx / kNB, i = idx % kNB;
      sm.VT[i][r] = vload(H, moff, n, k, b, r0 + r, i, m);
    }
    __syncthreads();
    float o[4][4];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) o[x][y] = 0.f;
#pragma unroll 8
    for (int i = 0; i < kNB; ++i) {
      float4 vv = *reinterpret_cast<const float4*>(&sm.VT[i][tr]);
      float4 ww = *reinterpret_cast<const float4*>(&sm.W2[i][tc]);
      const float vx[4] = {vv.x, vv.y, vv.z, vv.w};
      const float wx[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) o[x][y] = fmaf(vx[x], wx[y], o[x][y]);
    }
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int r = r0 + tr + x;
      if (r >= m) continue;
      const int R = k + r;
#pragma unroll
      for (int y = 0; y < 4; ++y) {
        const int Cc = cs + tc + y;
        if (Cc < c1) C[moff + (size_t)R * n + Cc] = cload(src, moff, n, R, Cc, kb, ident) - o[x][y];
      }
    }
  }
}

}  // namespace

cudaError_t launch_apply(const float* H, const float* T, const float* src, float* C,
                         int64_t batch, int n, int k, int b, int c0, int c1, int trans_t,
                         int identity_fill, float* tcws, cudaStream_t s) {
  if (batch == 0 || c0 >= c1) return cudaSuccess;
  if (tcws != nullptr && apply_tc_supported(n))
    return launch_apply_tc(H, T, src, C, batch, n, k, b, c0, c1, trans_t, identity_fill, tcws, s);
  return launch_apply_simt(H, T, src, C, batch, n, k, b, c0, c1, trans_t, identity_fill, s);
}

cudaError_t launch_apply_simt(const float* H, const float* T, const float* src, float* C,
                              int64_t batch, int n, int k, int b, int c0, int c1, int trans_t,
                              int identity_fill, cudaStream_t s) {
  if (batch == 0 || c0 >= c1) return cudaSuccess;
  const size_t smem = sizeof(ApplySmem);
  // The opt-in shared-memory limit is a per-device function attribute; set it once per device.
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(apply_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  dim3 grid((unsigned)((int64_t)((c1 - c0 + kTN - 1) / kTN) * batch));
  const double m = n - k, nc = c1 - c0;
  LaunchTimer timer("apply_kernel", s, (double)batch * (8.0 * m * nc + 4.0 * m * b),
                    (double)batch * 4.0 * m * nc * b);
  apply_kernel<<<grid, kThreads, smem, s>>>(H, T, src, C, n, k, b, c0, c1, trans_t, identity_fill);
  return cudaGetLastError();
}

}  // namespace qrb
