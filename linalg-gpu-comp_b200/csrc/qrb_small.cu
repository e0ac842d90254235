// Small-n fused QR: one CTA factors one n x n matrix (n <= 64) entirely on chip
// and, in the same launch, forms Q.
//
// Replaces the reference's fused small-n path (Triton _fused_qr_kernel,
// submission.py:521-612), which re-reduces the whole N_POW2^2 register tile every
// step, and adds the Q formation its checker does with householder_product
// (reference_repo/reference.py:144).
//
// Layout.  NP (32 or 64) is n rounded up.  The CTA has NP/16 warps; warp w owns
// columns [16w, 16w+16).  Lane = 4*rg + cg (rg in 0..7, cg in 0..3) owns rows
// {rg + 8i : i < NP/8} and columns {16w + 4cg + cc : cc < 4}, held in registers.
// A column reduction over rows is then 8 partial sums in registers followed by a
// 3-level xor shuffle across the 8 lanes sharing cg -- no shared memory and no
// CTA barrier.  Only the pivot column's reflector crosses warps, through a
// double-buffered shared vector, so geqrf costs one __syncthreads per column and
// orgqr (backward accumulation, reflectors read from the H tile in shared memory)
// needs none.  Warps whose columns are all left of the active column skip work.
#include "qrb_internal.cuh"

namespace qrb {
namespace {

template <int NP>
struct SmallCfg {
  static constexpr int kWarps = NP / 16;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kR = NP / 8;     // rows per thread
  static constexpr int kLD = NP + 4;    // padded row stride of the shared tile (16 B aligned)
};

template <int NP>
__device__ __forceinline__ void load_tile(float* tile, const float* __restrict__ g, int n) {
  using C = SmallCfg<NP>;
  const int tid = threadIdx.x;
  if ((n & 3) == 0) {
    const int n4 = n >> 2;
    for (int idx = tid; idx < NP * (NP / 4); idx += C::kThreads) {
      int r = idx / (NP / 4), c4 = idx % (NP / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < n && c4 < n4) v = __ldg(reinterpret_cast<const float4*>(g + (size_t)r * n) + c4);
      *reinterpret_cast<float4*>(tile + r * C::kLD + 4 * c4) = v;
    }
  } else {
    for (int idx = tid; idx < NP * NP; idx += C::kThreads) {
      int r = idx / NP, c = idx % NP;
      tile[r * C::kLD + c] = (r < n && c < n) ? __ldg(g + (size_t)r * n + c) : 0.f;
    }
  }
}

template <int NP>
__device__ __forceinline__ void store_tile(const float* tile, float* __restrict__ g, int n) {
  using C = SmallCfg<NP>;
  const int tid = threadIdx.x;
  if ((n & 3) == 0) {
    const int n4 = n >> 2;
    for (int idx = tid; idx < n * n4; idx += C::kThreads) {
      int r = idx / n4, c4 = idx % n4;
      reinterpret_cast<float4*>(g + (size_t)r * n)[c4] =
          *reinterpret_cast<const float4*>(tile + r * C::kLD + 4 * c4);
    }
  } else {
    for (int idx = tid; idx < n * n; idx += C::kThreads) {
      int r = idx / n, c = idx % n;
      g[(size_t)r * n + c] = tile[r * C::kLD + c];
    }
  }
}

// Column-group reduction: sum over the 8 lanes that share cg (lane bits 2..4).
__device__ __forceinline__ float rg_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

template <int NP>
__global__ void __launch_bounds__(SmallCfg<NP>::kThreads)
small_qr_kernel(const float* __restrict__ A, float* __restrict__ H, float* __restrict__ tau,
                float* __restrict__ Q, int n, int mode) {
  using C = SmallCfg<NP>;
  constexpr int R = C::kR;
  __shared__ __align__(16) float tile[NP * C::kLD];
  __shared__ float vbuf[2][NP];
  __shared__ float taus[NP];

  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = lane >> 2, cg = lane & 3;
  const int col0 = 16 * warp + 4 * cg;       // first of my 4 columns
  const size_t off = (size_t)b * n * n;

  float a[R][4];

  if (mode & 1) {
    // ---------------- geqrf ------------------------------------------------
    load_tile<NP>(tile, A + off, n);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < R; ++i) {
      float4 v = *reinterpret_cast<const float4*>(tile + (rg + 8 * i) * C::kLD + col0);
      a[i][0] = v.x; a[i][1] = v.y; a[i][2] = v.z; a[i][3] = v.w;
    }

    for (int j = 0; j < n; ++j) {
      const int pw = j >> 4, pcg = (j >> 2) & 3, pcc = j & 3;
      float* vb = vbuf[j & 1];
      if (warp == pw) {
        float x[R];
        float tail = 0.f, alpha = 0.f;
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const int r = rg + 8 * i;
          float xi = pcc == 0 ? a[i][0] : pcc == 1 ? a[i][1] : pcc == 2 ? a[i][2] : a[i][3];
          x[i] = xi;
          tail += r > j ? xi * xi : 0.f;
          alpha += r == j ? xi : 0.f;
        }
        tail = rg_sum(tail);
        alpha = rg_sum(alpha);
        const Reflector f = make_reflector(alpha, tail, j == n - 1);
        if (cg == pcg) {
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const int r = rg + 8 * i;
            const float v = r > j ? x[i] * f.inv_v0 : (r == j ? 1.f : 0.f);
            vb[r] = v;
            const float h = r > j ? v : (r == j ? f.beta : x[i]);
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
              if (cc == pcc) a[i][cc] = h;
          }
          if (rg == 0) taus[j] = f.tau;
        }
      }
      __syncthreads();
      if (16 * warp + 15 > j) {
        const float t = taus[j];
        float v[R];
#pragma unroll
        for (int i = 0; i < R; ++i) v[i] = vb[rg + 8 * i];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float p = 0.f;
#pragma unroll
          for (int i = 0; i < R; ++i) p = fmaf(v[i], a[i][cc], p);
          p = rg_sum(p);
          const float s = (col0 + cc > j) ? t * p : 0.f;
#pragma unroll
          for (int i = 0; i < R; ++i) a[i][cc] = fmaf(-s, v[i], a[i][cc]);
        }
      }
    }
    // H (registers) -> tile -> global; tau -> global.
#pragma unroll
    for (int i = 0; i < R; ++i)
      *reinterpret_cast<float4*>(tile + (rg + 8 * i) * C::kLD + col0) =
          make_float4(a[i][0], a[i][1], a[i][2], a[i][3]);
    __syncthreads();
    store_tile<NP>(tile, H + off, n);
    for (int j = threadIdx.x; j < n; j += C::kThreads) tau[(size_t)b * n + j] = taus[j];
  } else {
    load_tile<NP>(tile, H + off, n);
    for (int j = threadIdx.x; j < n; j += C::kThreads) taus[j] = tau[(size_t)b * n + j];
    __syncthreads();
  }

  if (mode & 2) {
    // ---------------- orgqr: Q = H_0 ... H_{n-1} I, backward ------------------
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int r = rg + 8 * i;
        a[i][cc] = (r == col0 + cc && r < n) ? 1.f : 0.f;
      }
    // Reflector j only touches columns >= j, so a warp starts at its last column.
    for (int j = min(n - 1, 16 * warp + 15); j >= 0; --j) {
      const float t = taus[j];
      float v[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int r = rg + 8 * i;
        v[i] = r > j ? tile[r * C::kLD + j] : (r == j ? 1.f : 0.f);
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float p = 0.f;
#pragma unroll
        for (int i = 0; i < R; ++i) p = fmaf(v[i], a[i][cc], p);
        p = rg_sum(p) * t;
#pragma unroll
        for (int i = 0; i < R; ++i) a[i][cc] = fmaf(-p, v[i], a[i][cc]);
      }
    }
    __syncthreads();   // every warp is done reading reflectors from the tile
#pragma unroll
    for (int i = 0; i < R; ++i)
      *reinterpret_cast<float4*>(tile + (rg + 8 * i) * C::kLD + col0) =
          make_float4(a[i][0], a[i][1], a[i][2], a[i][3]);
    __syncthreads();
    store_tile<NP>(tile, Q + off, n);
  }
}

}  // namespace

cudaError_t launch_small(const float* A, float* H, float* tau, float* Q,
                         int64_t batch, int n, int mode, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  if (n <= 32) {
    small_qr_kernel<32><<<(unsigned)batch, SmallCfg<32>::kThreads, 0, s>>>(A, H, tau, Q, n, mode);
  } else {
    small_qr_kernel<64><<<(unsigned)batch, SmallCfg<64>::kThreads, 0, s>>>(A, H, tau, Q, n, mode);
  }
  return cudaGetLastError();
}

}  // namespace qrb
