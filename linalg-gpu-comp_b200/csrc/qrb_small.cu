// Small-n fused QR: one CTA factors one n x n matrix (n <= 64) entirely on chip
// and, in the same launch, forms Q.
//
// Replaces the reference's fused small-n path (Triton _fused_qr_kernel,
// submission.py:521-612), which re-reduces the whole N_POW2^2 register tile every
// step, and adds the Q formation its checker does with householder_product
// (reference_repo/reference.py:144).
//
// n <= 32 takes tiny_qr_kernel (one warp per matrix, at the end of this file).
//
// Layout (32 < n <= 64).  NP = 64 is n rounded up.  Four lanes share a column: lane =
// 8*rg + cl (rg in 0..3) of warp w owns two columns -- 16w + cl and 16w + 8 + cl -- and
// the rows {rg + 4i}, all in registers, so the CTA has NP/16 warps (small register
// footprint per matrix: more matrices in flight per SM).  A column reduction over rows is a
// register sum plus two xor shuffles (8, 16).
//
// Reflectors are published unscaled: u_j = (0.., v0, x_{j+1}, .., x_{n-1}) with
// v0 = alpha - beta, so v = u / v0 and H_j = I - s_j u u^T with s_j = tau_j / v0^2.
// The column owner writes u_j to shared memory once; consumers fold s_j into a
// per-column coefficient, so no dynamic row index is needed in the update and
// H's sub-diagonal is divided by v0 once at the end.
//
// geqrf step j: every warp still owning a column > j waits on one named barrier,
// applies H_j to its columns (dot + update on the 16-row blocks that can be
// non-zero, chosen at compile time from j / 16), and the warp owning column j+1
// then forms ||x||^2 of that column (row predicates only in the one or two
// blocks that straddle row j+1) and publishes u_{j+1}.
// orgqr (backward accumulation) reads the stored u_j and needs no barrier.
#include "qrb_internal.cuh"

namespace qrb {
namespace {

constexpr int kRG = 4;            // lanes per column
constexpr int kCPL = 2;           // columns per lane
constexpr int kCW = 32 / kRG * kCPL;   // columns per warp

template <int NP>
struct SmallCfg {
  static constexpr int kWarps = NP / kCW;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kR = NP / kRG;    // rows per lane
  static constexpr int kB = kR / 4;      // float4 blocks per lane (4*kRG matrix rows each)
  static constexpr int kBlockRows = 4 * kRG;
  // Column ownership is blocked (warp w owns 16 consecutive columns), so warps retire
  // as the factorisation passes them.
  static constexpr int kKKStep = 8;      // between a lane's kk columns
};

__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Sum over the kRG lanes of a column (lane bits 3 and 4).
__device__ __forceinline__ float col_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

// Shared state: U[j][rg][b] = rows rg + kRG*(4b..4b+3) of u_j; S[j] = tau_j / v0_j^2.
template <int NP>
struct SmallSmem {
  float4 U[NP][kRG][SmallCfg<NP>::kB];
  float S[NP];
};

template <int NP>
__device__ __forceinline__ int row_of(int rg, int i) { return rg + kRG * i; }

// Write u_c (the calling lanes own column c) into U[c].  Blocks below B0 are zero,
// blocks beyond B0+1 are copied as they are, the rest are masked by row.
template <int NP, int B0>
__device__ __forceinline__ void publish_u(SmallSmem<NP>& sm, const float (&a)[SmallCfg<NP>::kR],
                                          int c, int rg, float v0) {
  constexpr int kB = SmallCfg<NP>::kB;
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = row_of<NP>(rg, 4 * b + q);
      if (b < B0) v[q] = 0.f;
      else if (b > B0 + 1) v[q] = a[4 * b + q];
      else v[q] = row > c ? a[4 * b + q] : (row == c ? v0 : 0.f);
    }
    sm.U[c][rg][b] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Sum of squares of rows > c and the value at row c (c in blocks B0 or B0+1).
template <int NP, int B0>
__device__ __forceinline__ void column_stats(const float (&a)[SmallCfg<NP>::kR], int c, int rg,
                                             float& tail, float& alpha) {
  constexpr int kB = SmallCfg<NP>::kB;
  float t0 = 0.f, t1 = 0.f;
  alpha = 0.f;
#pragma unroll
  for (int b = B0; b < kB; ++b)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int row = row_of<NP>(rg, 4 * b + q);
      const float x = a[4 * b + q];
      if (b > B0 + 1) {
        if (q & 1) t1 = fmaf(x, x, t1); else t0 = fmaf(x, x, t0);
      } else {
        t0 += row > c ? x * x : 0.f;
        alpha += row == c ? x : 0.f;
      }
    }
  tail = t0 + t1;
}

// One geqrf step: apply H_j (u_j, s_j) to this lane's columns; if `pivot`, also
// produce the reflector of column j+1 (held in a[pk] by lanes with cl == (j+1) % 8).
template <int NP, int B0>
__device__ __forceinline__ void geqrf_step(SmallSmem<NP>& sm, float (&a)[kCPL][SmallCfg<NP>::kR], int j,
                                           int n, int rg, int col0, bool pivot, Reflector (&mine)[kCPL]) {
  constexpr int kB = SmallCfg<NP>::kB;
  constexpr int kKK = SmallCfg<NP>::kKKStep;
  float4 u[kB];
#pragma unroll
  for (int b = B0; b < kB; ++b) u[b] = sm.U[j][rg][b];
  const float sj = sm.S[j];
  float d[kCPL];
#pragma unroll
  for (int kk = 0; kk < kCPL; ++kk) {
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
    for (int b = B0; b < kB; ++b) {
      d0 = fmaf(u[b].x, a[kk][4 * b + 0], d0);
      d1 = fmaf(u[b].y, a[kk][4 * b + 1], d1);
      d2 = fmaf(u[b].z, a[kk][4 * b + 2], d2);
      d3 = fmaf(u[b].w, a[kk][4 * b + 3], d3);
    }
    d[kk] = (d0 + d1) + (d2 + d3);
  }
#pragma unroll
  for (int kk = 0; kk < kCPL; ++kk) d[kk] = col_sum(d[kk]);
#pragma unroll
  for (int kk = 0; kk < kCPL; ++kk) {
    const float coef = col0 + kKK * kk > j ? sj * d[kk] : 0.f;
#pragma unroll
    for (int b = B0; b < kB; ++b) {
      a[kk][4 * b + 0] = fmaf(-coef, u[b].x, a[kk][4 * b + 0]);
      a[kk][4 * b + 1] = fmaf(-coef, u[b].y, a[kk][4 * b + 1]);
      a[kk][4 * b + 2] = fmaf(-coef, u[b].z, a[kk][4 * b + 2]);
      a[kk][4 * b + 3] = fmaf(-coef, u[b].w, a[kk][4 * b + 3]);
    }
  }
  if (pivot) {
    const int c = j + 1;
    const int pk = (c % kCW) >> 3;
#pragma unroll
    for (int kk = 0; kk < kCPL; ++kk) {
      if (kk != pk) continue;
      float tail, alpha;
      column_stats<NP, B0>(a[kk], c, rg, tail, alpha);
      tail = col_sum(tail);
      alpha = col_sum(alpha);
      if (col0 + kKK * kk == c) {
        mine[kk] = make_reflector(alpha, tail, c == n - 1);
        publish_u<NP, B0>(sm, a[kk], c, rg, mine[kk].v0);
        if (rg == 0) sm.S[c] = mine[kk].tau * mine[kk].inv_v0 * mine[kk].inv_v0;
      }
    }
  }
}

// One orgqr step: Q[:, col] -= s_j u_j (u_j^T Q[:, col]) for this lane's columns.
template <int NP, int B0>
__device__ __forceinline__ void orgqr_step(const SmallSmem<NP>& sm, float (&q)[kCPL][SmallCfg<NP>::kR],
                                           int j, int rg) {
  constexpr int kB = SmallCfg<NP>::kB;
  float4 u[kB];
#pragma unroll
  for (int b = B0; b < kB; ++b) u[b] = sm.U[j][rg][b];
  const float sj = sm.S[j];
  float d[kCPL];
#pragma unroll
  for (int kk = 0; kk < kCPL; ++kk) {
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
    for (int b = B0; b < kB; ++b) {
      d0 = fmaf(u[b].x, q[kk][4 * b + 0], d0);
      d1 = fmaf(u[b].y, q[kk][4 * b + 1], d1);
      d2 = fmaf(u[b].z, q[kk][4 * b + 2], d2);
      d3 = fmaf(u[b].w, q[kk][4 * b + 3], d3);
    }
    d[kk] = (d0 + d1) + (d2 + d3);
  }
#pragma unroll
  for (int kk = 0; kk < kCPL; ++kk) {
    const float coef = sj * col_sum(d[kk]);
#pragma unroll
    for (int b = B0; b < kB; ++b) {
      q[kk][4 * b + 0] = fmaf(-coef, u[b].x, q[kk][4 * b + 0]);
      q[kk][4 * b + 1] = fmaf(-coef, u[b].y, q[kk][4 * b + 1]);
      q[kk][4 * b + 2] = fmaf(-coef, u[b].z, q[kk][4 * b + 2]);
      q[kk][4 * b + 3] = fmaf(-coef, u[b].w, q[kk][4 * b + 3]);
    }
  }
}

template <int NP>
__device__ __forceinline__ void geqrf_step_dispatch(SmallSmem<NP>& sm, float (&a)[kCPL][SmallCfg<NP>::kR],
                                                    int j, int n, int rg, int col0, bool pivot,
                                                    Reflector (&mine)[kCPL]) {
  const int blk = j / SmallCfg<NP>::kBlockRows;
  if (blk == 0) geqrf_step<NP, 0>(sm, a, j, n, rg, col0, pivot, mine);
  else if (blk == 1) geqrf_step<NP, 1>(sm, a, j, n, rg, col0, pivot, mine);
  else if constexpr (SmallCfg<NP>::kB > 2) {
    if (blk == 2) geqrf_step<NP, 2>(sm, a, j, n, rg, col0, pivot, mine);
    else geqrf_step<NP, 3>(sm, a, j, n, rg, col0, pivot, mine);
  }
}

template <int NP>
__device__ __forceinline__ void orgqr_step_dispatch(const SmallSmem<NP>& sm,
                                                    float (&q)[kCPL][SmallCfg<NP>::kR], int j, int rg) {
  const int blk = j / SmallCfg<NP>::kBlockRows;
  if (blk == 0) orgqr_step<NP, 0>(sm, q, j, rg);
  else if (blk == 1) orgqr_step<NP, 1>(sm, q, j, rg);
  else if constexpr (SmallCfg<NP>::kB > 2) {
    if (blk == 2) orgqr_step<NP, 2>(sm, q, j, rg);
    else orgqr_step<NP, 3>(sm, q, j, rg);
  }
}

template <int NP>
__global__ void __launch_bounds__(SmallCfg<NP>::kThreads, NP == 64 ? 7 : 8)
small_qr_kernel(const float* __restrict__ A, float* __restrict__ H, float* __restrict__ tau,
                float* __restrict__ Q, int n, int mode) {
  using C = SmallCfg<NP>;
  constexpr int R = C::kR;
  __shared__ SmallSmem<NP> sm;

  const int64_t b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rg = lane >> 3, cl = lane & 7;
  constexpr int kW = C::kWarps;
  constexpr int kKK = C::kKKStep;
  const int col0 = kCW * warp + cl;          // my columns: col0 + kKK * kk
  const int wlast = kCW * warp + kCW - 1;    // my last column
  const size_t off = (size_t)b * n * n;

  float a[kCPL][R];
  Reflector mine[kCPL];
#pragma unroll
  for (int kk = 0; kk < kCPL; ++kk) mine[kk] = {0.f, 0.f, 1.f, 1.f};

  if (mode & 1) {
    // ---------------- geqrf --------------------------------------------------
#pragma unroll
    for (int kk = 0; kk < kCPL; ++kk)
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const int row = row_of<NP>(rg, i), col = col0 + kKK * kk;
        a[kk][i] = (row < n && col < n) ? __ldg(A + off + (size_t)row * n + col) : 0.f;
      }
    if (warp == 0) {   // reflector of column 0
      float tail, alpha;
      column_stats<NP, 0>(a[0], 0, rg, tail, alpha);
      tail = col_sum(tail);
      alpha = col_sum(alpha);
      if (col0 == 0) {
        mine[0] = make_reflector(alpha, tail, n == 1);
        publish_u<NP, 0>(sm, a[0], 0, rg, mine[0].v0);
        if (rg == 0) sm.S[0] = mine[0].tau * mine[0].inv_v0 * mine[0].inv_v0;
      }
    }
    const int jlast = min(n - 1, wlast);
    for (int j = 0; j <= jlast; ++j) {
      // the warps whose last column is >= j take part in step j
      const int active = kW - j / kCW;
      named_barrier(1, 32 * active);
      const bool pivot = (j + 1 < n) && (j + 1) / kCW == warp;
      if (wlast > j) geqrf_step_dispatch<NP>(sm, a, j, n, rg, col0, pivot, mine);
    }
    // H: divide the sub-diagonal of each column by its v0, beta on the diagonal.
#pragma unroll
    for (int kk = 0; kk < kCPL; ++kk) {
      const int col = col0 + kKK * kk;
      if (col < n) {
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const int row = row_of<NP>(rg, i);
          const float h = row > col ? a[kk][i] * mine[kk].inv_v0 : (row == col ? mine[kk].beta : a[kk][i]);
          if (row < n) H[off + (size_t)row * n + col] = h;
        }
        if (rg == 0) tau[(size_t)b * n + col] = mine[kk].tau;
      }
    }
    __syncthreads();   // all u_j and s_j published
  } else {
    // orgqr only: rebuild u_j = v_j (v0 := 1) and s_j = tau_j from (H, tau).
#pragma unroll
    for (int kk = 0; kk < kCPL; ++kk) {
      const int col = col0 + kKK * kk;
      if (col < n) {
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const int row = row_of<NP>(rg, i);
          a[kk][i] = (row < n && row > col) ? __ldg(H + off + (size_t)row * n + col) : (row == col ? 1.f : 0.f);
        }
        if (rg == 0) sm.S[col] = __ldg(tau + (size_t)b * n + col);
#pragma unroll
        for (int bb = 0; bb < C::kB; ++bb)
          sm.U[col][rg][bb] = make_float4(a[kk][4 * bb], a[kk][4 * bb + 1], a[kk][4 * bb + 2], a[kk][4 * bb + 3]);
      }
    }
    __syncthreads();
  }

  if (mode & 2) {
    // ---------------- orgqr: Q = H_0 ... H_{n-1} I, backward ------------------
#pragma unroll
    for (int kk = 0; kk < kCPL; ++kk)
#pragma unroll
      for (int i = 0; i < R; ++i)
        a[kk][i] = (row_of<NP>(rg, i) == col0 + kKK * kk && col0 + kKK * kk < n) ? 1.f : 0.f;
    // Reflector j only touches columns >= j, so a warp starts at its last column.
    for (int j = min(n - 1, wlast); j >= 0; --j) orgqr_step_dispatch<NP>(sm, a, j, rg);
#pragma unroll
    for (int kk = 0; kk < kCPL; ++kk) {
      const int col = col0 + kKK * kk;
      if (col < n) {
#pragma unroll
        for (int i = 0; i < R; ++i) {
          const int row = row_of<NP>(rg, i);
          if (row < n) Q[off + (size_t)row * n + col] = a[kk][i];
        }
      }
    }
  }
}

// ---- n <= 32: one warp per matrix, lane c owns column c (all 32 rows in registers) ----
// Every dot product over rows stays inside a lane, so a step is one broadcast of column
// j (a shuffle per row below the pivot, every lane forming the same ||x||^2 in the same
// order) and lane-local FMAs -- no barrier and no shared memory.  The steps are fully
// unrolled, so row predicates are resolved at compile time.  geqrf follows
// submissions/v1.py:9-38 (via make_reflector); orgqr is the same backward accumulation as
// the n <= 64 kernel.
constexpr int kTinyWarps = 4;

__global__ void __launch_bounds__(kTinyWarps * 32)
tiny_qr_kernel(const float* __restrict__ A, float* __restrict__ H, float* __restrict__ tau,
               float* __restrict__ Q, int64_t batch, int n, int mode) {
  constexpr unsigned kFull = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int64_t mat = (int64_t)blockIdx.x * kTinyWarps + (threadIdx.x >> 5);
  if (mat >= batch) return;   // whole warp
  const size_t moff = (size_t)mat * n * n;
  const bool col = lane < n;
  float a[32];
  float my_tau = 0.f;
  if (mode & 1) {
#pragma unroll
    for (int r = 0; r < 32; ++r) a[r] = (r < n && col) ? __ldg(A + moff + (size_t)r * n + lane) : 0.f;
    // Reflectors are applied unscaled (u = (v0, x_{j+1}, ..), H_j = I - (tau / v0^2) u u^T);
    // lane j keeps its raw column and scales it once at the end.
    float my_inv = 1.f, my_beta = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < n) {
        const float alpha = __shfl_sync(kFull, a[j], j);
        float x[32];
        float t[4] = {0.f, 0.f, 0.f, 0.f}, d[4] = {0.f, 0.f, 0.f, 0.f};   // 4 chains
#pragma unroll
        for (int r = j + 1; r < 32; ++r) {
          x[r] = __shfl_sync(kFull, a[r], j);
          t[r & 3] = fmaf(x[r], x[r], t[r & 3]);
          d[r & 3] = fmaf(x[r], a[r], d[r & 3]);
        }
        const Reflector f = make_reflector(alpha, (t[0] + t[1]) + (t[2] + t[3]), j == n - 1);
        const float w = fmaf(f.v0, a[j], (d[0] + d[1]) + (d[2] + d[3]));   // u^T a_c
        const float coef = lane > j ? f.tau * f.inv_v0 * f.inv_v0 * w : 0.f;
        a[j] = fmaf(-coef, f.v0, a[j]);
#pragma unroll
        for (int r = j + 1; r < 32; ++r) a[r] = fmaf(-coef, x[r], a[r]);
        if (lane == j) {
          my_inv = f.inv_v0;
          my_beta = f.beta;
          my_tau = f.tau;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      a[r] = r > lane ? a[r] * my_inv : (r == lane ? my_beta : a[r]);
      if (r < n && col) H[moff + (size_t)r * n + lane] = a[r];
    }
    if (col) tau[(size_t)mat * n + lane] = my_tau;
  } else {
#pragma unroll
    for (int r = 0; r < 32; ++r) a[r] = (r < n && col) ? __ldg(H + moff + (size_t)r * n + lane) : 0.f;
    if (col) my_tau = __ldg(tau + (size_t)mat * n + lane);
  }
  if (mode & 2) {
    // Q = H_0 H_1 .. H_{n-1} I, accumulated backwards; lane c owns column c of Q.
    float q[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) q[r] = r == lane ? 1.f : 0.f;
#pragma unroll
    for (int j = 31; j >= 0; --j) {
      if (j < n) {
        const float tj = __shfl_sync(kFull, my_tau, j);
        float v[32];
        float w[4] = {q[j], 0.f, 0.f, 0.f};   // v_j = 1; 4 chains
#pragma unroll
        for (int r = j + 1; r < 32; ++r) {
          v[r] = __shfl_sync(kFull, a[r], j);
          w[r & 3] = fmaf(v[r], q[r], w[r & 3]);
        }
        const float c = tj * ((w[0] + w[1]) + (w[2] + w[3]));
        q[j] -= c;
#pragma unroll
        for (int r = j + 1; r < 32; ++r) q[r] = fmaf(-c, v[r], q[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 32; ++r)
      if (r < n && col) Q[moff + (size_t)r * n + lane] = q[r];
  }
}

}  // namespace

cudaError_t launch_small(const float* A, float* H, float* tau, float* Q,
                         int64_t batch, int n, int mode, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  const double nn = (double)n * n;
  const double bytes = (double)batch * (((mode & 1) ? 8 * nn : 4 * nn) + ((mode & 2) ? 4 * nn : 0) + 4.0 * n);
  const double flops = (double)batch * (((mode & 1) ? 4.0 / 3 : 0) + ((mode & 2) ? 4.0 / 3 : 0)) * nn * n;
  LaunchTimer timer(n <= 32 ? "tiny_qr_kernel" : "small_qr_kernel", s, bytes, flops);
  if (n <= 32) {
    const unsigned grid = (unsigned)((batch + kTinyWarps - 1) / kTinyWarps);
    tiny_qr_kernel<<<grid, kTinyWarps * 32, 0, s>>>(A, H, tau, Q, batch, n, mode);
  } else {
    small_qr_kernel<64><<<(unsigned)batch, SmallCfg<64>::kThreads, 0, s>>>(A, H, tau, Q, n, mode);
  }
  return cudaGetLastError();
}

}  // namespace qrb
