// Wide block reflectors for large n: the trailing update and Q formation applied
// 128 reflectors at a time,
//     C[K:, c0:] -= V op(T) (V^T C[K:, c0:]),   V = H[K:, K:K+128] (unit lower),
// so that each trailing element is streamed through HBM once per 128 columns of the
// factorisation instead of once per 32.  The reference gets its fat trailing GEMMs
// the same way -- 256-wide blocks, geqrf panels and BF16x9 cublasLt products
// (_qr_blocked, submission.py:838-894); here the block is factored as four 32-wide
// panels (qrb_panel.cu) with narrow in-slab updates, and the block's products run on
// the 5th-generation tensor cores in 3xTF32 (two tf32 pieces per operand, three
// products, smallest first; see qrb_apply_tc.cu for the accuracy argument).
//
// Per block (K, width bw <= 128):
//   vsplit_kernel   V (masked to the unit lower trapezoid) -> two tf32 pieces in HBM,
//                   [batch][n][128] each, the B operand of ygemm_kernel.
//   ygemm_kernel    Y[c][j] = sum_r C[r][c] V[r][j] for 128-column strips of C over a
//                   chunk of rows: TMA stages of 32 rows, C split in shared memory,
//                   M=128 N=128 K=8 MMAs into one TMEM accumulator per stage (double
//                   buffered), stage partials summed in fp32 registers.  In geqrf the
//                   first strip is the block itself masked to V, which gives the Gram
//                   matrix V^T V of the block.
//   tbuild_kernel   T (128 x 128) of the block from the four panel T factors and the
//                   Gram matrix: T_ab = -T_aa sum_{a<c<=b} G_ac T_cb.
//   w2tc_kernel     W2[c][a] = sum_j op(T)[a][j] Y[c][j] on the tensor cores, stored
//                   as two tf32 pieces [batch][n][128] (the K-major B operand of the
//                   update).
//   wupdate_kernel  C -= V W2: persistent CTA pairs over (matrix, 256-row tile, strip
//                   group); each CTA's 128 rows of V live in its tensor memory (the
//                   MMA's A operand), C strips of 64 columns (three-slot ring) and
//                   half of their W2 pieces (two-slot ring) stream in by TMA, the
//                   leader issues M=256 N=64 K=8 pair MMAs into four TMEM
//                   accumulators; the epilogue subtracts and stores coalesced rows.
//
// Every wait on another role of the CTA is bounded (mbar_wait_abort): a wait that runs
// out records an error code in g_qrb_device_error and raises a CTA-wide abort flag;
// every role then stops issuing work, the CTA waits (bounded) for its own TMA loads,
// MMAs and stores in flight, releases its tensor memory and exits.  No TMA load uses
// cluster multicast.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "qrb_internal.cuh"
#include "qrb_sm100.cuh"

namespace qrb {
namespace {

using namespace sm100;

constexpr int kWB = kWideNB;   // reflectors per wide block

// The three (A piece, B piece) products of 3xTF32, smallest first.
__device__ __constant__ int kWTermA[3] = {1, 0, 0};
__device__ __constant__ int kWTermB[3] = {0, 1, 0};

__device__ __forceinline__ float vmask_w(float x, int r, int j, int bw) {
  if (j >= bw) return 0.f;
  return r > j ? x : (r == j ? 1.f : 0.f);
}

__device__ __forceinline__ uint32_t off32b_w(int r, int q) {   // 128B swizzle, 32-byte atoms
  return r * 128u + (((((uint32_t)q >> 1) ^ (uint32_t)r) & 3u) << 5) + ((uint32_t)(q & 1) << 4);
}
__device__ __forceinline__ uint32_t off128_w(int r, int q) {   // 128B swizzle
  return r * 128u + ((((uint32_t)q ^ (uint32_t)r) & 7u) << 4);
}

// `err` is the library's device error flag (device_error_flag()).
__device__ __forceinline__ bool wwait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  return mbar_wait_abort(bar, parity, abort, err, code);
}

// ---- vsplit: V pieces of the block ------------------------------------------------------
__global__ void __launch_bounds__(256)
vsplit_kernel(const float* __restrict__ H, float* __restrict__ vp0, float* __restrict__ vp1, int n, int K,
              int bw, int64_t units) {
  const int m = n - K;
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int q = (int)(u & 31);
    const int64_t t = u >> 5;
    const int r = (int)(t % m);
    const int64_t mat = t / m;
    const int j0 = 4 * q;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    if (j0 < bw) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(H + ((size_t)mat * n + K + r) * n + K + j0));
      a[0] = v.x;
      a[1] = v.y;
      a[2] = v.z;
      a[3] = v.w;
    }
    float x0[4], x1[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) split2_tf32(vmask_w(a[e], r, j0 + e, bw), x0[e], x1[e]);
    const size_t o = ((size_t)mat * n + K + r) * kWB + j0;
    *reinterpret_cast<float4*>(vp0 + o) = make_float4(x0[0], x0[1], x0[2], x0[3]);
    *reinterpret_cast<float4*>(vp1 + o) = make_float4(x1[0], x1[1], x1[2], x1[3]);
  }
}

// ---- ygemm: Y = C^T V over a row chunk, per 128-column strip ---------------------------
constexpr int kYStages = 4;
constexpr uint32_t kYBox = 32 * 128;          // 32 rows x 32 fp32
constexpr uint32_t kYPiece = 4 * kYBox;       // 32 rows x 128 columns
constexpr uint32_t kYStage = 3 * kYPiece;     // C (raw), then V pieces 0, 1
constexpr uint32_t kYOffV = kYPiece;
constexpr uint32_t kYBarOff = kYStages * kYStage;
constexpr uint32_t kSmemY = kYBarOff + 256 + 1024;
constexpr int kYThreads = 320;   // producer, MMA, 4 converter warps, 4 gather warps

struct YBars {
  uint64_t full[kYStages], split[kYStages], sfree[kYStages], accf[2], acce[2], drain;
  uint32_t tmem;
  int abort;
};

// MODE 0 (geqrf): strip 0 is the block itself, read from H and masked to V (the Gram
// matrix); other strips read `src`.  MODE 1 (orgqr): entries with row or column below
// K + bw are the identity (Q not yet formed there).
template <int MODE>
__global__ void __launch_bounds__(kYThreads, 1)
ygemm_kernel(const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_h,
             const __grid_constant__ CUtensorMap map_v0, const __grid_constant__ CUtensorMap map_v1,
             float* __restrict__ ypart, int64_t batch, int n, int K, int bw, int nstrips, int chunk, int nsplit,
             int ncolsY, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  YBars& bars = *reinterpret_cast<YBars*>(sm + kYBarOff);
  volatile int* abort = &bars.abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x % nsplit;
  const int t = blockIdx.x / nsplit;
  const int strip = t % nstrips;
  const int mat = t / nstrips;
  const int cs = K + strip * kWB;
  const int r0 = K + split * chunk;
  const int r1 = min(n, r0 + chunk);
  const int nst = (r1 - r0 + 31) / 32;
  const int kb = K + bw;
  const bool gram = (MODE == 0 && strip == 0);

  if (tid == 0) {
    for (int i = 0; i < kYStages; ++i) {
      mbar_init(&bars.full[i], 1);
      mbar_init(&bars.split[i], 4);
      mbar_init(&bars.sfree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.accf[i], 1);
      mbar_init(&bars.acce[i], 4);
    }
    mbar_init(&bars.drain, 1);
    bars.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bars.tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;
  constexpr uint32_t kYA = 256;   // A (C^T pieces) per stage: columns kYA + 64 st (piece 0), + 32 (piece 1)

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const CUtensorMap* cmap = gram ? &map_h : &map_c;
      prefetch_tensormap(cmap);
      prefetch_tensormap(&map_v0);
      prefetch_tensormap(&map_v1);
      int last_use[kYStages] = {-1, -1, -1, -1};
      for (int s = 0; s < nst; ++s) {
        const int st = s % kYStages, use = s / kYStages;
        if (use > 0 && !wwait(&bars.sfree[st], (use - 1) & 1, abort, err, 31)) break;
        unsigned char* sb = sm + st * kYStage;
        const int y = r0 + s * 32;
        mbar_arrive_expect_tx(&bars.full[st], kYPiece + 2 * kYPiece);
#pragma unroll
        for (int j = 0; j < 4; ++j) tma_load_3d(sb + j * kYBox, cmap, cs + 32 * j, y, mat, &bars.full[st]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          tma_load_3d(sb + kYOffV + j * kYBox, &map_v0, 32 * j, y, mat, &bars.full[st]);
          tma_load_3d(sb + kYOffV + kYPiece + j * kYBox, &map_v1, 32 * j, y, mat, &bars.full[st]);
        }
        last_use[st] = use;
      }
      if (*abort) {   // let every load this CTA issued land before its shared memory goes away
        for (int st = 0; st < kYStages; ++st)
          if (last_use[st] >= 0) mbar_wait(&bars.full[st], last_use[st] & 1, 1u << 22);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(128, 128, 0, 1);   // A from tensor memory, B MN-major
      bool issued = false;
      for (int s = 0; s < nst; ++s) {
        const int st = s % kYStages, acc = s & 1;
        if (!wwait(&bars.split[st], (s / kYStages) & 1, abort, err, 32)) break;
        if (s >= 2 && !wwait(&bars.acce[acc], ((s >> 1) - 1) & 1, abort, err, 33)) break;
        tc_fence_after();
        const uint32_t base = smem_u32(sm + st * kYStage);
        const uint32_t d = tmem + acc * 128;
#pragma unroll
        for (int tt = 0; tt < 3; ++tt) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t a = tmem + kYA + 64 * st + 32 * kWTermA[tt] + 8 * kk;
            const uint64_t bd = sdesc_sw128_32b(base + kYOffV + kWTermB[tt] * kYPiece + kk * 1024, kYBox, 512);
            mma_tf32_ta(d, a, bd, idesc, (tt > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&bars.accf[acc]);
        mma_commit(&bars.sfree[st]);
        issued = true;
      }
      if (*abort && issued) {   // tensor memory must not be released under running MMAs
        mma_commit(&bars.drain);
        mbar_wait(&bars.drain, 0, 1u << 22);
      }
    }
  } else if (warp < 6) {
    // ---------------- converters: C^T pieces into the tensor memory ----------------
    // Thread = strip column c = TMEM lane (warp w writes lanes 32 (w % 4)..): its 32 rows
    // of the stage, split into two tf32 pieces, become K columns of the A operand.  Taking
    // A from the tensor memory halves the MMAs' shared-memory reads, and the split pieces
    // are no longer written back to shared memory: the stage loop was bound by shared-
    // memory bandwidth (TMA writes, converter traffic and both MMA operands).
    const int qd = warp & 3;
    const int c = 32 * qd + lane;
    const uint32_t tl = (uint32_t)(32 * qd) << 16;
    const int Cc = cs + c;
    for (int s = 0; s < nst; ++s) {
      const int st = s % kYStages;
      if (!wwait(&bars.full[st], (s / kYStages) & 1, abort, err, 34)) break;
      const unsigned char* p0 = sm + st * kYStage + (c >> 5) * kYBox + (c & 3) * 4;
      const int y = r0 + s * 32;
      float x0[32], x1[32];
#pragma unroll
      for (int r = 0; r < 32; ++r) {
        float a = *reinterpret_cast<const float*>(p0 + off32b_w(r, (c & 31) >> 2));
        const int R = y + r;
        if (MODE == 0) {
          if (gram) a = vmask_w(a, R - K, Cc - K, bw);
        } else {
          if (R < n && Cc < n && (R < kb || Cc < kb)) a = R == Cc ? 1.f : 0.f;
        }
        split2_tf32(a, x0[r], x1[r]);
      }
      tmem_st32(tmem + tl + kYA + 64 * st, x0);
      tmem_st32(tmem + tl + kYA + 64 * st + 32, x1);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.split[st]);
    }
  } else {
    // ---------------- gatherers: stage partials -> fp32 register sums ----------------
    const int q = warp & 3;   // TMEM lanes 32q.. = strip columns 32q + lane
    float y[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) y[j] = 0.f;
    bool ok = true;
    for (int s = 0; s < nst; ++s) {
      const int acc = s & 1;
      if (!wwait(&bars.accf[acc], (s >> 1) & 1, abort, err, 35)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float p[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + acc * 128 + 32 * c, p);
#pragma unroll
        for (int j = 0; j < 32; ++j) y[32 * c + j] += p[j];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.acce[acc]);
    }
    if (ok && !*abort) {
      const int i = 32 * q + lane;
      float4* dst = reinterpret_cast<float4*>(
          ypart + ((((size_t)split * batch + mat) * ncolsY) + (cs - K) + i) * kWB);
#pragma unroll
      for (int c = 0; c < 32; ++c) dst[c] = make_float4(y[4 * c], y[4 * c + 1], y[4 * c + 2], y[4 * c + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- tbuild: T of the wide block from the panel T factors and the Gram matrix -----------
constexpr uint32_t kSmemT = (2 * 128 * 129 + 32 * 33) * 4;

__global__ void __launch_bounds__(256)
tbuild_kernel(const float* __restrict__ ypart, int nsplit, int64_t batch, int ncolsY,
              const float* __restrict__ t32, int np, float* __restrict__ t128) {
  extern __shared__ float smw[];
  float(*G)[129] = reinterpret_cast<float(*)[129]>(smw);
  float(*X)[129] = reinterpret_cast<float(*)[129]>(smw + 128 * 129);
  float(*S)[33] = reinterpret_cast<float(*)[33]>(smw + 2 * 128 * 129);
  const int tid = threadIdx.x;
  // One CTA per (matrix, 32-column block b of T): column block b depends only on the
  // blocks above it in the same column (T_ab = -T_aa sum_{a<c<=b} G_ac T_cb).
  const int64_t mat = blockIdx.x >> 2;
  const int bcol = (int)(blockIdx.x & 3);
  // Gram strip (summed over the row chunks) and the diagonal T blocks, 16 float4 per
  // thread with all loads in flight before the shared-memory stores.
  {
    float4 g[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) g[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsplit; ++sp) {
      const float4* src = reinterpret_cast<const float4*>(ypart + ((size_t)sp * batch + mat) * ncolsY * kWB);
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float4 v = __ldg(src + tid + 256 * k);
        g[k].x += v.x;
        g[k].y += v.y;
        g[k].z += v.z;
        g[k].w += v.w;
      }
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int u = tid + 256 * k, i = u >> 5, j = 4 * (u & 31);
      G[i][j] = g[k].x;
      G[i][j + 1] = g[k].y;
      G[i][j + 2] = g[k].z;
      G[i][j + 3] = g[k].w;
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int u = tid + 256 * k, i = u >> 5, j = 4 * (u & 31);
      const int a = i >> 5, b = j >> 5;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (a == b && a < np)
        t = __ldg(reinterpret_cast<const float4*>(t32 + ((size_t)a * batch + mat) * 1024 + (i & 31) * 32 + (j & 31)));
      X[i][j] = t.x;
      X[i][j + 1] = t.y;
      X[i][j + 2] = t.z;
      X[i][j + 3] = t.w;
    }
  }
  __syncthreads();
  const int ti = tid >> 3, tj = (tid & 7) * 4;
  for (int b = bcol; b == bcol && b < np; ++b) {
    for (int a = b - 1; a >= 0; --a) {
      // S = sum_{c=a+1..b} G_ac X_cb
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = a + 1; c <= b; ++c) {
#pragma unroll 8
        for (int l = 0; l < 32; ++l) {
          const float g = G[32 * a + ti][32 * c + l];
#pragma unroll
          for (int e = 0; e < 4; ++e) s[e] = fmaf(g, X[32 * c + l][32 * b + tj + e], s[e]);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) S[ti][tj + e] = s[e];
      __syncthreads();
      // X_ab = -T_aa S
      float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
      for (int l = 0; l < 32; ++l) {
        const float x = X[32 * a + ti][32 * a + l];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = fmaf(x, S[l][tj + e], o[e]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) X[32 * a + ti][32 * b + tj + e] = -o[e];
      __syncthreads();
    }
  }
  // Column block bcol of T (rows 0-127, 32 columns).
  float4* T = reinterpret_cast<float4*>(t128 + (size_t)mat * kWB * kWB);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int u = tid + 256 * k, i = u >> 3, j = 32 * bcol + 4 * (u & 7);
    T[i * 32 + (j >> 2)] = make_float4(X[i][j], X[i][j + 1], X[i][j + 2], X[i][j + 3]);
  }
}

// ---- w2tc: W2 = Y op(T)^T on the tensor cores ------------------------------------------------
// One CTA per (matrix, 128 columns): D[c][a] = sum_j Y[c][j] op(T)[a][j] as M=128 N=128
// K=8 tf32 MMAs (3xTF32).  Y (the columns' rows of the Y partials, summed over the row
// chunks) is split into the tensor memory (A operand, lane = column); op(T)^T is staged
// by TMA and split in place in shared memory (B operand: T itself for geqrf, which is
// then MN-major, or T^T for orgqr, K-major); the result is split into the two W2 pieces
// and leaves through TMA stores.  Replaces w2build_kernel's fp32 SIMT product.
constexpr uint32_t kW2TBox32 = 32 * 128;      // 32 rows x 32 fp32
constexpr uint32_t kW2TBox128 = 128 * 128;    // 128 rows x 32 fp32
constexpr uint32_t kW2TPiece = 4 * kW2TBox128;   // 64 KB: a 128 x 128 operand
constexpr uint32_t kW2TOffY = 2 * kW2TPiece;     // T pieces first, then the raw Y tile
constexpr uint32_t kW2TBar = kW2TOffY + kW2TPiece;
constexpr uint32_t kSmemW2T = kW2TBar + 64 + 1024;

template <int TRANS>
__global__ void __launch_bounds__(128, 1)
w2tc_kernel(const __grid_constant__ CUtensorMap map_t, const __grid_constant__ CUtensorMap map_y,
            const __grid_constant__ CUtensorMap map_w0, const __grid_constant__ CUtensorMap map_w1, int64_t batch,
            int n, int K, int cfirst, int ngroups, int nsplit, int blk, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  uint64_t* tbar = reinterpret_cast<uint64_t*>(sm + kW2TBar);
  uint64_t* ybar = tbar + 1;
  uint64_t* mbar = tbar + 2;   // two: one per accumulator buffer
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tbar + 4);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int mat = (int)(blockIdx.x / ngroups);
  const int cg = cfirst + (int)(blockIdx.x % ngroups) * 128;   // first column of the group
  const int zt = blk * (int)batch + mat;                        // T factor index (block, matrix)

  if (tid == 0) {
    mbar_init(tbar, 1);
    mbar_init(ybar, 1);
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_mbar_init();
    prefetch_tensormap(&map_t);
    prefetch_tensormap(&map_y);
    // T lands raw in piece 0; geqrf: 16 boxes (32 a x 32 j rows, MN-major B, 32-byte
    // atoms), orgqr: 4 boxes (32 j x 128 a rows, K-major B).
    mbar_arrive_expect_tx(tbar, kW2TPiece);
    if (TRANS) {
      for (int jb = 0; jb < 4; ++jb)
        for (int ab = 0; ab < 4; ++ab)
          tma_load_3d(sm + (jb * 4 + ab) * kW2TBox32, &map_t, 32 * ab, 32 * jb, zt, tbar);
    } else {
      for (int jb = 0; jb < 4; ++jb) tma_load_3d(sm + jb * kW2TBox128, &map_t, 32 * jb, 0, zt, tbar);
    }
    mbar_arrive_expect_tx(ybar, kW2TPiece);
    for (int jb = 0; jb < 4; ++jb)
      tma_load_3d(sm + kW2TOffY + jb * kW2TBox128, &map_y, 32 * jb, cg - K, mat, ybar);
  }
  if (warp == 0) tmem_alloc(tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tl = (uint32_t)(32 * warp) << 16;
  bool bad = false;

  // ---- T -> two tf32 pieces in place (piece 1 64 KB further) ----
  bad = !mbar_wait(tbar, 0);
  if (!__syncthreads_or(bad)) {
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
      const int u = tid + 128 * i;   // float4 index 0..4095
      uint32_t off;
      if (TRANS) {
        const int bx = u >> 8, r = (u >> 3) & 31, q = u & 7;
        off = bx * kW2TBox32 + off32b_w(r, q);
      } else {
        const int bx = u >> 10, r = (u >> 3) & 127, q = u & 7;
        off = bx * kW2TBox128 + off128_w(r, q);
      }
      const float4 v = *reinterpret_cast<const float4*>(sm + off);
      const float a4[4] = {v.x, v.y, v.z, v.w};
      float x0[4], x1[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) split2_tf32(a4[e], x0[e], x1[e]);
      *reinterpret_cast<float4*>(sm + off) = make_float4(x0[0], x0[1], x0[2], x0[3]);
      *reinterpret_cast<float4*>(sm + kW2TPiece + off) = make_float4(x1[0], x1[1], x1[2], x1[3]);
    }
    fence_proxy_async();
  } else {
    bad = true;
  }

  // ---- Y rows (thread = column), summed over the row chunks, into the tensor memory ----
  float y[128];
#pragma unroll
  for (int j = 0; j < 128; ++j) y[j] = 0.f;
  for (int sp = 0; sp < nsplit && !bad; ++sp) {
    bad = !mbar_wait(ybar, sp & 1);
    if (__syncthreads_or(bad)) {
      bad = true;
      break;
    }
#pragma unroll
    for (int jb = 0; jb < 4; ++jb)
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(sm + kW2TOffY + jb * kW2TBox128 + off128_w(tid, q));
        y[32 * jb + 4 * q] += v.x;
        y[32 * jb + 4 * q + 1] += v.y;
        y[32 * jb + 4 * q + 2] += v.z;
        y[32 * jb + 4 * q + 3] += v.w;
      }
    __syncthreads();   // every row read before the next partial overwrites the tile
    if (tid == 0 && sp + 1 < nsplit) {
      mbar_arrive_expect_tx(ybar, kW2TPiece);
      for (int jb = 0; jb < 4; ++jb)
        tma_load_3d(sm + kW2TOffY + jb * kW2TBox128, &map_y, 32 * jb, cg - K, (sp + 1) * (int)batch + mat, ybar);
    }
  }
  if (!bad) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float x0[32], x1[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) split2_tf32(y[32 * c + j], x0[j], x1[j]);
      tmem_st32(tmem + tl + 32 * c, x0);
      tmem_st32(tmem + tl + 128 + 32 * c, x1);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  bad = __syncthreads_or(bad);
  // Four K stages of 32 (12 MMAs each, small products first) into two alternating TMEM
  // accumulators; the stage partials are summed in fp32 registers (reusing y[]).  One
  // long tensor-core accumulation rounds every add against the running sum and costs
  // accuracy (orthogonality at n = 2048 5.7e-6 against 3.7e-6 with stages).
  constexpr uint32_t idesc = idesc_tf32(128, 128, 0, TRANS ? 1 : 0);
  auto issue_stage = [&](int st) {
    tc_fence_after();
    const uint32_t tb = smem_u32(sm);
    const uint32_t d = tmem + 256 + (st & 1) * 128;
#pragma unroll
    for (int tt = 0; tt < 3; ++tt) {
#pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const int kk = 4 * st + k4;
        const uint32_t bb = tb + kWTermB[tt] * kW2TPiece;
        const uint64_t bd = TRANS ? sdesc_sw128_32b(bb + (kk >> 2) * 4 * kW2TBox32 + (kk & 3) * 1024, kW2TBox32, 512)
                                  : sdesc_sw128(bb + (kk >> 2) * kW2TBox128 + (kk & 3) * 32, 16, 1024);
        mma_tf32_ta(d, tmem + kWTermA[tt] * 128 + kk * 8, bd, idesc, (tt > 0 || k4 > 0) ? 1u : 0u);
      }
    }
    mma_commit(&mbar[st & 1]);
  };
  if (!bad && tid == 0) {
    issue_stage(0);
    issue_stage(1);
  }
#pragma unroll
  for (int j = 0; j < 128; ++j) y[j] = 0.f;
  for (int st = 0; st < 4 && !bad; ++st) {
    bad = !mbar_wait(&mbar[st & 1], (st >> 1) & 1);
    if (__syncthreads_or(bad)) {
      bad = true;
      if (tid == 0) atomicCAS(err, 0, 61);
      break;
    }
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float d[32];
      tmem_ld32(tmem + tl + 256 + (st & 1) * 128 + 32 * c, d);
#pragma unroll
      for (int j = 0; j < 32; ++j) y[32 * c + j] += d[j];
    }
    tc_fence_before();
    __syncthreads();   // the buffer is read by every warp before stage st + 2 overwrites it
    if (tid == 0 && st + 2 < 4) issue_stage(st + 2);
  }
  bad = __syncthreads_or(bad);
  if (!bad) {
    // W2 row c (this thread's column) -> pieces, staged K-major over the T buffers (free:
    // every MMA has completed) for the stores.
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float x0[4], x1[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) split2_tf32(y[32 * c + 4 * q + e], x0[e], x1[e]);
        const uint32_t off = c * kW2TBox128 + off128_w(tid, q);
        *reinterpret_cast<float4*>(sm + off) = make_float4(x0[0], x0[1], x0[2], x0[3]);
        *reinterpret_cast<float4*>(sm + kW2TPiece + off) = make_float4(x1[0], x1[1], x1[2], x1[3]);
      }
    }
    fence_proxy_async();
  }
  tc_fence_before();
  bad = __syncthreads_or(bad);
  if (!bad && tid == 0) {
    for (int c = 0; c < 4; ++c) {
      tma_store_3d(&map_w0, sm + c * kW2TBox128, 32 * c, cg, mat);
      tma_store_3d(&map_w1, sm + kW2TPiece + c * kW2TBox128, 32 * c, cg, mat);
    }
    tma_store_commit();
    tma_store_wait_all();
  }
  if (bad && tid == 0) atomicCAS(err, 0, 60);
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- wupdate: C -= V W2 with V in tensor memory, by CTA pairs -----------------------------
// A 2-CTA cluster owns 256 rows (128 per CTA) of one matrix and a group of 64-column
// strips.  Each CTA splits its 128 x 128 V tile into its own tensor memory; the even
// (leader) CTA issues M=256 N=64 K=8 pair MMAs (cta_group::2) whose B operand -- the
// strip's W2 pieces -- is split along N between the two CTAs' shared memory, so each
// CTA streams only half of W2 per strip: as many W2 bytes from L2 as C bytes from HBM.
// (With single-CTA M=128 tiles W2 traffic was twice the C traffic and its L2 latency
// set the pace; a tf32 MMA also costs at least ~44 cycles whatever its N, so N=32
// strips were MMA-issue-bound.)
// Warp roles per CTA: 0 = C and V producer, 1 = MMA issuer (leader) and TMEM owner,
// 2-5 and 7-10 = two epilogue warpgroups taking alternate strips (C -= V W2), 6 = W2
// producer, 11-14 = V splitter (each item's V tile into the tensor memory).
// Barriers the MMA waits on live in the leader (W2 landed in both CTAs, both CTAs'
// epilogues done with an accumulator, both V tiles ready); the leader's commits arrive
// in both CTAs.
constexpr int kUCSlots = 3;                        // half-strips of C (64 columns)
constexpr int kUWSlots = 4;                        // W2 chunks (K = 32)
constexpr int kUAcc = 2;
constexpr int kUTN = 128;                          // strip width (N of the pair MMA)
constexpr int kUHalf = kUTN / 2;                   // W2 columns each CTA holds
constexpr uint32_t kUCBox = 128 * 128;             // 128 rows x 32 fp32
constexpr uint32_t kUCSlot = 2 * kUCBox;           // one C half-strip: 128 rows x 64 columns
constexpr uint32_t kUOffV = 0;                     // V staging: 4 boxes of 128 rows x 32
constexpr uint32_t kUWPiece = kUHalf * 128;        // 64 strip columns x 32 K values (8 KB)
constexpr uint32_t kUWSlot = 2 * kUWPiece;         // one K chunk, two tf32 pieces
constexpr uint32_t kUOffW = kUOffV + 4 * kUCBox;
constexpr uint32_t kUOffC = kUOffW + kUWSlots * kUWSlot;
constexpr uint32_t kUBarOff = kUOffC + kUCSlots * kUCSlot;
constexpr uint32_t kSmemU = kUBarOff + 512 + 1024;
constexpr int kUThreads = 480;

struct UBars {
  uint64_t cfull[kUCSlots], cempty[kUCSlots], wfull[kUWSlots], wempty[kUWSlots], vfull, vempty, vready,
      accf[kUAcc], acce[kUAcc], drain, vdone;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(UBars) <= 512, "barrier block");
static_assert(kSmemU <= 232448, "shared memory");

struct UItem {
  int mat, y0, s0, s1;   // y0: first row of the pair's 256-row tile
};

__device__ __forceinline__ UItem u_item(int64_t item, int K, int ntiles, int ngroups, int gsize, int nstrips) {
  UItem it;
  const int g = (int)(item % ngroups);
  const int64_t t = item / ngroups;
  it.y0 = K + (int)(t % ntiles) * 256;
  it.mat = (int)(t / ntiles);
  it.s0 = g * gsize;
  it.s1 = min(nstrips, it.s0 + gsize);
  return it;
}

template <bool IDENT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kUThreads, 1)
wupdate_kernel(const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_src, float* dst,
               const __grid_constant__ CUtensorMap map_w0, const __grid_constant__ CUtensorMap map_w1, int64_t batch,
               int n, int K, int bw, int c0, int nstrips, int ntiles, int ngroups, int gsize, int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  UBars& bars = *reinterpret_cast<UBars*>(sm + kUBarOff);
  volatile int* abort = &bars.abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int kb = K + bw;
  const int64_t nitems = batch * ntiles * ngroups;
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int rowoff = 128 * (int)rank;   // this CTA's rows within the pair's tile

  if (tid == 0) {
    for (int i = 0; i < kUCSlots; ++i) {
      mbar_init(&bars.cfull[i], 1);
      mbar_init(&bars.cempty[i], 4);
    }
    for (int i = 0; i < kUWSlots; ++i) {
      mbar_init(&bars.wfull[i], 1);
      mbar_init(&bars.wempty[i], 1);
    }
    mbar_init(&bars.vfull, 1);
    mbar_init(&bars.vempty, 4);
    mbar_init(&bars.vready, 8);   // both CTAs' epilogue warps (leader's copy is used)
    for (int i = 0; i < kUAcc; ++i) {
      mbar_init(&bars.accf[i], 1);
      mbar_init(&bars.acce[i], 8);   // both CTAs' epilogue warps (leader's copy is used)
    }
    mbar_init(&bars.drain, 1);
    mbar_init(&bars.vdone, 1);
    bars.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(&bars.tmem, 512);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();   // the peer's barriers exist before anything is signalled across the pair
  tc_fence_after();
  const uint32_t tmem = bars.tmem;
  constexpr uint32_t kAcc = 256;   // accumulators after the two V pieces (128 columns each)
  // The leader's copies of the barriers both CTAs signal.
  const uint32_t lead_wfull0 = mapa_shared(smem_u32(&bars.wfull[0]), 0);
  const uint32_t lead_acce0 = mapa_shared(smem_u32(&bars.acce[0]), 0);
  const uint32_t lead_vready = mapa_shared(smem_u32(&bars.vready), 0);

  if (warp == 0) {
    // ---------------- C and V producer (each CTA, its own rows) ----------------
    if (lane == 0) {
      prefetch_tensormap(&map_src);
      prefetch_tensormap(&map_v);
      int gs = 0, iter = 0, v_last = -1;
      int last_use[kUCSlots];
#pragma unroll
      for (int i = 0; i < kUCSlots; ++i) last_use[i] = -1;
      bool stop = false;
      for (int64_t item = pair; item < nitems && !stop; item += npairs, ++iter) {
        const UItem it = u_item(item, K, ntiles, ngroups, gsize, nstrips);
        const int y = it.y0 + rowoff;
        if (iter > 0 && !wwait(&bars.vempty, (iter - 1) & 1, abort, err, 41)) break;
        mbar_arrive_expect_tx(&bars.vfull, 4 * kUCBox);
#pragma unroll
        for (int j = 0; j < 4; ++j) tma_load_3d(sm + kUOffV + j * kUCBox, &map_v, K + 32 * j, y, it.mat, &bars.vfull);
        v_last = iter;
        for (int hs = 2 * it.s0; hs < 2 * it.s1; ++hs, ++gs) {   // half-strips
          const int slot = gs % kUCSlots, use = gs / kUCSlots;
          if (use > 0 && !wwait(&bars.cempty[slot], (use - 1) & 1, abort, err, 42)) {
            stop = true;
            break;
          }
          mbar_arrive_expect_tx(&bars.cfull[slot], kUCSlot);
          unsigned char* cb = sm + kUOffC + slot * kUCSlot;
          tma_load_3d(cb, &map_src, c0 + hs * 64, y, it.mat, &bars.cfull[slot]);
          tma_load_3d(cb + kUCBox, &map_src, c0 + hs * 64 + 32, y, it.mat, &bars.cfull[slot]);
          last_use[slot] = use;
        }
      }
      if (*abort) {   // let every load this CTA issued land before its shared memory goes away
        if (v_last >= 0) mbar_wait(&bars.vfull, v_last & 1, 1u << 22);
        for (int sl = 0; sl < kUCSlots; ++sl)
          if (last_use[sl] >= 0) mbar_wait(&bars.cfull[sl], last_use[sl] & 1, 1u << 22);
      }
    }
  } else if (warp == 6) {
    // ---------------- W2 producer (each CTA, its half of the strip's columns) ----------------
    if (lane == 0) {
      prefetch_tensormap(&map_w0);
      prefetch_tensormap(&map_w1);
      int gs = 0;
      int last_use[kUWSlots];
#pragma unroll
      for (int i = 0; i < kUWSlots; ++i) last_use[i] = -1;
      bool stop = false;
      for (int64_t item = pair; item < nitems && !stop; item += npairs) {
        const UItem it = u_item(item, K, ntiles, ngroups, gsize, nstrips);
        for (int cidx = 4 * it.s0; cidx < 4 * it.s1; ++cidx, ++gs) {   // K chunks of strips
          const int slot = gs % kUWSlots, use = gs / kUWSlots;
          if (use > 0 && !wwait(&bars.wempty[slot], (use - 1) & 1, abort, err, 50)) {
            stop = true;
            break;
          }
          unsigned char* sl = sm + kUOffW + slot * kUWSlot;
          const int cs = c0 + (cidx >> 2) * kUTN + kUHalf * (int)rank, kc = cidx & 3;
          const uint32_t bar = lead_wfull0 + slot * (uint32_t)sizeof(uint64_t);
          // The leader expects both halves' bytes; the peer's copies count on the leader's barrier.
          if (leader) mbar_arrive_expect_tx(&bars.wfull[slot], 2 * kUWSlot);
          tma_load_3d_pair(sl, &map_w0, 32 * kc, cs, it.mat, bar);
          tma_load_3d_pair(sl + kUWPiece, &map_w1, 32 * kc, cs, it.mat, bar);
          last_use[slot] = use;
        }
      }
      (void)last_use;   // after an abort the leader's drain waits for both halves (see the MMA role)
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_tf32(256, kUTN, 0, 0);
      int gs = 0, gc = 0, iter = 0;
      bool issued = false, stop = false;
      int w_last[kUWSlots];
#pragma unroll
      for (int i = 0; i < kUWSlots; ++i) w_last[i] = -1;
      for (int64_t item = pair; item < nitems && !stop; item += npairs, ++iter) {
        const UItem it = u_item(item, K, ntiles, ngroups, gsize, nstrips);
        if (!wwait(&bars.vready, iter & 1, abort, err, 43)) break;
        for (int s = it.s0; s < it.s1 && !stop; ++s, ++gs) {
          const int acc = gs % kUAcc;
          if (gs >= kUAcc && !wwait(&bars.acce[acc], ((gs / kUAcc) - 1) & 1, abort, err, 45)) {
            stop = true;
            break;
          }
          const uint32_t d = tmem + kAcc + acc * kUTN;
          // The strip's four K chunks stay resident: the two small products of every chunk
          // go in first, then the hi x hi products, releasing each chunk after its last use
          // (the small terms accumulate before the large ones over the whole K, as in one
          // K = 128 chain; chunk-by-chunk order measurably loses accuracy).
          for (int pass = 0; pass < 2 && !stop; ++pass) {
            for (int kc = 0; kc < 4; ++kc) {
              const int g = gc + kc, slot = g % kUWSlots;
              if (pass == 0) {
                w_last[slot] = g / kUWSlots;
                if (!wwait(&bars.wfull[slot], (g / kUWSlots) & 1, abort, err, 44)) {
                  stop = true;
                  break;
                }
                tc_fence_after();
              }
              const uint32_t wb = smem_u32(sm + kUOffW + slot * kUWSlot);
#pragma unroll
              for (int tt = 0; tt < 3; ++tt) {
                if ((tt == 2) != (pass == 1)) continue;
#pragma unroll
                for (int k4 = 0; k4 < 4; ++k4) {
                  const uint32_t a = tmem + kWTermA[tt] * 128 + (4 * kc + k4) * 8;
                  // Each CTA's half: 64 rows (strip columns) x 32 K values, K-major.
                  const uint64_t bd = sdesc_sw128(wb + kWTermB[tt] * kUWPiece + k4 * 32, 16, 1024);
                  mma_tf32_ta_pair(d, a, bd, idesc, (pass > 0 || kc > 0 || tt > 0 || k4 > 0) ? 1u : 0u);
                }
              }
              if (pass == 1) mma_commit_pair(&bars.wempty[slot]);
              issued = true;
            }
          }
          gc += 4;
          if (!stop) mma_commit_pair(&bars.accf[acc]);
        }
        if (!stop) mma_commit_pair(&bars.vdone);   // the item's MMAs no longer read V
      }
      if (*abort) {
        if (issued) {   // tensor memory must not be released under running MMAs
          mma_commit_pair(&bars.drain);
          mbar_wait(&bars.drain, 0, 1u << 22);
        }
        for (int sl = 0; sl < kUWSlots; ++sl)   // both CTAs' W2 copies have landed
          if (w_last[sl] >= 0) mbar_wait(&bars.wfull[sl], w_last[sl] & 1, 1u << 22);
      }
    }
  } else if (warp >= 11) {
    // ---------------- V splitter (warps 11-14) ----------------
    // V rows of this CTA, masked to the unit lower trapezoid, split into the tensor memory
    // once the previous item's MMAs have completed (`vdone`, committed once per item: one
    // phase per item, and the MMAs of item i + 1 wait for this split, so the wait is never
    // more than one phase behind).  A warpgroup of its own, so that the next item's MMAs
    // wait only for the split, not for an epilogue warpgroup to finish its last strip.
    const int q = warp & 3;
    const int r = 32 * q + lane;   // row within this CTA's 128 = TMEM lane
    const uint32_t tl = (uint32_t)(32 * q) << 16;
    int iter = 0;
    for (int64_t item = pair; item < nitems; item += npairs, ++iter) {
      const UItem it = u_item(item, K, ntiles, ngroups, gsize, nstrips);
      const int R = it.y0 + rowoff + r;
      if (iter > 0 && !wwait(&bars.vdone, (iter - 1) & 1, abort, err, 51)) break;
      if (!wwait(&bars.vfull, iter & 1, abort, err, 46)) break;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x0[32], x1[32];
        const unsigned char* box = sm + kUOffV + c * kUCBox;
#pragma unroll
        for (int qq = 0; qq < 8; ++qq) {
          const float4 v = *reinterpret_cast<const float4*>(box + off128_w(r, qq));
          const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e)
            split2_tf32(vmask_w(a[e], R - K, 32 * c + 4 * qq + e, bw), x0[4 * qq + e], x1[4 * qq + e]);
        }
        tmem_st32(tmem + tl + 32 * c, x0);
        tmem_st32(tmem + tl + 128 + 32 * c, x1);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars.vempty);               // staging free for the next item's V
        mbar_arrive_cluster(lead_vready);        // this CTA's quarter of V is in TMEM
      }
    }
  } else {
    // ---------------- epilogue warpgroups (warps 2-5: wg 0, 7-10: wg 1) ----------------
    const int wg = warp >= 7 ? 1 : 0;
    const int q = warp & 3;
    const int r = 32 * q + lane;   // row within this CTA's 128 = TMEM lane
    const uint32_t tl = (uint32_t)(32 * q) << 16;
    int gs = 0, iter = 0;
    bool stop = false;
    for (int64_t item = pair; item < nitems && !stop; item += npairs, ++iter) {
      const UItem it = u_item(item, K, ntiles, ngroups, gsize, nstrips);
      const int y = it.y0 + rowoff;
      const int R = y + r;
      for (int s = it.s0; s < it.s1 && !stop; ++s, ++gs) {
        if ((gs & 1) != wg) continue;
        const int acc = gs % kUAcc;
        if (!wwait(&bars.accf[acc], (gs / kUAcc) & 1, abort, err, 48)) {
          stop = true;
          break;
        }
        tc_fence_after();
        // Two 64-column halves, each in its own C slot (half-strip 2 gs + h2).
        for (int h2 = 0; h2 < 2; ++h2) {
          const int hs = 2 * gs + h2, slot = hs % kUCSlots;
          const int cs = c0 + s * kUTN + 64 * h2;
          unsigned char* cbox = sm + kUOffC + slot * kUCSlot;
          if (!wwait(&bars.cfull[slot], (hs / kUCSlots) & 1, abort, err, 47)) {
            stop = true;
            break;
          }
          float d[2][32];
          tmem_ld32(tmem + tl + kAcc + acc * kUTN + 64 * h2, d[0]);
          tmem_ld32(tmem + tl + kAcc + acc * kUTN + 64 * h2 + 32, d[1]);
          if (h2 == 1) {   // the accumulator is free once its second half is read
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(lead_acce0 + acc * (uint32_t)sizeof(uint64_t));
          }
          // Row R of the half-strip: C - V W2 is written back in place into the slot, then
          // the warp stores its 32 rows to global memory coalesced (lanes 0-15 and 16-31
          // each cover one 256-byte row per instruction).
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int qq = 0; qq < 8; ++qq) {
              float4* cp = reinterpret_cast<float4*>(cbox + h * kUCBox + off128_w(r, qq));
              const float4 cv4 = *cp;
              float cv[4] = {cv4.x, cv4.y, cv4.z, cv4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                if constexpr (IDENT) {
                  const int Cc = cs + 32 * h + 4 * qq + e;
                  if (R < n && Cc < n && (R < kb || Cc < kb)) cv[e] = R == Cc ? 1.f : 0.f;
                }
                cv[e] -= d[h][4 * qq + e];
              }
              *cp = make_float4(cv[0], cv[1], cv[2], cv[3]);
            }
          }
          __syncwarp();
          {
            const int sub = lane >> 4, q4 = lane & 15;   // row parity, float4 column 0..15
            const int h = q4 >> 3, qq = q4 & 7;
#pragma unroll 4
            for (int i = 0; i < 16; ++i) {
              const int rr = 32 * q + 2 * i + sub;       // tile row written by this lane
              const int Rg = y + rr;
              const float4 v = *reinterpret_cast<const float4*>(cbox + h * kUCBox + off128_w(rr, qq));
              if (Rg < n && cs + 4 * q4 < n)
                *reinterpret_cast<float4*>(dst + ((size_t)it.mat * n + Rg) * n + cs + 4 * q4) = v;
            }
          }
          // Release the slot only after this warp's reads of it have completed (their values
          // are consumed by the stores above) and are ordered before the TMA (async proxy)
          // that refills it; releasing right after issuing the loads let a slow warp read
          // the next strip's data.
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.cempty[slot]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();   // neither CTA leaves while the pair's MMAs or signals may touch it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ---- host side ---------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn_w() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D fp32 map: `cols` x `rows` x `depth` with row pitch `pitch` floats; boxes of 32
// columns x box_rows rows.
bool wmap(CUtensorMap* map, const float* base, uint64_t cols, uint64_t pitch, uint64_t rows, uint64_t depth,
          int box_rows, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn_w();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {cols, rows, depth};
  cuuint64_t strides[2] = {pitch * 4, pitch * rows * 4};
  cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int nblocks(int n) { return (n + kWB - 1) / kWB; }
int ycols(int n) { return nblocks(n) * kWB; }

// Row chunks of the Y reduction: enough CTAs (one per SM) for about two waves, but
// never chunks under 512 rows.
struct YPlan {
  int nstrips, nsplit, chunk;
};

YPlan y_plan(int64_t batch, int n, int K, int cend) {
  YPlan p;
  const int m = n - K;
  p.nstrips = (cend - K + kWB - 1) / kWB;
  const int64_t units = (int64_t)p.nstrips * (batch > 0 ? batch : 1);
  const int64_t target = 2 * (int64_t)sm_count();
  int ns = (int)((target + units - 1) / units);
  const int max_split = (m + 511) / 512;
  ns = ns < 1 ? 1 : (ns > max_split ? max_split : ns);
  if (ns > 8) ns = 8;
  int chunk = (m + ns - 1) / ns;
  chunk = (chunk + 31) / 32 * 32;
  p.chunk = chunk;
  p.nsplit = (m + chunk - 1) / chunk;
  return p;
}

struct WideWs {
  float *t128, *vp0, *vp1, *w0, *w1, *ypart;
};

size_t al(size_t x) { return (x + 63) & ~size_t(63); }   // floats: keep 256-byte alignment

WideWs carve(float* ws, int64_t batch, int n) {
  WideWs w;
  const size_t mat = (size_t)batch * n * kWB;
  w.t128 = ws;
  w.vp0 = w.t128 + al((size_t)nblocks(n) * batch * kWB * kWB);
  w.vp1 = w.vp0 + al(mat);
  w.w0 = w.vp1 + al(mat);
  w.w1 = w.w0 + al(mat);
  w.ypart = w.w1 + al(mat);
  return w;
}

bool set_smem_attrs() {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return true;
  if (cudaFuncSetAttribute(ygemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemY) != cudaSuccess ||
      cudaFuncSetAttribute(ygemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemY) != cudaSuccess ||
      cudaFuncSetAttribute(wupdate_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemU) !=
          cudaSuccess ||
      cudaFuncSetAttribute(wupdate_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemU) !=
          cudaSuccess ||
      cudaFuncSetAttribute(tbuild_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemT) != cudaSuccess ||
      cudaFuncSetAttribute(w2tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemW2T) != cudaSuccess ||
      cudaFuncSetAttribute(w2tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemW2T) != cudaSuccess)
    return false;
  done.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

cudaError_t run_vsplit(const float* H, const WideWs& w, int64_t batch, int n, int K, int bw, cudaStream_t s) {
  const int64_t units = batch * (int64_t)(n - K) * 32;
  int64_t blocks = (units + 255) / 256;
  const int64_t cap = 64 * (int64_t)sm_count();   // about one unit per thread: every load in flight at once
  if (blocks > cap) blocks = cap;
  LaunchTimer timer("vsplit_kernel", s, (double)batch * (n - K) * (4.0 * bw + 8.0 * kWB));
  vsplit_kernel<<<(unsigned)blocks, 256, 0, s>>>(H, w.vp0, w.vp1, n, K, bw, units);
  return cudaGetLastError();
}

// Y over columns [K, cend) of `src` (MODE 0: strip 0 from H, masked to V).
cudaError_t run_ygemm(int mode, const float* src, const float* H, const WideWs& w, int64_t batch, int n, int K,
                      int bw, int cend, YPlan& plan, cudaStream_t s) {
  plan = y_plan(batch, n, K, cend);
  int* err = device_error_flag();
  if (err == nullptr) return cudaErrorInvalidValue;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
  CUtensorMap mc, mh, mv0, mv1;
  if (!wmap(&mc, src, n, n, n, batch, 32, sw) || !wmap(&mh, H, n, n, n, batch, 32, sw) ||
      !wmap(&mv0, w.vp0, kWB, kWB, n, batch, 32, sw) || !wmap(&mv1, w.vp1, kWB, kWB, n, batch, 32, sw))
    return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((int64_t)plan.nstrips * batch * plan.nsplit);
  const double m = n - K, nc = cend - K;
  // Algorithmic bytes: C once, the V pieces once, the Y partials written (the V pieces
  // are read again for every strip, but from L2).
  LaunchTimer timer("ygemm_kernel", s,
                    (double)batch * (4.0 * m * nc + 8.0 * m * kWB + 4.0 * plan.nsplit * nc * kWB),
                    (double)batch * 2.0 * m * nc * kWB);
  if (mode == 0)
    ygemm_kernel<0><<<grid, kYThreads, kSmemY, s>>>(mc, mh, mv0, mv1, w.ypart, batch, n, K, bw, plan.nstrips,
                                                      plan.chunk, plan.nsplit, ycols(n), err);
  else
    ygemm_kernel<1><<<grid, kYThreads, kSmemY, s>>>(mc, mh, mv0, mv1, w.ypart, batch, n, K, bw, plan.nstrips,
                                                      plan.chunk, plan.nsplit, ycols(n), err);
  return cudaGetLastError();
}

cudaError_t run_tbuild(const WideWs& w, const YPlan& plan, const float* t32blk, int np, int blk, int64_t batch,
                       int n, cudaStream_t s) {
  LaunchTimer timer("tbuild_kernel", s, (double)batch * (plan.nsplit + 1) * kWB * kWB * 4.0);
  tbuild_kernel<<<(unsigned)(batch * 4), 256, kSmemT, s>>>(w.ypart, plan.nsplit, batch, ycols(n), t32blk, np,
                                                    w.t128 + (size_t)blk * batch * kWB * kWB);
  return cudaGetLastError();
}

cudaError_t run_w2build(const WideWs& w, const YPlan& plan, int blk, int64_t batch, int n, int K, int cfirst,
                        int trans_t, cudaStream_t s) {
  const int ngroups = (n - cfirst + 127) / 128;
  if (ngroups <= 0) return cudaSuccess;
  int* err = device_error_flag();
  if (err == nullptr) return cudaErrorInvalidValue;
  CUtensorMap mt, my, mw0, mw1;
  const int nblk = nblocks(n);
  // T factors [block][batch][128][128]: rows of 128 a (geqrf boxes 32 x 32 with 32-byte
  // atoms; orgqr boxes 32 x 128); Y partials [split][batch][ncolsY][128]; W2 pieces.
  const bool ok_t = trans_t ? wmap(&mt, w.t128, kWB, kWB, kWB, (uint64_t)nblk * batch, 32,
                                   CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B)
                            : wmap(&mt, w.t128, kWB, kWB, kWB, (uint64_t)nblk * batch, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!ok_t || !wmap(&my, w.ypart, kWB, kWB, ycols(n), (uint64_t)plan.nsplit * batch, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !wmap(&mw0, w.w0, kWB, kWB, n, batch, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !wmap(&mw1, w.w1, kWB, kWB, n, batch, 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const double nc = n - cfirst;
  LaunchTimer timer("w2tc_kernel", s, (double)batch * nc * kWB * 4.0 * (plan.nsplit + 2) + batch * ngroups * 65536.0,
                    (double)batch * nc * kWB * kWB);
  if (trans_t)
    w2tc_kernel<1><<<(unsigned)(batch * ngroups), 128, kSmemW2T, s>>>(mt, my, mw0, mw1, batch, n, K, cfirst, ngroups,
                                                                       plan.nsplit, blk, err);
  else
    w2tc_kernel<0><<<(unsigned)(batch * ngroups), 128, kSmemW2T, s>>>(mt, my, mw0, mw1, batch, n, K, cfirst, ngroups,
                                                                       plan.nsplit, blk, err);
  return cudaGetLastError();
}

cudaError_t run_wupdate(bool ident, const float* H, const float* src, float* dst, const WideWs& w, int64_t batch,
                        int n, int K, int bw, int c0, cudaStream_t s) {
  int* err = device_error_flag();
  if (err == nullptr) return cudaErrorInvalidValue;
  CUtensorMap mv, msrc, mw0, mw1;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!wmap(&mv, H, n, n, n, batch, 128, sw) || !wmap(&msrc, src, n, n, n, batch, 128, sw) ||
      !wmap(&mw0, w.w0, kWB, kWB, n, batch, kUHalf, sw) || !wmap(&mw1, w.w1, kWB, kWB, n, batch, kUHalf, sw))
    return cudaErrorInvalidValue;
  const int m = n - K;
  const int nstrips = (n - c0 + kUTN - 1) / kUTN;
  const int ntiles = (m + 255) / 256;   // 256-row tiles, one per CTA pair
  const int64_t tiles = batch * ntiles;
  const int pairs = sm_count() / 2;
  // At least four items per pair so the last round is short; strip groups (each
  // reloading V) only when there are too few row tiles for that.
  int ngroups = (int)((4 * (int64_t)pairs + tiles - 1) / tiles);
  ngroups = ngroups < 1 ? 1 : (ngroups > nstrips ? nstrips : ngroups);
  const int gsize = (nstrips + ngroups - 1) / ngroups;
  ngroups = (nstrips + gsize - 1) / gsize;
  const int64_t items = tiles * ngroups;
  const unsigned grid = 2u * (unsigned)(items < pairs ? items : pairs);
  const double mm = m, nc = n - c0;
  LaunchTimer timer("wupdate_kernel", s, (double)batch * (8.0 * mm * nc + 4.0 * mm * kWB * ngroups),
                    (double)batch * 2.0 * mm * nc * kWB);
  if (ident)
    wupdate_kernel<true><<<grid, kUThreads, kSmemU, s>>>(mv, msrc, dst, mw0, mw1, batch, n, K, bw, c0, nstrips,
                                                         ntiles, ngroups, gsize, err);
  else
    wupdate_kernel<false><<<grid, kUThreads, kSmemU, s>>>(mv, msrc, dst, mw0, mw1, batch, n, K, bw, c0, nstrips,
                                                          ntiles, ngroups, gsize, err);
  return cudaGetLastError();
}

}  // namespace

bool wide_supported(int n) { return n % 4 == 0 && n >= kWideMinN && encode_fn_w() != nullptr; }

size_t wide_ws_floats(int64_t batch, int n) {
  // Y partials: the most row chunks any block's product uses, over both the full-width
  // product (columns [K, n)) and the Gram-only one (the block's own 128 columns, which
  // has fewer strips and so may split its rows into more chunks).
  size_t ymax = 0;
  for (int K = 0; K < n; K += kWB) {
    const int bw = n - K < kWB ? n - K : kWB;
    for (const int cend : {n, K + bw}) {
      const YPlan p = y_plan(batch, n, K, cend);
      const size_t y = (size_t)p.nsplit * batch * ycols(n) * kWB;
      if (y > ymax) ymax = y;
    }
  }
  const size_t mat = (size_t)batch * n * kWB;
  return al((size_t)nblocks(n) * batch * kWB * kWB) + 4 * al(mat) + al(ymax);
}

int wide_block_launches(int64_t batch, int n, int K, bool update, bool tfactor, bool orgqr) {
  (void)batch;
  (void)K;
  if (orgqr) return 4;   // vsplit, ygemm, w2tc, wupdate
  int c = 0;
  if (update || tfactor) c += 2;   // vsplit, ygemm
  if (tfactor) c += 1;             // tbuild
  if (update) c += 2;              // w2tc, wupdate
  return c;
}

cudaError_t wide_geqrf_block(const float* src, float* H, const float* t32blk, float* ws, int64_t batch, int n,
                             int K, int bw, bool want_t, bool update, cudaStream_t s) {
  if (!set_smem_attrs()) return cudaErrorInvalidValue;
  update = update && K + bw < n;
  if (!update && !want_t) return cudaSuccess;
  const WideWs w = carve(ws, batch, n);
  const int blk = K / kWB;
  cudaError_t e = run_vsplit(H, w, batch, n, K, bw, s);
  if (e != cudaSuccess) return e;
  YPlan plan;
  e = run_ygemm(0, update ? src : H, H, w, batch, n, K, bw, update ? n : K + bw, plan, s);
  if (e != cudaSuccess) return e;
  if (want_t || update) {
    // T is needed by the update as well (W2 = T^T Y).
    e = run_tbuild(w, plan, t32blk, (bw + kNB - 1) / kNB, blk, batch, n, s);
    if (e != cudaSuccess) return e;
  }
  if (!update) return cudaSuccess;
  e = run_w2build(w, plan, blk, batch, n, K, K + bw, 1, s);
  if (e != cudaSuccess) return e;
  return run_wupdate(false, H, src, H, w, batch, n, K, bw, K + bw, s);
}

cudaError_t wide_orgqr_block(const float* H, float* Q, float* ws, int64_t batch, int n, int K, int bw,
                             cudaStream_t s) {
  if (!set_smem_attrs()) return cudaErrorInvalidValue;
  const WideWs w = carve(ws, batch, n);
  const int blk = K / kWB;
  cudaError_t e = run_vsplit(H, w, batch, n, K, bw, s);
  if (e != cudaSuccess) return e;
  YPlan plan;
  e = run_ygemm(1, Q, H, w, batch, n, K, bw, n, plan, s);
  if (e != cudaSuccess) return e;
  e = run_w2build(w, plan, blk, batch, n, K, K, 0, s);
  if (e != cudaSuccess) return e;
  return run_wupdate(true, H, Q, Q, w, batch, n, K, bw, K, s);
}

}  // namespace qrb
