// Block reflector application on the 5th-generation tensor cores:
//     C[k:, c0:] -= V op(T) (V^T C[k:, c0:])
// for the trailing update of geqrf (op = T^T) and the backward blocks of orgqr
// (op = T).  Replaces the reference's cuBLAS bmm / solve_triangular / baddbmm chain
// (_wy_trailing_trisolve, submission.py:434-460) and its cublasLt BF16x9 trailing
// GEMMs (submission.py:875-884).
//
// Near-fp32 accuracy from the tf32 tensor pipe (3xTF32): every operand is split in
// shared memory into two tf32 pieces (x = x0 + x1, exact to 2^-22 |x|) and
// tcgen05.mma kind::tf32 accumulates x1y0 + x0y1 + x0y0, smallest first.  The QR
// residuals measured against the fp32 checker are within 5% of those of a three-piece,
// six-product split (which costs 15-20% more time at n >= 256).  Operands travel
// through HBM as plain fp32 (V straight from H, masked to the unit lower trapezoid
// where it is split).  Two or three launches per panel:
//   wpart_kernel   W^T (64 x 32) = C^T V for a 64-column strip over one row chunk:
//                  TMA streams 32-row stages of C and V (MN-major operands, which
//                  for tf32 take the 128-byte swizzle with 32-byte atoms), threads
//                  split both, one thread issues M=64 N=32 K=8 MMAs into one TMEM
//                  accumulator per stage, stage partials are summed in registers;
//                  with a single row chunk it also forms W2 = op(T) W itself;
//   w2_kernel      only with several row chunks: W = sum of the chunk partials (fixed
//                  order), W2 = op(T) W in fp32, in the K-major layout of the next step;
//   update_kernel  C -= V W2 by persistent warp-specialised CTAs: per 128-row
//                  tile, M=128 N=64 K=32 MMAs into double-buffered TMEM, the
//                  epilogue subtracts from the TMA-loaded C tile and TMA-stores it.
// Every mbarrier wait is bounded; a wait that runs out records an error code in
// g_qrb_device_error and stops the CTA: no further TMA, MMA or stores are issued, the
// CTA waits (bounded) for the copies and MMAs it already has in flight, releases its
// tensor memory and exits without writing results.
// Requires n % 4 == 0 (TMA row strides are multiples of 16 bytes) and the workspace
// of tc_ws_floats floats; launch_apply falls back to the SIMT kernel otherwise.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "qrb_internal.cuh"
#include "qrb_sm100.cuh"

__device__ int g_qrb_device_error = 0;

namespace qrb {
namespace {

using namespace sm100;

constexpr int kTN = 64;        // strip width: M of the W^T product, N of the update
constexpr int kR1 = 32;        // rows per W^T stage
constexpr int kR3 = 128;       // rows per update tile (M)
constexpr int kThreads = 128;

// Shared-memory boxes (fp32, rows of 32 floats = 128 bytes).  TMA lands raw fp32 C in
// piece 0 of a W^T stage, which the split pass overwrites.
constexpr int kPieces = 2;
constexpr int kTerms = 3;
constexpr uint32_t kBox1 = kR1 * 128;            // 32 rows x 32 floats
constexpr uint32_t kStage1 = 3 * kPieces * kBox1;   // C pieces (2 boxes each), then V pieces
constexpr uint32_t kOffV1 = 2 * kPieces * kBox1;
constexpr uint32_t kBox3 = kR3 * 128;            // 128 rows x 32 floats

// The three (A piece, B piece) products kept, smallest first.  The tensor core's fp32
// accumulation rounds each add relative to the running sum, so the 2^-11 terms of a
// stage go in before its leading terms; an accumulator then takes four
// full-size roundings (one per K step), and stage partials are summed in fp32 registers,
// which keeps the error at the level of an fp32 SIMT dot product of the same length.
__device__ __constant__ int kTermA[kTerms] = {1, 0, 0};
__device__ __constant__ int kTermB[kTerms] = {0, 1, 0};

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_qrb_device_error, 0, code); }

// Bounded wait of one thread; false (with the code recorded) when it ran out.
__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_wait(bar, parity)) return true;
  record_error(code);
  return false;
}

// Bounded wait inside a warp-specialised CTA (gives up when another role already did).
__device__ __forceinline__ bool wait_role(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  return mbar_wait_abort(bar, parity, abort, &g_qrb_device_error, code);
}

// V[r][j] of the unit lower trapezoidal block (r relative to the panel top).
__device__ __forceinline__ float vmask(float x, int r, int j, int b) {
  if (j >= b) return 0.f;
  return r > j ? x : (r == j ? 1.f : 0.f);
}

// Offset of the float4 (row r, columns 4q..4q+3) in the two swizzles.
__device__ __forceinline__ uint32_t off32b(int r, int q) {
  return r * 128u + (((((uint32_t)q >> 1) ^ (uint32_t)r) & 3u) << 5) + ((uint32_t)(q & 1) << 4);
}
__device__ __forceinline__ uint32_t off128(int r, int q) {
  return r * 128u + ((((uint32_t)q ^ (uint32_t)r) & 7u) << 4);
}

__device__ __forceinline__ void split4_store(unsigned char* p0, uint32_t pstride, uint32_t off, float4 v) {
  float a[4] = {v.x, v.y, v.z, v.w}, x0[4], x1[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) split2_tf32(a[e], x0[e], x1[e]);
  *reinterpret_cast<float4*>(p0 + off) = make_float4(x0[0], x0[1], x0[2], x0[3]);
  *reinterpret_cast<float4*>(p0 + pstride + off) = make_float4(x1[0], x1[1], x1[2], x1[3]);
}

constexpr int kMaxSplit = 8;            // row chunks of the W^T reduction
constexpr uint32_t kWBox = kTN * 128;   // W2 piece box: 64 strip columns x 32 floats

// ---- (A) W^T partial over one row chunk: part[split][mat][strip][64][32] -------------
// Three CTAs per SM: two 24 KB stages.  V arrives raw from H (masked to the unit lower
// trapezoid here) and is split with C.  With a single row chunk (nsplit == 1) the CTA
// holds the whole W^T of its strip and finishes W2 = op(T) W itself (the work of
// w2_kernel, same arithmetic order), so the update needs no second launch.
constexpr uint32_t kSmemA = 2 * kStage1 + 64 + 1024;   // stages, 5 mbarriers + TMEM slot, alignment

template <bool IDENT>
__global__ void __launch_bounds__(kThreads, 3)
wpart_kernel(const __grid_constant__ CUtensorMap map_src32, const __grid_constant__ CUtensorMap map_hv32,
             float* __restrict__ part, const float* __restrict__ Tg, float* __restrict__ w2, int64_t batch,
             int n, int k, int b, int c0, int nstrips, int chunk, int nsplit, int trans_t) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  uint64_t* tma1 = reinterpret_cast<uint64_t*>(sm + 2 * kStage1);
  uint64_t* mma1 = tma1 + 2;
  uint64_t* drain = mma1 + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x % nsplit;
  const int t = blockIdx.x / nsplit;
  const int strip = t % nstrips;
  const int mat = t / nstrips;
  const int cs = c0 + strip * kTN;
  const int r0 = k + split * chunk;
  const int r1 = min(n, r0 + chunk);
  const int nst = (r1 - r0 + kR1 - 1) / kR1;   // chunk % 32 == 0: stages never cross chunks
  const int kb = k + b;
  // T of the panel, fetched early for the direct W2 path: thread holds T[tid / 32 + 4e][tid % 32].
  float treg[8];
  if (nsplit == 1) {
#pragma unroll
    for (int e = 0; e < 8; ++e) treg[e] = __ldg(Tg + (size_t)mat * 32 * 32 + tid + 128 * e);
  }

  if (tid == 0) {
    mbar_init(&tma1[0], 1);
    mbar_init(&tma1[1], 1);
    mbar_init(&mma1[0], 1);
    mbar_init(&mma1[1], 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tensormap(&map_src32);
    prefetch_tensormap(&map_hv32);
  }
  if (warp == 0) tmem_alloc(tslot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // Stage loads armed but not yet waited on by the CTA (for the drain after an abort).
  int armed_hi = -1;
  auto issue_stage = [&](int s) {
    armed_hi = s;
    unsigned char* st = sm + (s & 1) * kStage1;
    const int y = r0 + s * kR1;
    mbar_arrive_expect_tx(&tma1[s & 1], 3 * kBox1);
    tma_load_3d(st, &map_src32, cs, y, mat, &tma1[s & 1]);
    tma_load_3d(st + kBox1, &map_src32, cs + 32, y, mat, &tma1[s & 1]);
    tma_load_3d(st + kOffV1, &map_hv32, k, y, mat, &tma1[s & 1]);
  };
  if (tid == 0) {
    issue_stage(0);
    if (nst > 1) issue_stage(1);
  }
  constexpr uint32_t idesc1 = idesc_tf32(kTN, 32, 1, 1);
  const uint32_t tm_lane = (uint32_t)(32 * warp) << 16;
  float wacc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) wacc[j] = 0.f;
  // Every decision to stop is made CTA-wide (__syncthreads_or), so all threads leave the
  // stage loop at the same iteration and no barrier is left waiting.
  auto gather_stage = [&](int s) -> bool {
    if (!wait_or_flag(&mma1[s & 1], (s >> 1) & 1, 13)) return false;
    tc_fence_after();
    float p[32];
    tmem_ld32(tmem + tm_lane + (s & 1) * 32, p);
#pragma unroll
    for (int j = 0; j < 32; ++j) wacc[j] += p[j];
    tc_fence_before();
    return true;
  };
  bool aborted = false, issued = false, issue_fail = false;
  for (int s = 0; s < nst; ++s) {
    const int buf = s & 1;
    const uint32_t par = (s >> 1) & 1;
    unsigned char* st = sm + buf * kStage1;
    const bool landed = wait_or_flag(&tma1[buf], par, 11);
    if (__syncthreads_or(!landed || issue_fail)) {
      aborted = true;
      break;
    }
    for (int u = tid; u < 2 * kR1 * 8; u += kThreads) {
      const int box = u >> 8, r = (u >> 3) & 31, q = u & 7;
      const uint32_t off = off32b(r, q);
      unsigned char* p0 = st + box * kBox1;
      float4 v = *reinterpret_cast<float4*>(p0 + off);
      if constexpr (IDENT) {
        const int R = r0 + s * kR1 + r;
        float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int Cc = cs + 32 * box + 4 * q + e;
          if (R < n && Cc < n && (R < kb || Cc < kb)) a[e] = R == Cc ? 1.f : 0.f;
        }
        v = make_float4(a[0], a[1], a[2], a[3]);
      }
      split4_store(p0, 2 * kBox1, off, v);
    }
    // V: rows of the stage relative to the panel top; the first 32 hold the unit
    // upper part of the reflectors (1 on the diagonal, 0 above), the rest is H as is.
    for (int u = tid; u < kR1 * 8; u += kThreads) {
      const int r = u >> 3, q = u & 7;
      const uint32_t off = off32b(r, q);
      unsigned char* p0 = st + kOffV1;
      float4 v = *reinterpret_cast<float4*>(p0 + off);
      const int rr = r0 + s * kR1 + r - k;
      if (rr < 32) {
        float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) a[e] = vmask(a[e], rr, 4 * q + e, b);
        v = make_float4(a[0], a[1], a[2], a[3]);
      }
      split4_store(p0, kBox1, off, v);
    }
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t base = smem_u32(st);
      const uint32_t d = tmem + buf * 32;
#pragma unroll
      for (int tt = 0; tt < kTerms; ++tt) {
#pragma unroll
        for (int kk = 0; kk < kR1 / 8; ++kk) {
          const uint64_t ad = sdesc_sw128_32b(base + 2 * kTermA[tt] * kBox1 + kk * 1024, kBox1, 512);
          const uint64_t bd = sdesc_sw128_32b(base + kOffV1 + kTermB[tt] * kBox1 + kk * 1024, kBox1, 512);
          mma_tf32(d, ad, bd, idesc1, (tt > 0 || kk > 0) ? 1u : 0u);
        }
      }
      mma_commit(&mma1[buf]);
      issued = true;
    }
    const bool gathered = s > 0 ? gather_stage(s - 1) : true;
    if (__syncthreads_or(!gathered)) {
      aborted = true;
      break;
    }
    if (tid == 0 && s + 2 < nst) {
      if (wait_or_flag(&mma1[buf], par, 12)) issue_stage(s + 2);
      else issue_fail = true;   // seen by every thread at the next stage's decision
    }
  }
  if (!aborted) aborted = __syncthreads_or(!gather_stage(nst - 1));
  if (aborted) {
    // Let this CTA's own copies and MMAs finish before its shared and tensor memory go.
    if (tid == 0) {
      for (int s = armed_hi - 1 < 0 ? 0 : armed_hi - 1; s <= armed_hi; ++s)
        mbar_wait(&tma1[s & 1], (s >> 1) & 1, 1u << 22);
      if (issued) {
        mma_commit(drain);
        mbar_wait(drain, 0, 1u << 22);
      }
    }
  } else if (nsplit == 1) {
    // M = 64 accumulator: lanes 0-15 of warp w hold W^T rows 16w + lane.
    // Every MMA has completed (gathered), so the stage buffers are free.
    __syncthreads();
    float(*Ws)[33] = reinterpret_cast<float(*)[33]>(sm);                   // Ws[i][j] = W^T[i][j]
    float(*Tt)[36] = reinterpret_cast<float(*)[36]>(sm + kTN * 33 * 4);   // Tt[j][a] = op(T)[a][j]
    if (lane < 16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) Ws[16 * warp + lane][j] = wacc[j];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int r = (tid >> 5) + 4 * e, c = tid & 31;   // treg[e] = T[r][c]
      if (trans_t) Tt[r][c] = treg[e];
      else Tt[c][r] = treg[e];
    }
    __syncthreads();
    // Thread: strip columns i0, i0 + 32 and reflectors a0..a0+7.
    const int i0 = tid >> 2, a0 = (tid & 3) * 8;
    float acc[2][8] = {};
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
      const float4 ta = *reinterpret_cast<const float4*>(&Tt[j][a0]);
      const float4 tb = *reinterpret_cast<const float4*>(&Tt[j][a0 + 4]);
      const float tv[8] = {ta.x, ta.y, ta.z, ta.w, tb.x, tb.y, tb.z, tb.w};
      const float wv[2] = {Ws[i0][j], Ws[i0 + 32][j]};
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[h][e] = fmaf(tv[e], wv[h], acc[h][e]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = i0 + 32 * h;
      if (cs + i < n) {
        float4* dst = reinterpret_cast<float4*>(w2 + ((size_t)mat * n + cs + i) * 32 + a0);
        dst[0] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
        dst[1] = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
      }
    }
  } else if (lane < 16) {
    const int i = 16 * warp + lane;
    float4* dst = reinterpret_cast<float4*>(
        part + ((((size_t)split * batch + mat) * nstrips + strip) * kTN + i) * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) dst[q] = make_float4(wacc[4 * q], wacc[4 * q + 1], wacc[4 * q + 2], wacc[4 * q + 3]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// ---- (A2) W2 = op(T) W, summed over the row chunks in a fixed order ------------------
// w2[mat][col][a] (col = absolute column, a = reflector), fp32: the K-major B operand of
// update_kernel, which splits it into tf32 pieces in shared memory.
__global__ void __launch_bounds__(256)
w2_kernel(const float* __restrict__ part, const float* __restrict__ Tg, float* __restrict__ w2, int64_t batch,
          int n, int c0, int nstrips, int nsplit, int trans_t) {
  __shared__ __align__(16) float Tt[32][36];   // Tt[j][a] = op(T)[a][j]
  __shared__ float Ws[kTN][33];                // Ws[i][j] = W^T[i][j]
  const int strip = blockIdx.x % nstrips;
  const int mat = blockIdx.x / nstrips;
  const int cs = c0 + strip * kTN;
  const float* T = Tg + (size_t)mat * 32 * 32;
  for (int idx = threadIdx.x; idx < 32 * 32; idx += blockDim.x) {
    const int r = idx >> 5, c = idx & 31;
    const float t = __ldg(T + idx);   // T[r][c]
    if (trans_t) Tt[r][c] = t;        // op(T) = T^T: op(T)[c][r] = T[r][c] -> Tt[r][c]
    else Tt[c][r] = t;                // op(T) = T:   op(T)[r][c] = T[r][c] -> Tt[c][r]
  }
  // Each thread sums 8 elements over the chunks (in chunk order); the 8 loads of a chunk
  // are independent, so they are in flight together.
  constexpr int kPer = kTN * 32 / 256;
  static_assert(kPer == 8, "w2_kernel: 256 threads, 8 elements each");
  float w[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) w[e] = 0.f;
#pragma unroll 2
  for (int sp = 0; sp < nsplit; ++sp) {
    const float* src = part + (((size_t)sp * batch + mat) * nstrips + strip) * kTN * 32;
    float v[kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) v[e] = __ldg(src + threadIdx.x + 256 * e);
#pragma unroll
    for (int e = 0; e < kPer; ++e) w[e] += v[e];
  }
#pragma unroll
  for (int e = 0; e < kPer; ++e) {
    const int idx = threadIdx.x + 256 * e;
    Ws[idx >> 5][idx & 31] = w[e];
  }
  __syncthreads();
  // Thread: strip columns i0, i0 + 32 and reflectors a0..a0+3 (8 outputs, register tile).
  const int i0 = threadIdx.x >> 3, a0 = (threadIdx.x & 7) * 4;
  float acc[2][4] = {};
#pragma unroll 8
  for (int j = 0; j < 32; ++j) {
    const float4 t = *reinterpret_cast<const float4*>(&Tt[j][a0]);
    const float w0 = Ws[i0][j], w1 = Ws[i0 + 32][j];
    acc[0][0] = fmaf(t.x, w0, acc[0][0]);
    acc[0][1] = fmaf(t.y, w0, acc[0][1]);
    acc[0][2] = fmaf(t.z, w0, acc[0][2]);
    acc[0][3] = fmaf(t.w, w0, acc[0][3]);
    acc[1][0] = fmaf(t.x, w1, acc[1][0]);
    acc[1][1] = fmaf(t.y, w1, acc[1][1]);
    acc[1][2] = fmaf(t.z, w1, acc[1][2]);
    acc[1][3] = fmaf(t.w, w1, acc[1][3]);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = i0 + 32 * h;
    if (cs + i < n)
      *reinterpret_cast<float4*>(w2 + ((size_t)mat * n + cs + i) * 32 + a0) =
          make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  }
}

// ---- (B) C -= V W2: persistent CTAs over (matrix, 128-row tile, strip group) items ---
// Warp roles: 0 = TMA producer, 1 = MMA issuer (and TMEM owner), 2-5 = epilogue (warp w
// reads TMEM lanes 32*(w%4).., i.e. tile rows 32*(w%4)+lane), 6-9 = converters, which
// split the raw fp32 V tile (from H, masked to the unit lower trapezoid) and each
// strip's raw W2 into tf32 pieces in place.  An item's V pieces stay in shared memory
// for its strips; each strip's W2 and C tile go through a ring of kSlotsB slots; two TMEM accumulators let the MMAs of one strip run under the
// epilogue of the previous one.  Ring positions and parities run on a per-CTA strip
// counter across items, so the pipeline does not drain between items (only the V
// reload waits for the previous item's last MMA).
constexpr int kSlotsB = 4;   // 32 KB of V pieces + 4 x 48 KB slots: 225 KB of shared memory
constexpr int kThreadsB = 320;
constexpr uint32_t kOffBV = 0;                              // V pieces: 2 x 16 KB
constexpr uint32_t kSlotW = 0;                              // in a slot: W2 pieces 2 x 8 KB
constexpr uint32_t kSlotC = kPieces * kWBox;                // then C: 2 boxes x 16 KB
constexpr uint32_t kSlotBytes = kSlotC + 2 * kBox3;         // 48 KB
constexpr uint32_t kOffBSlots = kPieces * kBox3;            // 32 KB
constexpr uint32_t kOffBBar = kOffBSlots + kSlotsB * kSlotBytes;
constexpr uint32_t kSmemB = kOffBBar + 256 + 1024;

struct BarsB {
  uint64_t full[kSlotsB], empty[kSlotsB], w2ready[kSlotsB], cdone[kSlotsB], vfull, vready, vempty, accf[2], acce[2],
      drain;
  uint32_t tmem;
  int abort;
};

struct ItemB {
  int mat, y0, s0, s1;   // matrix, first tile row, strip range [s0, s1)
};

__device__ __forceinline__ ItemB item_b(int64_t item, int k, int ntiles, int ngroups, int gsize, int nstrips) {
  ItemB it;
  const int g = (int)(item % ngroups);
  const int64_t t = item / ngroups;
  it.y0 = k + (int)(t % ntiles) * kR3;
  it.mat = (int)(t / ntiles);
  it.s0 = g * gsize;
  it.s1 = min(nstrips, it.s0 + gsize);
  return it;
}

template <bool IDENT>
__global__ void __launch_bounds__(kThreadsB, 1)
update_kernel(const __grid_constant__ CUtensorMap map_src128, const __grid_constant__ CUtensorMap map_h128,
              const __grid_constant__ CUtensorMap map_hv128, const __grid_constant__ CUtensorMap map_w,
              int64_t batch, int n, int k, int b, int c0, int c1, int nstrips, int ntiles, int ngroups, int gsize,
              int store_to_h) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  BarsB& bars = *reinterpret_cast<BarsB*>(sm + kOffBBar);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kb = k + b;
  const int64_t nitems = batch * ntiles * ngroups;

  if (tid == 0) {
    for (int i = 0; i < kSlotsB; ++i) {
      mbar_init(&bars.full[i], 1);
      mbar_init(&bars.empty[i], 1);
      mbar_init(&bars.w2ready[i], 4);
      mbar_init(&bars.cdone[i], 4);
    }
    mbar_init(&bars.drain, 1);
    bars.abort = 0;
    mbar_init(&bars.vfull, 1);
    mbar_init(&bars.vready, 4);
    mbar_init(&bars.vempty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.accf[i], 1);
      mbar_init(&bars.acce[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bars.tmem, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;
  volatile int* abort = &bars.abort;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tensormap(&map_src128);
      prefetch_tensormap(&map_w);
      prefetch_tensormap(&map_hv128);
      int gs = 0, iter = 0, v_last = -1;
      int last_use[kSlotsB] = {-1, -1, -1, -1};
      bool stop = false;
      for (int64_t item = blockIdx.x; item < nitems && !stop; item += gridDim.x, ++iter) {
        const ItemB it = item_b(item, k, ntiles, ngroups, gsize, nstrips);
        // last MMA of the previous item
        if (iter > 0 && !wait_role(&bars.vempty, (iter - 1) & 1, abort, 20)) break;
        mbar_arrive_expect_tx(&bars.vfull, kBox3);
        tma_load_3d(sm + kOffBV, &map_hv128, k, it.y0, it.mat, &bars.vfull);
        v_last = iter;
        for (int s = it.s0; s < it.s1; ++s, ++gs) {
          const int slot = gs % kSlotsB, use = gs / kSlotsB;
          if (use > 0 && !wait_role(&bars.empty[slot], (use - 1) & 1, abort, 21)) {
            stop = true;
            break;
          }
          unsigned char* sl = sm + kOffBSlots + slot * kSlotBytes;
          const int cs = c0 + s * kTN;
          mbar_arrive_expect_tx(&bars.full[slot], kWBox + 2 * kBox3);
          tma_load_3d(sl + kSlotW, &map_w, 0, cs, it.mat, &bars.full[slot]);
          tma_load_3d(sl + kSlotC, &map_src128, cs, it.y0, it.mat, &bars.full[slot]);
          tma_load_3d(sl + kSlotC + kBox3, &map_src128, cs + 32, it.y0, it.mat, &bars.full[slot]);
          last_use[slot] = use;
        }
      }
      if (*abort) {   // let this CTA's loads land before its shared memory goes away
        if (v_last >= 0) mbar_wait(&bars.vfull, v_last & 1, 1u << 22);
        for (int sl = 0; sl < kSlotsB; ++sl)
          if (last_use[sl] >= 0) mbar_wait(&bars.full[sl], last_use[sl] & 1, 1u << 22);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc3 = idesc_tf32(kR3, kTN, 0, 0);
      const uint32_t vb = smem_u32(sm + kOffBV);
      int gs = 0, iter = 0;
      bool issued = false, stop = false;
      for (int64_t item = blockIdx.x; item < nitems && !stop; item += gridDim.x, ++iter) {
        const ItemB it = item_b(item, k, ntiles, ngroups, gsize, nstrips);
        if (!wait_role(&bars.vready, iter & 1, abort, 22)) break;
        for (int s = it.s0; s < it.s1; ++s, ++gs) {
          const int slot = gs % kSlotsB, acc = gs & 1;
          if (!wait_role(&bars.w2ready[slot], (gs / kSlotsB) & 1, abort, 23) ||
              (gs >= 2 && !wait_role(&bars.acce[acc], ((gs >> 1) - 1) & 1, abort, 24))) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t wb = smem_u32(sm + kOffBSlots + slot * kSlotBytes + kSlotW);
          const uint32_t d = tmem + acc * kTN;
#pragma unroll
          for (int t3 = 0; t3 < kTerms; ++t3) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = sdesc_sw128(vb + kTermA[t3] * kBox3 + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(wb + kTermB[t3] * kWBox + kk * 32, 16, 1024);
              mma_tf32(d, ad, bd, idesc3, (t3 > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(&bars.accf[acc]);
          issued = true;
        }
        if (!stop) mma_commit(&bars.vempty);   // V of this item no longer read once these complete
      }
      if (*abort && issued) {   // tensor memory must not be released under running MMAs
        mma_commit(&bars.drain);
        mbar_wait(&bars.drain, 0, 1u << 22);
      }
    }
  } else if (warp >= 6) {
    // ---------------- converters (warps 6-9) ----------------
    const int ct = tid - 192;   // 0..127
    int gs = 0, iter = 0;
    bool stop = false;
    for (int64_t item = blockIdx.x; item < nitems && !stop; item += gridDim.x, ++iter) {
      const ItemB it = item_b(item, k, ntiles, ngroups, gsize, nstrips);
      if (!wait_role(&bars.vfull, iter & 1, abort, 27)) break;
      // V tile: 128 rows x 8 float4; rows relative to the panel top below 32 are masked.
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int u = ct + 128 * i;
        const int r = u >> 3, q = u & 7;
        const uint32_t off = off128(r, q);
        unsigned char* p0 = sm + kOffBV;
        float4 v = *reinterpret_cast<float4*>(p0 + off);
        const int rr = it.y0 - k + r;
        if (rr < 32) {
          float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) a[e] = vmask(a[e], rr, 4 * q + e, b);
          v = make_float4(a[0], a[1], a[2], a[3]);
        }
        split4_store(p0, kBox3, off, v);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.vready);
      for (int s = it.s0; s < it.s1; ++s, ++gs) {
        const int slot = gs % kSlotsB;
        if (!wait_role(&bars.full[slot], (gs / kSlotsB) & 1, abort, 28)) {
          stop = true;
          break;
        }
        unsigned char* p0 = sm + kOffBSlots + slot * kSlotBytes + kSlotW;
#pragma unroll
        for (int i = 0; i < 4; ++i) {   // W2: 64 rows x 8 float4
          const int u = ct + 128 * i;
          const uint32_t off = off128(u >> 3, u & 7);
          split4_store(p0, kWBox, off, *reinterpret_cast<float4*>(p0 + off));
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.w2ready[slot]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2-5) ----------------
    const int q = warp & 3;
    const int r = 32 * q + lane;   // tile row
    const CUtensorMap* map_store = store_to_h ? &map_h128 : &map_src128;
    const bool leader = (warp == 2 && lane == 0);
    int gs = 0;
    bool stop = false;
    for (int64_t item = blockIdx.x; item < nitems && !stop; item += gridDim.x) {
      const ItemB it = item_b(item, k, ntiles, ngroups, gsize, nstrips);
      const int R = it.y0 + r;
      for (int s = it.s0; s < it.s1; ++s, ++gs) {
        const int slot = gs % kSlotsB, acc = gs & 1;
        const int cs = c0 + s * kTN;
        unsigned char* cbox = sm + kOffBSlots + slot * kSlotBytes + kSlotC;
        if (!wait_role(&bars.full[slot], (gs / kSlotsB) & 1, abort, 25) ||
            !wait_role(&bars.accf[acc], (gs >> 1) & 1, abort, 26)) {
          stop = true;
          break;
        }
        tc_fence_after();
        float d[2][32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + acc * kTN, d[0]);
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + acc * kTN + 32, d[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.acce[acc]);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          unsigned char* box = cbox + half * kBox3;
#pragma unroll
          for (int qq = 0; qq < 8; ++qq) {
            const uint32_t off = off128(r, qq);
            float4 c = *reinterpret_cast<float4*>(box + off);
            float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if constexpr (IDENT) {
                const int Cc = cs + 32 * half + 4 * qq + e;
                if (R < n && Cc < n && (R < kb || Cc < kb)) cv[e] = R == Cc ? 1.f : 0.f;
              }
              cv[e] -= d[half][4 * qq + e];
            }
            *reinterpret_cast<float4*>(box + off) = make_float4(cv[0], cv[1], cv[2], cv[3]);
          }
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.cdone[slot]);
        if (leader) {
          // every epilogue warp has written its rows of the tile
          if (!wait_role(&bars.cdone[slot], (gs / kSlotsB) & 1, abort, 29)) {
            stop = true;
            break;
          }
          tma_store_3d(map_store, cbox, cs, it.y0, it.mat);
          if (cs + 32 < c1) tma_store_3d(map_store, cbox + kBox3, cs + 32, it.y0, it.mat);
          tma_store_commit();
          // The store of the previous strip has finished reading its slot: hand it back.
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          if (gs > 0) mbar_arrive(&bars.empty[(gs - 1) % kSlotsB]);
        }
      }
    }
    if (leader) tma_store_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ---- host: tensor maps -------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 3-D fp32 map {cols, rows, depth} with row pitch `pitch` floats (>= cols), 32-column boxes.
bool make_map(CUtensorMap* map, const float* base, uint64_t cols, uint64_t pitch, uint64_t rows, uint64_t depth,
              int box_rows, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
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

}  // namespace

bool apply_tc_supported(int n) { return n % 4 == 0 && n >= 64 && encode_fn() != nullptr; }

// Tensor-core workspace: W2 ([batch][n][32] fp32), then the W^T partials
// ([split][batch][strip][64][32]).
size_t tc_ws_floats(int64_t batch, int n) {
  return (size_t)batch * n * 32 + (size_t)kMaxSplit * batch * ((n + kTN - 1) / kTN) * kTN * 32;
}

namespace {

// Row chunks of the W^T reduction: up to ~6 waves of CTAs at 4 per SM, but never chunks
// under 512 rows (short chunks cost more in partial traffic and in the w2 sum than they
// gain in balance; measured on b512_n256, b256_n512, b32_n2048).
struct SplitPlan {
  int nsplit, chunk;
};

SplitPlan split_plan(int64_t batch, int n, int k, int c0, int c1) {
  const int m = n - k;
  const int64_t units = (int64_t)((c1 - c0 + kTN - 1) / kTN) * batch;
  // 24 = 4 resident CTAs per SM x 6 waves
  const int64_t target = 24 * (int64_t)sm_count();
  int nsplit = (int)((target + units - 1) / units);
  nsplit = nsplit < 1 ? 1 : (nsplit > kMaxSplit ? kMaxSplit : nsplit);
  // Row chunks of at least 512 rows, or 128 for n >= 2048, where the in-block updates
  // of the wide path (at most 96 columns: few strips) need the row split for parallelism
  // (measured b32_n2048 13.34 -> 13.09 ms, b4 6.80 -> 6.43 ms; smaller n lose with it:
  // b512_n256 1.52 -> 1.73 ms).
  const int min_chunk = n >= 2048 ? 128 : 512;
  const int max_split = (m + min_chunk - 1) / min_chunk;
  if (nsplit > max_split) nsplit = max_split < 1 ? 1 : max_split;
  int chunk = (m + nsplit - 1) / nsplit;
  chunk = (chunk + kR1 - 1) / kR1 * kR1;
  return {(m + chunk - 1) / chunk, chunk};
}

template <bool IDENT>
cudaError_t launch_split(const CUtensorMap& s32, const CUtensorMap& v32, const CUtensorMap& s128,
                         const CUtensorMap& h128, const CUtensorMap& v128, const CUtensorMap& w, const float* T,
                         float* part, float* w2, int64_t batch, int n, int k, int b, int c0, int c1, int trans_t,
                         int store_to_h, cudaStream_t st) {
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(wpart_kernel<IDENT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemA);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(update_kernel<IDENT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemB);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int m = n - k;
  const int nstrips = (c1 - c0 + kTN - 1) / kTN;
  const int ntiles = (m + kR3 - 1) / kR3;
  const int64_t units = (int64_t)nstrips * batch;
  const SplitPlan sp = split_plan(batch, n, k, c0, c1);
  const int nsplit = sp.nsplit, chunk = sp.chunk;
  const double mm = m, nc = c1 - c0;
  {
    LaunchTimer timer("wpart_kernel", st, (double)batch * (4.0 * mm * nc + 4.0 * mm * b * nstrips),
                      (double)batch * 2.0 * mm * nc * b);
    wpart_kernel<IDENT><<<(unsigned)(units * nsplit), kThreads, kSmemA, st>>>(
        s32, v32, part, T, w2, batch, n, k, b, c0, nstrips, chunk, nsplit, trans_t);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  if (nsplit > 1) {
    LaunchTimer timer("w2_kernel", st, (double)units * (nsplit + 1) * kTN * 32 * 4.0);
    w2_kernel<<<(unsigned)units, 256, 0, st>>>(part, T, w2, batch, n, c0, nstrips, nsplit, trans_t);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  // Persistent update: at least four items per SM so the last round is short; strip
  // groups (each reloading V) only when there are too few row tiles for that.
  const int64_t tiles = batch * ntiles;
  int ngroups = (int)((4 * (int64_t)sm_count() + tiles - 1) / tiles);
  ngroups = ngroups < 1 ? 1 : (ngroups > nstrips ? nstrips : ngroups);
  const int gsize = (nstrips + ngroups - 1) / ngroups;
  ngroups = (nstrips + gsize - 1) / gsize;
  const int64_t items = tiles * ngroups;
  const int sms = sm_count();
  const unsigned gridb = (unsigned)(items < sms ? items : sms);
  LaunchTimer timer("update_kernel", st, (double)batch * (8.0 * mm * nc + 4.0 * mm * b),
                    (double)batch * 2.0 * mm * nc * b);
  update_kernel<IDENT><<<gridb, kThreadsB, kSmemB, st>>>(s128, h128, v128, w, batch, n, k, b, c0, c1, nstrips,
                                                         ntiles, ngroups, gsize, store_to_h);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_apply_tc(const float* H, const float* T, const float* src, float* C, int64_t batch,
                            int n, int k, int b, int c0, int c1, int trans_t, int identity_fill, float* tcws,
                            cudaStream_t s) {
  if (batch == 0 || c0 >= c1) return cudaSuccess;
  if (tcws == nullptr) return cudaErrorInvalidValue;
  const int store_to_h = (C == H) ? 1 : 0;
  if (!store_to_h && C != src) return cudaErrorInvalidValue;   // C is either H or the source
  float* w2 = tcws;
  float* part = w2 + (size_t)batch * n * 32;
  // 32-row boxes feed MN-major operands (32-byte-atom swizzle); 128-row boxes are
  // K-major operands and the epilogue tile (plain 128-byte swizzle).  The maps of C
  // (source and store) end at column c1: loads beyond it read zeros and stores beyond
  // it are dropped, so a column-limited update touches nothing right of c1.
  const CUtensorMapSwizzle sw1 = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, sw3 = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap m_s32, m_s128, m_v32, m_v128, m_h128, m_w;
  if (!make_map(&m_s32, src, c1, n, n, batch, kR1, sw1) || !make_map(&m_s128, src, c1, n, n, batch, kR3, sw3) ||
      !make_map(&m_h128, H, c1, n, n, batch, kR3, sw3) || !make_map(&m_v32, H, n, n, n, batch, kR1, sw1) ||
      !make_map(&m_v128, H, n, n, n, batch, kR3, sw3) || !make_map(&m_w, w2, 32, 32, n, batch, kTN, sw3))
    return cudaErrorInvalidValue;
  return identity_fill ? launch_split<true>(m_s32, m_v32, m_s128, m_h128, m_v128, m_w, T, part, w2, batch, n, k,
                                            b, c0, c1, trans_t, store_to_h, s)
                       : launch_split<false>(m_s32, m_v32, m_s128, m_h128, m_v128, m_w, T, part, w2, batch, n, k,
                                             b, c0, c1, trans_t, store_to_h, s);
}

int tc_update_launches(int64_t batch, int n, int k, int c0, int c1) {
  return split_plan(batch, n, k, c0, c1).nsplit > 1 ? 3 : 2;
}

int* device_error_flag() {
  static std::atomic<int*> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (dev >= 0 && dev < 64) {
    int* p = cache[dev].load(std::memory_order_acquire);
    if (p != nullptr) return p;
  }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_qrb_device_error) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (dev >= 0 && dev < 64) cache[dev].store(static_cast<int*>(p), std::memory_order_release);
  return static_cast<int*>(p);
}

int take_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_qrb_device_error, sizeof v) != cudaSuccess) return -1;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_qrb_device_error, &zero, sizeof zero);
  }
  return v;
}

}  // namespace qrb
