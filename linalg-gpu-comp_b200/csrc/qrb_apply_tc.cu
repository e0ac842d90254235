// Block reflector application on the 5th-generation tensor cores:
//     C[k:, c0:] -= V op(T) (V^T C[k:, c0:])
// for the trailing update of geqrf (op = T^T) and the backward blocks of orgqr
// (op = T).  Replaces the reference's cuBLAS bmm / solve_triangular / baddbmm chain
// (_wy_trailing_trisolve, submission.py:434-460) and its cublasLt BF16x9 trailing
// GEMMs (submission.py:875-884).
//
// One CTA (4 warps) owns one matrix and a 64-column strip of C over all m rows.
// V (the panel's unit lower trapezoidal reflectors) is split into its three tf32 pieces
// once per panel by vprep_kernel and TMA-loaded piece by piece; without that workspace
// (the allocation-free entry point) each CTA splits V itself.
//   phase 1  W^T (64 x 32) = C^T V  : TMA streams 32-row stages of C and V into
//            shared memory (both operands MN-major, which for tf32 takes the 128-byte
//            swizzle with 32-byte atoms), threads split every value into three
//            tf32 pieces (x = x0 + x1 + x2), and one thread issues tcgen05.mma
//            kind::tf32, M=64 N=32 K=8, for the six products of weight >= 2^-22
//            (x0y0, x0y1, x1y0, x0y2, x1y1, x2y0), issued smallest class first
//            into one TMEM accumulator per stage; threads sum the stage partials in
//            fp32 registers.  Together: fp32 accuracy from the tf32 tensor pipe.
//   phase 2  W2 = op(T) W in registers (fp32), written K-major/swizzled as 3 pieces.
//   phase 3  per 128-row tile: TMA loads V and C, tcgen05.mma M=128 N=64 K=32 gives
//            V W2 in TMEM, the epilogue subtracts it from C in shared memory and a
//            TMA store writes the tile back.
// Every mbarrier wait is bounded; a wait that runs out records an error code in
// g_qrb_device_error and the kernel carries on to its TMEM release and exit.
// Requires n % 4 == 0 (TMA row strides are multiples of 16 bytes).
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "qrb_internal.cuh"
#include "qrb_sm100.cuh"

__device__ int g_qrb_device_error = 0;

namespace qrb {
namespace {

using namespace sm100;

constexpr int kTN = 64;        // strip width: phase-1 M, phase-3 N
constexpr int kR1 = 32;        // rows per phase-1 stage
constexpr int kR3 = 128;       // rows per phase-3 tile (M)
constexpr int kThreads = 128;
// TMEM: phase 1 uses two stage accumulators x 32 columns, phase 3 one x 64 columns.
constexpr uint32_t kTmemCols = 64;

// Shared-memory plan (bytes from a 1024-aligned base).  Operands are stored as three
// tf32 pieces; TMA lands raw fp32 in piece 0, which the split pass overwrites.
constexpr int kPieces = 3;
constexpr uint32_t kBox1 = kR1 * 128;            // 32 rows x 32 floats
constexpr uint32_t kStage1 = 9 * kBox1;          // C pieces 0..2 (2 boxes each), V pieces 0..2
constexpr uint32_t kBox3 = kR3 * 128;            // 128 rows x 32 floats
constexpr uint32_t kOffP3C = 0;                  // phase 3 aliases phase 1
constexpr uint32_t kOffP3V = 2 * kBox3;          // V pieces at kOffP3V + p * kBox3
constexpr uint32_t kRegionP = 5 * kBox3;         // 80 KB >= 2 * kStage1 (72 KB)
constexpr uint32_t kWPiece = kTN * 128;          // W2 piece: 64 rows x 32 floats
constexpr uint32_t kOffW = kRegionP;
constexpr uint32_t kOffT = kOffW + kPieces * kWPiece;
constexpr uint32_t kOffBar = kOffT + 32 * 33 * 4 + 32;
constexpr uint32_t kSmemBytes = kOffBar + 8 * 8 + 16 + 1024;   // + alignment slack

// The six (A piece, B piece) products kept, smallest first.  The tensor core's fp32
// accumulation rounds each add relative to the running sum, so all 2^-22 and 2^-11
// terms of a stage go in before its leading terms; an accumulator then takes four
// full-size roundings (one per K step), and stage partials are summed in fp32 registers,
// which keeps the error at the level of an fp32 SIMT dot product of the same length.
__device__ __constant__ int kTermA[6] = {2, 1, 0, 1, 0, 0};
__device__ __constant__ int kTermB[6] = {0, 1, 2, 0, 1, 0};

struct Bars {
  uint64_t tma1[2], mma1[2], tma3, mma3;
  uint32_t tmem;
};

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_qrb_device_error, 0, code); }

__device__ __forceinline__ void wait_or_flag(uint64_t* bar, uint32_t parity, int code) {
  if (!mbar_wait(bar, parity)) record_error(code);
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
  float a[4] = {v.x, v.y, v.z, v.w}, x0[4], x1[4], x2[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) split3_tf32(a[e], x0[e], x1[e], x2[e]);
  *reinterpret_cast<float4*>(p0 + off) = make_float4(x0[0], x0[1], x0[2], x0[3]);
  *reinterpret_cast<float4*>(p0 + pstride + off) = make_float4(x1[0], x1[1], x1[2], x1[3]);
  *reinterpret_cast<float4*>(p0 + 2 * pstride + off) = make_float4(x2[0], x2[1], x2[2], x2[3]);
}

// V pieces of one panel: vp[p][mat][row][32], rows k..n-1 written (masked V, 3 tf32 pieces).
__global__ void vprep_kernel(const float* __restrict__ H, float* __restrict__ vp, int64_t batch, int n,
                             int k, int b) {
  const int m = n - k;
  const int64_t total = batch * (int64_t)m * 32;
  const size_t piece = (size_t)batch * n * 32;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e & 31);
    const int64_t t = e >> 5;
    const int r = (int)(t % m);
    const int64_t mat = t / m;
    float x = 0.f;
    if (c < b) x = r > c ? __ldg(H + (size_t)mat * n * n + (size_t)(k + r) * n + k + c) : (r == c ? 1.f : 0.f);
    float x0, x1, x2;
    split3_tf32(x, x0, x1, x2);
    const size_t o = ((size_t)mat * n + k + r) * 32 + c;
    vp[o] = x0;
    vp[piece + o] = x1;
    vp[2 * piece + o] = x2;
  }
}

template <bool PREP, bool IDENT>
__global__ void __launch_bounds__(kThreads, 1)
apply_tc_kernel(const __grid_constant__ CUtensorMap map_src32, const __grid_constant__ CUtensorMap map_src128,
                const __grid_constant__ CUtensorMap map_v32, const __grid_constant__ CUtensorMap map_v128,
                const __grid_constant__ CUtensorMap map_h128, const float* __restrict__ Tg, int64_t batch,
                int n, int k, int b, int c0, int trans_t, int store_to_h) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                       ~uintptr_t(1023));
  Bars& bars = *reinterpret_cast<Bars*>(sm + kOffBar);
  float (*Ts)[33] = reinterpret_cast<float (*)[33]>(sm + kOffT);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nstrips = (n - c0 + kTN - 1) / kTN;
  const int mat = blockIdx.x / nstrips;
  const int cs = c0 + (int)(blockIdx.x % nstrips) * kTN;
  const int m = n - k, kb = k + b;
  const int nst = (m + kR1 - 1) / kR1;
  const int ntile = (m + kR3 - 1) / kR3;
  const int bz = (int)batch;   // z stride between V pieces in the prepared-V maps

  if (tid == 0) {
    mbar_init(&bars.tma1[0], 1);
    mbar_init(&bars.tma1[1], 1);
    mbar_init(&bars.mma1[0], 1);
    mbar_init(&bars.mma1[1], 1);
    mbar_init(&bars.tma3, 1);
    mbar_init(&bars.mma3, 1);
    fence_mbar_init();
    prefetch_tensormap(&map_src32);
    prefetch_tensormap(&map_v32);
  }
  if (warp == 0) tmem_alloc(&bars.tmem, kTmemCols);
  // op(T) into shared memory.
  const float* T = Tg + (size_t)mat * 32 * 32;
  for (int idx = tid; idx < 32 * 32; idx += kThreads) {
    const int r = idx >> 5, c = idx & 31;
    const float t = __ldg(T + idx);
    if (trans_t) Ts[c][r] = t; else Ts[r][c] = t;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars.tmem;

  auto issue_stage = [&](int s) {
    unsigned char* st = sm + (s & 1) * kStage1;
    const int y = k + s * kR1;
    mbar_arrive_expect_tx(&bars.tma1[s & 1], (PREP ? 5 : 3) * kBox1);
    tma_load_3d(st, &map_src32, cs, y, mat, &bars.tma1[s & 1]);
    tma_load_3d(st + kBox1, &map_src32, cs + 32, y, mat, &bars.tma1[s & 1]);
    if constexpr (PREP) {
#pragma unroll
      for (int p = 0; p < kPieces; ++p)
        tma_load_3d(st + (6 + p) * kBox1, &map_v32, 0, y, p * bz + mat, &bars.tma1[s & 1]);
    } else {
      tma_load_3d(st + 6 * kBox1, &map_v32, k, y, mat, &bars.tma1[s & 1]);
    }
  };

  // ---------------- phase 1: W^T = C^T V ------------------------------------------
  if (tid == 0) {
    issue_stage(0);
    if (nst > 1) issue_stage(1);
  }
  constexpr uint32_t idesc1 = idesc_tf32(kTN, 32, 1, 1);
  const uint32_t tm_lane = (uint32_t)(32 * warp) << 16;   // this warp's TMEM lanes
  float wacc[32];                                          // W^T row (lanes 0-15 meaningful)
#pragma unroll
  for (int j = 0; j < 32; ++j) wacc[j] = 0.f;
  // The partial of stage s lives in TMEM columns (s & 1) * 32 ..+32.
  auto gather_stage = [&](int s) {
    wait_or_flag(&bars.mma1[s & 1], (s >> 1) & 1, 3);
    tc_fence_after();
    float p[32];
    tmem_ld32(tmem + tm_lane + (s & 1) * 32, p);
#pragma unroll
    for (int j = 0; j < 32; ++j) wacc[j] += p[j];
    tc_fence_before();
  };
  for (int s = 0; s < nst; ++s) {
    const int buf = s & 1;
    const uint32_t par = (s >> 1) & 1;
    unsigned char* st = sm + buf * kStage1;
    wait_or_flag(&bars.tma1[buf], par, 1);
    // C: 2 boxes x 32 rows x 8 float4 -> three pieces, piece 0 in place.
    for (int u = tid; u < 2 * kR1 * 8; u += kThreads) {
      const int box = u >> 8, r = (u >> 3) & 31, q = u & 7;
      const uint32_t off = off32b(r, q);
      unsigned char* p0 = st + box * kBox1;
      float4 v = *reinterpret_cast<float4*>(p0 + off);
      if constexpr (IDENT) {
        const int R = k + s * kR1 + r;
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
    if constexpr (!PREP) {
      for (int u = tid; u < kR1 * 8; u += kThreads) {
        const int r = u >> 3, q = u & 7;
        const uint32_t off = off32b(r, q);
        unsigned char* p0 = st + 6 * kBox1;
        float4 v = *reinterpret_cast<float4*>(p0 + off);
        float a[4] = {v.x, v.y, v.z, v.w};
        const int rr = s * kR1 + r;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = 4 * q + e;
          a[e] = rr < 32 ? vmask(a[e], rr, col, b) : (col >= b ? 0.f : a[e]);
        }
        split4_store(p0, kBox1, off, make_float4(a[0], a[1], a[2], a[3]));
      }
    }
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t base = smem_u32(st);
      const uint32_t d = tmem + buf * 32;
#pragma unroll
      for (int t = 0; t < 6; ++t) {
#pragma unroll
        for (int kk = 0; kk < kR1 / 8; ++kk) {   // 8 K rows = 1024 bytes per MMA
          const uint64_t ad = sdesc_sw128_32b(base + 2 * kTermA[t] * kBox1 + kk * 1024, kBox1, 512);
          const uint64_t bd = sdesc_sw128_32b(base + (6 + kTermB[t]) * kBox1 + kk * 1024, kBox1, 512);
          mma_tf32(d, ad, bd, idesc1, (t > 0 || kk > 0) ? 1u : 0u);
        }
      }
      mma_commit(&bars.mma1[buf]);
    }
    // Fold the previous stage's partial while this stage's MMAs run, then refill.
    if (s > 0) gather_stage(s - 1);
    __syncthreads();
    if (tid == 0 && s + 2 < nst) {
      wait_or_flag(&bars.mma1[buf], par, 2);   // MMAs of stage s done reading this buffer
      issue_stage(s + 2);
    }
  }
  gather_stage(nst - 1);
  tc_fence_after();

  // ---------------- phase 2: W2 = op(T) W  (row i of W^T per lane pair) ---------------
  {
    // M = 64 layout: TMEM lanes 0-15 of each warp hold W^T rows 16*warp + lane.
    float w[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = __shfl_sync(0xffffffffu, wacc[j], lane & 15);
    const int i = 16 * warp + (lane & 15);                 // strip column
    const int a0 = (lane >> 4) * 16;                       // my 16 outputs
    unsigned char* wp = sm + kOffW;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int a = a0 + 4 * q + e;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) acc = fmaf(Ts[a][j], w[j], acc);
        o[e] = acc;
      }
      split4_store(wp, kWPiece, off128(i, (a0 >> 2) + q), make_float4(o[0], o[1], o[2], o[3]));
    }
  }
  tc_fence_before();
  fence_proxy_async();
  __syncthreads();
  tc_fence_after();

  // ---------------- phase 3: C -= V W2, 128-row tiles -----------------------------------
  constexpr uint32_t idesc3 = idesc_tf32(kR3, kTN, 0, 0);
  const CUtensorMap* map_store = store_to_h ? &map_h128 : &map_src128;
  unsigned char* c3 = sm + kOffP3C;
  unsigned char* v3 = sm + kOffP3V;
  for (int t = 0; t < ntile; ++t) {
    const int y0 = k + t * kR3;
    if (tid == 0) {
      if (t > 0) tma_store_wait_read();          // previous tile's store has read c3
      mbar_arrive_expect_tx(&bars.tma3, (PREP ? 5 : 3) * kBox3);
      tma_load_3d(c3, &map_src128, cs, y0, mat, &bars.tma3);
      tma_load_3d(c3 + kBox3, &map_src128, cs + 32, y0, mat, &bars.tma3);
      if constexpr (PREP) {
#pragma unroll
        for (int p = 0; p < kPieces; ++p)
          tma_load_3d(v3 + p * kBox3, &map_v128, 0, y0, p * bz + mat, &bars.tma3);
      } else {
        tma_load_3d(v3, &map_v128, k, y0, mat, &bars.tma3);
      }
    }
    wait_or_flag(&bars.tma3, t & 1, 4);
    if constexpr (!PREP) {
      for (int u = tid; u < kR3 * 8; u += kThreads) {
        const int r = u >> 3, q = u & 7;
        const uint32_t off = off128(r, q);
        float4 v = *reinterpret_cast<float4*>(v3 + off);
        float a[4] = {v.x, v.y, v.z, v.w};
        const int rr = t * kR3 + r;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = 4 * q + e;
          a[e] = rr < 32 ? vmask(a[e], rr, col, b) : (col >= b ? 0.f : a[e]);
        }
        split4_store(v3, kBox3, off, make_float4(a[0], a[1], a[2], a[3]));
      }
      fence_proxy_async();
    }
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t vb = smem_u32(v3), wb = smem_u32(sm + kOffW);
#pragma unroll
      for (int t3 = 0; t3 < 6; ++t3) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {   // 8 reflectors = 32 bytes per MMA
          const uint64_t ad = sdesc_sw128(vb + kTermA[t3] * kBox3 + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(wb + kTermB[t3] * kWPiece + kk * 32, 16, 1024);
          mma_tf32(tmem, ad, bd, idesc3, (t3 > 0 || kk > 0) ? 1u : 0u);
        }
      }
      mma_commit(&bars.mma3);
    }
    wait_or_flag(&bars.mma3, t & 1, 5);
    tc_fence_after();
    // Epilogue: row 32*warp + lane of the tile.
    {
      const int r = 32 * warp + lane;
      const int R = y0 + r;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float d[32];
        tmem_ld32(tmem + tm_lane + 32 * half, d);
        unsigned char* box = c3 + half * kBox3;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t off = off128(r, q);
          float4 c = *reinterpret_cast<float4*>(box + off);
          float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if constexpr (IDENT) {
              const int Cc = cs + 32 * half + 4 * q + e;
              if (R < n && Cc < n && (R < kb || Cc < kb)) cv[e] = R == Cc ? 1.f : 0.f;
            }
            cv[e] -= d[4 * q + e];
          }
          *reinterpret_cast<float4*>(box + off) = make_float4(cv[0], cv[1], cv[2], cv[3]);
        }
      }
    }
    tc_fence_before();
    fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tma_store_3d(map_store, c3, cs, y0, mat);
      tma_store_3d(map_store, c3 + kBox3, cs + 32, y0, mat);
      tma_store_commit();
    }
  }
  if (tid == 0) tma_store_wait_all();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
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

// 3-D fp32 map {cols, rows, depth} with row pitch `cols` floats, 32-column boxes.
bool make_map(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint64_t depth,
              int box_rows, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {cols, rows, depth};
  cuuint64_t strides[2] = {cols * 4, cols * rows * 4};
  cuuint32_t box[3] = {32, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool PREP, bool IDENT>
cudaError_t launch_t(const CUtensorMap& s32, const CUtensorMap& s128, const CUtensorMap& v32,
                     const CUtensorMap& v128, const CUtensorMap& h128, const float* T, int64_t batch, int n,
                     int k, int b, int c0, int trans_t, int store_to_h, cudaStream_t st) {
  static std::atomic<unsigned long long> attr_done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(apply_tc_kernel<PREP, IDENT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(bit, std::memory_order_acq_rel);
  }
  const unsigned grid = (unsigned)((int64_t)((n - c0 + kTN - 1) / kTN) * batch);
  apply_tc_kernel<PREP, IDENT><<<grid, kThreads, kSmemBytes, st>>>(s32, s128, v32, v128, h128, T, batch, n, k,
                                                                   b, c0, trans_t, store_to_h);
  return cudaGetLastError();
}

}  // namespace

bool apply_tc_supported(int n) { return n % 4 == 0 && n >= 64 && encode_fn() != nullptr; }

size_t vprep_floats(int64_t batch, int n) { return (size_t)kPieces * batch * n * 32; }

cudaError_t launch_apply_tc(const float* H, const float* T, const float* src, float* C, int64_t batch,
                            int n, int k, int b, int c0, int trans_t, int identity_fill, float* vprep,
                            cudaStream_t s) {
  if (batch == 0 || c0 >= n) return cudaSuccess;
  const int store_to_h = (C == H) ? 1 : 0;
  if (!store_to_h && C != src) return cudaErrorInvalidValue;   // C is either H or the source
  // Phase-1 boxes feed MN-major operands (32-byte-atom swizzle); phase-3 boxes are
  // K-major operands and the epilogue tile (plain 128-byte swizzle).
  const CUtensorMapSwizzle sw1 = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, sw3 = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap m_s32, m_s128, m_v32, m_v128, m_h128;
  if (!make_map(&m_s32, src, n, n, batch, kR1, sw1) || !make_map(&m_s128, src, n, n, batch, kR3, sw3) ||
      !make_map(&m_h128, H, n, n, batch, kR3, sw3))
    return cudaErrorInvalidValue;
  if (vprep != nullptr) {
    const int64_t total = batch * (int64_t)(n - k) * 32;
    const unsigned blocks = (unsigned)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
    vprep_kernel<<<blocks, 256, 0, s>>>(H, vprep, batch, n, k, b);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (!make_map(&m_v32, vprep, 32, n, kPieces * batch, kR1, sw1) ||
        !make_map(&m_v128, vprep, 32, n, kPieces * batch, kR3, sw3))
      return cudaErrorInvalidValue;
    return identity_fill
               ? launch_t<true, true>(m_s32, m_s128, m_v32, m_v128, m_h128, T, batch, n, k, b, c0, trans_t,
                                      store_to_h, s)
               : launch_t<true, false>(m_s32, m_s128, m_v32, m_v128, m_h128, T, batch, n, k, b, c0, trans_t,
                                       store_to_h, s);
  }
  if (!make_map(&m_v32, H, n, n, batch, kR1, sw1) || !make_map(&m_v128, H, n, n, batch, kR3, sw3))
    return cudaErrorInvalidValue;
  return identity_fill
             ? launch_t<false, true>(m_s32, m_s128, m_v32, m_v128, m_h128, T, batch, n, k, b, c0, trans_t,
                                     store_to_h, s)
             : launch_t<false, false>(m_s32, m_s128, m_v32, m_v128, m_h128, T, batch, n, k, b, c0, trans_t,
                                      store_to_h, s);
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
