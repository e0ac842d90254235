// C ABI of libqrb200 (declared in include/qrb200.h): argument checks, workspace
// layout and the regime dispatch of the batched QR.
//
// Dispatch (replaces custom_kernel's shape dispatch, submission.py:905-921):
//   n <= 64  : one fused CTA per matrix (qrb_small.cu) -- geqrf and Q in one launch.
//   n >  64  : right-looking blocked Householder, panel width 32:
//                for each panel k: panel geqr2 + T (qrb_panel.cu), then the
//                trailing update A[k:, k+32:] -= V T^T V^T A (qrb_apply_tc.cu on
//                the tensor cores for n % 4 == 0, qrb_apply.cu otherwise);
//              Q by backward block accumulation Q[k:, k:] -= V T V^T Q[k:, k:]
//              over the same T factors, with the identity generated on the fly.
// Workspace: the T factors of every panel, [panel][batch][32][32] fp32, then the
// tensor-core update's scratch (see ws_bytes).
//
// Large n (n % 4 == 0, n >= kWideMinN) takes the wide-block path instead: panels of 32
// are grouped into blocks of 128 columns; inside a block each panel updates only the
// rest of the block (column-limited 32-wide update), and the block as a whole updates
// the trailing matrix and forms Q with 128-wide block reflectors (qrb_wide.cu).
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/qrb200.h"
#include "qrb_internal.cuh"

namespace {

thread_local std::string g_last_msg;
thread_local int g_last_status = QRB_OK;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_msg = buf;
  g_last_status = status;
  return status;
}

}  // namespace

namespace qrb {
int set_error(int status, const char* msg) {
  g_last_msg = msg;
  g_last_status = status;
  return status;
}
}  // namespace qrb

namespace {

int cuda_fail(cudaError_t e, const char* what) {
  return fail(QRB_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int n_panels(int n) { return (n + qrb::kNB - 1) / qrb::kNB; }

size_t t_bytes(int64_t batch, int n) {
  return (size_t)n_panels(n) * (size_t)batch * qrb::kNB * qrb::kNB * sizeof(float);
}

// Sizes the workspace for the wide path whenever n qualifies (a pure size rule, so the
// answer does not depend on the device); dispatch additionally needs TMA support.
bool wide_eligible(int n) { return n % 4 == 0 && n >= qrb::kWideMinN; }

// Smallest n dispatched to the wide path: kWideDefaultN, or the environment variable
// QRB_WIDE_MIN_N (read once per process; values below kWideMinN are raised to it).
int wide_min_n() {
  static const int v = [] {
    const char* e = std::getenv("QRB_WIDE_MIN_N");
    int x = e != nullptr ? std::atoi(e) : qrb::kWideDefaultN;
    return x < qrb::kWideMinN ? qrb::kWideMinN : x;
  }();
  return v;
}

bool use_wide(int n) { return wide_eligible(n) && n >= wide_min_n() && qrb::wide_supported(n); }

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace: the T factors of every panel, then (for the tensor-core path, n % 4 == 0)
// the update's scratch: W2 and the row-chunk partials of W^T (qrb::tc_ws_floats), then
// (wide path) the block T factors, V and W2 pieces and Y partials (qrb::wide_ws_floats).
size_t ws_bytes(int64_t batch, int n) {
  if (n <= qrb::kSmallMaxN) return 0;
  size_t bytes = t_bytes(batch, n);
  if (n % 4 == 0) bytes = al256(bytes) + qrb::tc_ws_floats(batch, n) * sizeof(float);
  if (wide_eligible(n)) bytes = al256(bytes) + qrb::wide_ws_floats(batch, n) * sizeof(float);
  return bytes;
}

float* tc_ws(void* ws, int64_t batch, int n) {
  if (n % 4 != 0) return nullptr;
  return reinterpret_cast<float*>(static_cast<char*>(ws) + al256(t_bytes(batch, n)));
}

float* wide_ws(void* ws, int64_t batch, int n) {
  return reinterpret_cast<float*>(static_cast<char*>(ws) + al256(al256(t_bytes(batch, n)) +
                                                                 qrb::tc_ws_floats(batch, n) * sizeof(float)));
}

// The kernels are built for sm_100a only: refuse anything else up front rather
// than failing with "no kernel image" deep inside a launch sequence.
int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  static int major_cache[64] = {0};
  int major = dev < 64 ? major_cache[dev] : 0;
  if (major == 0) {
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    if (dev < 64) major_cache[dev] = major;
  }
  if (major != 10) return fail(QRB_ERR_DEVICE, "device %d has compute capability %d.x; libqrb200 needs sm_100", dev, major);
  return QRB_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_common(int64_t batch, int n, const void* ws, size_t wsb) {
  if (batch < 0) return fail(QRB_ERR_INVALID_ARG, "batch must be >= 0 (got %lld)", (long long)batch);
  if (n < 1) return fail(QRB_ERR_INVALID_ARG, "n must be >= 1 (got %d)", n);
  if (n > QRB_MAX_N) return fail(QRB_ERR_UNSUPPORTED, "n = %d exceeds QRB_MAX_N = %d", n, QRB_MAX_N);
  if (batch > (int64_t)1 << 31) return fail(QRB_ERR_UNSUPPORTED, "batch = %lld exceeds 2^31", (long long)batch);
  const size_t need = ws_bytes(batch, n);
  if (need > 0 && (ws == nullptr || wsb < need))
    return fail(QRB_ERR_WORKSPACE, "workspace of %zu bytes required, %zu given%s", need, wsb,
                ws == nullptr ? " (null)" : "");
  if (need > 0 && (reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
    return fail(QRB_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
  return QRB_OK;
}

// Matrices are read and written with 16-byte vector accesses; tau only needs float alignment.
int check_ptr(const void* p, const char* name, bool vec = true) {
  if (p == nullptr) return fail(QRB_ERR_INVALID_ARG, "%s is null", name);
  if (vec ? !aligned16(p) : (reinterpret_cast<uintptr_t>(p) & 3u) != 0)
    return fail(QRB_ERR_INVALID_ARG, "%s must be %d-byte aligned", name, vec ? 16 : 4);
  return QRB_OK;
}

#define QRB_TRY(x)                   \
  do {                               \
    int _s = (x);                    \
    if (_s != QRB_OK) return _s;     \
  } while (0)
#define QRB_CUDA(x, what)                          \
  do {                                             \
    cudaError_t _e = (x);                          \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

float* panel_T(void* ws, int64_t batch, int p) {
  return static_cast<float*>(ws) + (size_t)p * (size_t)batch * qrb::kNB * qrb::kNB;
}

// Wide path: blocks of up to 128 columns, four panels each.  `with_t`: keep every
// block's T factor for a following Q formation.
int wide_geqrf(const float* A, float* H, float* tau, int64_t batch, int n, void* ws, bool with_t,
               cudaStream_t s) {
  float* tcw = tc_ws(ws, batch, n);
  float* wws = wide_ws(ws, batch, n);
  for (int K = 0; K < n; K += qrb::kWideNB) {
    const int bw = n - K < qrb::kWideNB ? n - K : qrb::kWideNB;
    for (int k = K; k < K + bw; k += qrb::kNB) {
      const int b = n - k < qrb::kNB ? n - k : qrb::kNB;
      const float* src = k == 0 ? A : H;
      float* T = panel_T(ws, batch, k / qrb::kNB);
      QRB_CUDA(qrb::launch_panel(src, H, tau, T, batch, n, k, b, s), "panel kernel launch");
      if (k + b < K + bw)
        QRB_CUDA(qrb::launch_apply(H, T, src, H, batch, n, k, b, k + b, K + bw, 1, 0, tcw, s),
                 "in-block update launch");
    }
    QRB_CUDA(qrb::wide_geqrf_block(K == 0 ? A : H, H, panel_T(ws, batch, K / qrb::kNB), wws, batch, n, K, bw,
                                   with_t, true, s),
             "wide block update launch");
  }
  return QRB_OK;
}

int wide_orgqr(const float* H, float* Q, int64_t batch, int n, void* ws, cudaStream_t s) {
  float* wws = wide_ws(ws, batch, n);
  for (int K = (n - 1) / qrb::kWideNB * qrb::kWideNB; K >= 0; K -= qrb::kWideNB) {
    const int bw = n - K < qrb::kWideNB ? n - K : qrb::kWideNB;
    QRB_CUDA(qrb::wide_orgqr_block(H, Q, wws, batch, n, K, bw, s), "wide orgqr block launch");
  }
  return QRB_OK;
}

int blocked_geqrf(const float* A, float* H, float* tau, int64_t batch, int n, void* ws,
                  cudaStream_t s) {
  if (use_wide(n)) return wide_geqrf(A, H, tau, batch, n, ws, false, s);
  const int np = n_panels(n);
  for (int p = 0; p < np; ++p) {
    const int k = p * qrb::kNB, b = n - k < qrb::kNB ? n - k : qrb::kNB;
    const float* src = p == 0 ? A : H;
    float* T = panel_T(ws, batch, p);
    QRB_CUDA(qrb::launch_panel(src, H, tau, T, batch, n, k, b, s), "panel kernel launch");
    if (k + b < n)
      QRB_CUDA(qrb::launch_apply(H, T, src, H, batch, n, k, b, k + b, n, 1, 0, tc_ws(ws, batch, n), s),
               "trailing update launch");
  }
  return QRB_OK;
}

int blocked_orgqr(const float* H, float* Q, int64_t batch, int n, void* ws, cudaStream_t s) {
  if (use_wide(n)) return wide_orgqr(H, Q, batch, n, ws, s);
  for (int p = n_panels(n) - 1; p >= 0; --p) {
    const int k = p * qrb::kNB, b = n - k < qrb::kNB ? n - k : qrb::kNB;
    QRB_CUDA(qrb::launch_apply(H, panel_T(ws, batch, p), Q, Q, batch, n, k, b, k, n, 0, 1, tc_ws(ws, batch, n), s),
             "orgqr block launch");
  }
  return QRB_OK;
}

// (H, tau[, Q]) of a device batch on stream s; arguments already checked.
// The QR in two halves: run_qr_h leaves (H, tau) final; run_qr_q forms Q from them
// (nothing to do for n <= 64, where one launch does both).  The host pipeline copies H
// out while Q is being formed.
int run_qr_h(const float* A, float* H, float* tau, float* Q, int64_t batch, int n, void* ws, cudaStream_t s) {
  if (n <= qrb::kSmallMaxN) {
    QRB_CUDA(qrb::launch_small(A, H, tau, Q, batch, n, Q != nullptr ? 3 : 1, s), "small-n kernel launch");
    return QRB_OK;
  }
  if (use_wide(n)) return wide_geqrf(A, H, tau, batch, n, ws, Q != nullptr, s);
  return blocked_geqrf(A, H, tau, batch, n, ws, s);
}

int run_qr_q(const float* H, float* Q, int64_t batch, int n, void* ws, cudaStream_t s) {
  if (Q == nullptr || n <= qrb::kSmallMaxN) return QRB_OK;
  if (use_wide(n)) return wide_orgqr(H, Q, batch, n, ws, s);
  return blocked_orgqr(H, Q, batch, n, ws, s);
}

int run_qr(const float* A, float* H, float* tau, float* Q, int64_t batch, int n, void* ws, cudaStream_t s) {
  QRB_TRY(run_qr_h(A, H, tau, Q, batch, n, ws, s));
  return run_qr_q(H, Q, batch, n, ws, s);
}

// Kernels run_qr enqueues (it mirrors that dispatch).
int64_t count_launches(int64_t batch, int n, bool with_q) {
  if (n <= qrb::kSmallMaxN) return 1;
  const int np = n_panels(n);
  auto update = [&](int k, int c0, int c1) -> int64_t {
    return n % 4 == 0 ? qrb::tc_update_launches(batch, n, k, c0, c1) : 1;
  };
  if (use_wide(n)) {
    int64_t total = 0;
    for (int K = 0; K < n; K += qrb::kWideNB) {
      const int bw = n - K < qrb::kWideNB ? n - K : qrb::kWideNB;
      for (int k = K; k < K + bw; k += qrb::kNB) {
        const int b = n - k < qrb::kNB ? n - k : qrb::kNB;
        total += 1;
        if (k + b < K + bw) total += update(k, k + b, K + bw);
      }
      const bool upd = K + bw < n;
      total += qrb::wide_block_launches(batch, n, K, upd, upd || with_q, false);
      if (with_q) total += qrb::wide_block_launches(batch, n, K, false, false, true);
    }
    return total;
  }
  int64_t total = np;
  for (int p = 0; p < np; ++p) {
    const int k = p * qrb::kNB, b = n - k < qrb::kNB ? n - k : qrb::kNB;
    if (k + b < n) total += update(k, k + b, n);
    if (with_q) total += update(k, k, n);
  }
  return total;
}

// ---- host-buffer pipeline -------------------------------------------------------
// The batch is cut into chunks that cycle through kSlots device slots; per chunk the
// copy-in stream moves A to the slot, the compute stream factors it in place (and
// forms Q), and the copy-out stream moves H, tau and Q back.  The two copy
// directions use separate copy engines, so with three slots the host link carries
// input and output at the same time while the SMs work on a third chunk.
constexpr int kSlots = 3;

int host_chunks(int64_t batch, int n) {
  const int k = n <= 128 ? 8 : (n <= 512 ? 4 : 2);
  return (int)(batch < k ? batch : k);
}

struct HostPlan {
  int64_t cb;            // matrices per chunk
  size_t x_off, t_off, q_off, w_off, slot_bytes, total;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

HostPlan host_plan(int64_t batch, int n, bool with_q) {
  HostPlan p{};
  const int k = host_chunks(batch, n);
  p.cb = k > 0 ? (batch + k - 1) / k : 0;
  const size_t mat = (size_t)p.cb * n * n * sizeof(float);
  p.x_off = 0;
  p.t_off = align256(mat);
  p.q_off = p.t_off + align256((size_t)p.cb * n * sizeof(float));
  p.w_off = p.q_off + (with_q ? align256(mat) : 0);
  p.slot_bytes = p.w_off + align256(ws_bytes(p.cb, n));
  p.total = p.cb > 0 ? kSlots * p.slot_bytes : 0;
  return p;
}

// Internal streams of the host pipeline, one triple per device, created on first use.
bool pipe_streams(int dev, cudaStream_t (&out)[3]) {
  static std::mutex mu;
  static cudaStream_t streams[64][3] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return false;
  if (streams[dev][0] == nullptr) {
    cudaStream_t t[3] = {nullptr, nullptr, nullptr};
    for (auto& x : t)
      if (cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking) != cudaSuccess) {
        for (auto y : t)
          if (y) cudaStreamDestroy(y);
        cudaGetLastError();
        return false;
      }
    for (int i = 0; i < 3; ++i) streams[dev][i] = t[i];
  }
  for (int i = 0; i < 3; ++i) out[i] = streams[dev][i];
  return true;
}

struct Events {
  cudaEvent_t e[4 * kSlots + 1] = {};
  int made = 0;
  cudaError_t create() {
    for (auto& x : e) {
      cudaError_t r = cudaEventCreateWithFlags(&x, cudaEventDisableTiming);
      if (r != cudaSuccess) return r;
      ++made;
    }
    return cudaSuccess;
  }
  ~Events() {
    for (int i = 0; i < made; ++i) cudaEventDestroy(e[i]);
  }
};

int host_qr(const float* A, float* H, float* tau, float* Q, int64_t batch, int n, void* dws, size_t dwsb,
            cudaStream_t s) {
  const HostPlan p = host_plan(batch, n, Q != nullptr);
  if (dws == nullptr || dwsb < p.total)
    return fail(QRB_ERR_WORKSPACE, "device workspace of %zu bytes required, %zu given%s", p.total, dwsb,
                dws == nullptr ? " (null)" : "");
  if ((reinterpret_cast<uintptr_t>(dws) & 255u) != 0)
    return fail(QRB_ERR_INVALID_ARG, "device workspace must be 256-byte aligned");
  QRB_TRY(check_device());
  int dev = 0;
  QRB_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  cudaStream_t st[3];
  if (!pipe_streams(dev, st)) return fail(QRB_ERR_CUDA, "could not create the pipeline streams");
  Events ev;   // [slot]: copied in, computed, copied out, H final; last: fork
  QRB_CUDA(ev.create(), "cudaEventCreate");
  cudaEvent_t* in_ev = ev.e;
  cudaEvent_t* done_ev = ev.e + kSlots;
  cudaEvent_t* out_ev = ev.e + 2 * kSlots;
  cudaEvent_t* h_ev = ev.e + 3 * kSlots;
  cudaEvent_t fork = ev.e[4 * kSlots];
  QRB_CUDA(cudaEventRecord(fork, s), "cudaEventRecord");
  for (auto x : st) QRB_CUDA(cudaStreamWaitEvent(x, fork, 0), "cudaStreamWaitEvent");
  const size_t nn = (size_t)n * n;
  int chunk = 0;
  for (int64_t b0 = 0; b0 < batch; ++chunk) {
    const int64_t cb = batch - b0 < p.cb ? batch - b0 : p.cb;
    const int slot = chunk % kSlots;
    char* base = static_cast<char*>(dws) + slot * p.slot_bytes;
    float* X = reinterpret_cast<float*>(base + p.x_off);
    float* T = reinterpret_cast<float*>(base + p.t_off);
    float* Qd = Q != nullptr ? reinterpret_cast<float*>(base + p.q_off) : nullptr;
    void* W = base + p.w_off;
    if (chunk >= kSlots) QRB_CUDA(cudaStreamWaitEvent(st[0], out_ev[slot], 0), "cudaStreamWaitEvent");
    QRB_CUDA(cudaMemcpyAsync(X, A + b0 * nn, cb * nn * sizeof(float), cudaMemcpyHostToDevice, st[0]),
             "copy-in");
    QRB_CUDA(cudaEventRecord(in_ev[slot], st[0]), "cudaEventRecord");
    QRB_CUDA(cudaStreamWaitEvent(st[1], in_ev[slot], 0), "cudaStreamWaitEvent");
    // H and tau go out while Q is formed (the Q kernels only read H).
    QRB_TRY(run_qr_h(X, X, T, Qd, cb, n, W, st[1]));
    QRB_CUDA(cudaEventRecord(h_ev[slot], st[1]), "cudaEventRecord");
    QRB_TRY(run_qr_q(X, Qd, cb, n, W, st[1]));
    QRB_CUDA(cudaEventRecord(done_ev[slot], st[1]), "cudaEventRecord");
    QRB_CUDA(cudaStreamWaitEvent(st[2], h_ev[slot], 0), "cudaStreamWaitEvent");
    QRB_CUDA(cudaMemcpyAsync(H + b0 * nn, X, cb * nn * sizeof(float), cudaMemcpyDeviceToHost, st[2]),
             "copy-out");
    QRB_CUDA(cudaMemcpyAsync(tau + b0 * n, T, cb * n * sizeof(float), cudaMemcpyDeviceToHost, st[2]),
             "copy-out");
    QRB_CUDA(cudaStreamWaitEvent(st[2], done_ev[slot], 0), "cudaStreamWaitEvent");
    if (Qd != nullptr)
      QRB_CUDA(cudaMemcpyAsync(Q + b0 * nn, Qd, cb * nn * sizeof(float), cudaMemcpyDeviceToHost, st[2]),
               "copy-out");
    QRB_CUDA(cudaEventRecord(out_ev[slot], st[2]), "cudaEventRecord");
    b0 += cb;
  }
  // Join: the copy-out stream is downstream of the other two.
  QRB_CUDA(cudaEventRecord(fork, st[2]), "cudaEventRecord");
  QRB_CUDA(cudaStreamWaitEvent(s, fork, 0), "cudaStreamWaitEvent");
  return QRB_OK;
}

}  // namespace

extern "C" {

int qrb_version(void) { return 100; }

const char* qrb_status_string(int status) {
  switch (status) {
    case QRB_OK: return "ok";
    case QRB_ERR_INVALID_ARG: return "invalid argument";
    case QRB_ERR_UNSUPPORTED: return "unsupported size";
    case QRB_ERR_WORKSPACE: return "workspace missing or too small";
    case QRB_ERR_CUDA: return "CUDA error";
    case QRB_ERR_DEVICE: return "unsupported device";
    default: return "unknown status";
  }
}

int qrb_last_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) {
    std::strncpy(buf, g_last_msg.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return g_last_status;
}

int qrb_device_error(void) { return qrb::take_device_error(); }

size_t qrb_workspace_size(int64_t batch, int n) {
  if (batch < 0 || n < 1 || n > QRB_MAX_N) return 0;
  return ws_bytes(batch, n);
}

int64_t qrb_kernel_launches(int64_t batch, int n, int with_q) {
  if (batch <= 0 || n < 1 || n > QRB_MAX_N) return 0;
  return count_launches(batch, n, with_q != 0);
}

int qrb_geqrf_f32(const float* A, float* H, float* tau, int64_t batch, int n, void* workspace,
                  size_t workspace_bytes, void* stream) {
  QRB_TRY(check_common(batch, n, workspace, workspace_bytes));
  if (batch == 0) return QRB_OK;   // nothing to do; pointers may be null
  QRB_TRY(check_ptr(A, "A"));
  QRB_TRY(check_ptr(H, "H"));
  QRB_TRY(check_ptr(tau, "tau", false));
  QRB_TRY(check_device());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n <= qrb::kSmallMaxN) {
    QRB_CUDA(qrb::launch_small(A, H, tau, nullptr, batch, n, 1, s), "small-n kernel launch");
    return QRB_OK;
  }
  return blocked_geqrf(A, H, tau, batch, n, workspace, s);
}

int qrb_orgqr_f32(const float* H, const float* tau, float* Q, int64_t batch, int n,
                  void* workspace, size_t workspace_bytes, void* stream) {
  QRB_TRY(check_common(batch, n, workspace, workspace_bytes));
  if (batch == 0) return QRB_OK;   // nothing to do; pointers may be null
  QRB_TRY(check_ptr(H, "H"));
  QRB_TRY(check_ptr(tau, "tau", false));
  QRB_TRY(check_ptr(Q, "Q"));
  if (Q == H) return fail(QRB_ERR_INVALID_ARG, "Q must not alias H");
  if (batch == 0) return QRB_OK;
  QRB_TRY(check_device());
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n <= qrb::kSmallMaxN) {
    QRB_CUDA(qrb::launch_small(nullptr, const_cast<float*>(H), const_cast<float*>(tau), Q, batch, n, 2, s),
             "small-n kernel launch");
    return QRB_OK;
  }
  QRB_CUDA(qrb::launch_larft(H, tau, static_cast<float*>(workspace), batch, n, s), "larft launch");
  if (use_wide(n)) {
    float* wws = wide_ws(workspace, batch, n);
    for (int K = 0; K < n; K += qrb::kWideNB) {
      const int bw = n - K < qrb::kWideNB ? n - K : qrb::kWideNB;
      QRB_CUDA(qrb::wide_geqrf_block(H, const_cast<float*>(H), panel_T(workspace, batch, K / qrb::kNB), wws, batch,
                                     n, K, bw, true, false, s),
               "wide T factor launch");
    }
  }
  return blocked_orgqr(H, Q, batch, n, workspace, s);
}

int qrb_qr_f32(const float* A, float* H, float* tau, float* Q, int64_t batch, int n,
               void* workspace, size_t workspace_bytes, void* stream) {
  QRB_TRY(check_common(batch, n, workspace, workspace_bytes));
  if (batch == 0) return QRB_OK;   // nothing to do; pointers may be null
  QRB_TRY(check_ptr(A, "A"));
  QRB_TRY(check_ptr(H, "H"));
  QRB_TRY(check_ptr(tau, "tau", false));
  QRB_TRY(check_ptr(Q, "Q"));
  if (Q == H || Q == A) return fail(QRB_ERR_INVALID_ARG, "Q must not alias A or H");
  QRB_TRY(check_device());
  return run_qr(A, H, tau, Q, batch, n, workspace, static_cast<cudaStream_t>(stream));
}

size_t qrb_host_workspace_size(int64_t batch, int n, int with_q) {
  if (batch < 0 || n < 1 || n > QRB_MAX_N) return 0;
  return host_plan(batch, n, with_q != 0).total;
}

int qrb_qr_f32_host(const float* A, float* H, float* tau, float* Q, int64_t batch, int n,
                    void* device_workspace, size_t device_workspace_bytes, void* stream) {
  if (batch < 0) return fail(QRB_ERR_INVALID_ARG, "batch must be >= 0 (got %lld)", (long long)batch);
  if (n < 1) return fail(QRB_ERR_INVALID_ARG, "n must be >= 1 (got %d)", n);
  if (n > QRB_MAX_N) return fail(QRB_ERR_UNSUPPORTED, "n = %d exceeds QRB_MAX_N = %d", n, QRB_MAX_N);
  if (batch > (int64_t)1 << 31) return fail(QRB_ERR_UNSUPPORTED, "batch = %lld exceeds 2^31", (long long)batch);
  if (batch == 0) return QRB_OK;
  if (A == nullptr) return fail(QRB_ERR_INVALID_ARG, "A is null");
  if (H == nullptr) return fail(QRB_ERR_INVALID_ARG, "H is null");
  if (tau == nullptr) return fail(QRB_ERR_INVALID_ARG, "tau is null");
  if (Q != nullptr && (Q == H || Q == A)) return fail(QRB_ERR_INVALID_ARG, "Q must not alias A or H");
  return host_qr(A, H, tau, Q, batch, n, device_workspace, device_workspace_bytes,
                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
