// Per-launch kernel timing (qrb_kernel_timing / qrb_kernel_timing_report) and the
// per-device SM count used to size persistent grids.
//
// When timing is on, every launch helper brackets its kernel with two CUDA events
// recorded on the launching stream and logs (kernel name, events, algorithmic bytes,
// flops).  The report synchronises on the logged events and sums durations per name.
// Off by default: the only cost then is one relaxed atomic load per launch.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/qrb200.h"
#include "qrb_internal.cuh"

namespace qrb {
namespace {

std::atomic<int> g_timing_on{0};

struct Record {
  const char* name;
  cudaEvent_t e0, e1;
  double bytes, flops;
};

struct Log {
  std::mutex mu;
  std::vector<Record> recs;
  std::vector<cudaEvent_t> pool;   // events of cleared records, reused
};

Log& log_() {
  static Log* l = new Log();   // never destroyed: launches may run during static teardown
  return *l;
}

cudaEvent_t take_event(Log& l) {
  if (!l.pool.empty()) {
    cudaEvent_t e = l.pool.back();
    l.pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

}  // namespace

LaunchTimer::LaunchTimer(const char* name, cudaStream_t s, double bytes, double flops)
    : name_(name), s_(s), bytes_(bytes), flops_(flops) {
  if (g_timing_on.load(std::memory_order_relaxed) == 0) return;
  Log& l = log_();
  std::lock_guard<std::mutex> lock(l.mu);
  e0_ = take_event(l);
  e1_ = take_event(l);
  if (e0_ == nullptr || e1_ == nullptr || cudaEventRecord(e0_, s_) != cudaSuccess) {
    cudaGetLastError();
    if (e0_) l.pool.push_back(e0_);
    if (e1_) l.pool.push_back(e1_);
    e0_ = e1_ = nullptr;
  }
}

LaunchTimer::~LaunchTimer() {
  if (e0_ == nullptr) return;
  Log& l = log_();
  std::lock_guard<std::mutex> lock(l.mu);
  if (cudaEventRecord(e1_, s_) != cudaSuccess) {
    cudaGetLastError();
    l.pool.push_back(e0_);
    l.pool.push_back(e1_);
    return;
  }
  l.recs.push_back(Record{name_, e0_, e1_, bytes_, flops_});
}

int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    cudaGetLastError();
    return 148;
  }
  if (dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return 148;
  }
  if (dev < 64) cache[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

}  // namespace qrb

extern "C" {

QRB_API void qrb_kernel_timing(int enable) { qrb::g_timing_on.store(enable != 0 ? 1 : 0); }

QRB_API size_t qrb_kernel_timing_report(char* buf, size_t len) {
  using qrb::Record;
  auto& l = qrb::log_();
  // A size query (buf == NULL) leaves the log in place; a report clears it.
  const bool consume = buf != nullptr && len > 0;
  std::vector<Record> recs;
  {
    std::lock_guard<std::mutex> lock(l.mu);
    if (consume) recs.swap(l.recs);
    else recs = l.recs;
  }
  struct Agg {
    long long count = 0;
    double ms = 0, bytes = 0, flops = 0;
  };
  std::map<std::string, Agg> agg;
  for (const Record& r : recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.e1) != cudaSuccess || cudaEventElapsedTime(&ms, r.e0, r.e1) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    Agg& a = agg[r.name];
    a.count += 1;
    a.ms += ms;
    a.bytes += r.bytes;
    a.flops += r.flops;
  }
  if (consume) {
    std::lock_guard<std::mutex> lock(l.mu);
    for (const Record& r : recs) {
      l.pool.push_back(r.e0);
      l.pool.push_back(r.e1);
    }
  }
  std::string out;
  char line[256];
  for (const auto& kv : agg) {
    snprintf(line, sizeof line, "%s %lld %.6f %.0f %.0f\n", kv.first.c_str(), kv.second.count, kv.second.ms,
             kv.second.bytes, kv.second.flops);
    out += line;
  }
  if (buf != nullptr && len > 0) {
    const size_t c = out.size() < len - 1 ? out.size() : len - 1;
    std::memcpy(buf, out.data(), c);
    buf[c] = '\0';
  }
  return out.size() + 1;
}

}  // extern "C"
