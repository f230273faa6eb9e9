// Per-kernel device timing: when enabled, every kernel launch made through
// the library is bracketed by CUDA events on its own stream, and
// fmoe_profile_read() resolves and aggregates them by kernel name.  This is
// the device-side replacement for the reference's phase accumulators
// (src/perf.rs:65-153), which time host-observed eval barriers.
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>
#include "internal.h"

namespace fmoe {

namespace {
struct Pending {
  const char* name;
  cudaEvent_t a, b;
};
struct Stat {
  std::string name;
  int64_t n;
  double ms;
};
std::atomic<int> g_enabled{0};
std::mutex g_mu;
std::vector<Pending> g_pending;
std::vector<Stat> g_stats;
}  // namespace

ProfScope::ProfScope(const char* name, cudaStream_t st) : name_(name), st_(st), a_(nullptr), b_(nullptr) {
  if (!g_enabled.load(std::memory_order_relaxed)) return;
  if (cudaEventCreate(&a_) != cudaSuccess || cudaEventCreate(&b_) != cudaSuccess) {
    a_ = b_ = nullptr;
    return;
  }
  cudaEventRecord(a_, st_);
}

ProfScope::~ProfScope() {
  if (!a_) return;
  cudaEventRecord(b_, st_);
  std::lock_guard<std::mutex> lk(g_mu);
  g_pending.push_back({name_, a_, b_});
}

}  // namespace fmoe

using namespace fmoe;

extern "C" {

int fmoe_profile_enable(int on) {
  g_enabled.store(on ? 1 : 0);
  return FMOE_OK;
}

int fmoe_profile_read(fmoe_kernel_stat_t* out, int max_entries, int reset) {
  std::lock_guard<std::mutex> lk(g_mu);
  int rc = FMOE_OK;
  for (auto& p : g_pending) {
    float ms = 0.f;
    if (cudaEventSynchronize(p.b) != cudaSuccess || cudaEventElapsedTime(&ms, p.a, p.b) != cudaSuccess)
      rc = set_error(FMOE_ERR_CUDA, "profile_read: event query failed");
    cudaEventDestroy(p.a);
    cudaEventDestroy(p.b);
    bool found = false;
    for (auto& s : g_stats)
      if (s.name == p.name) {
        s.n += 1;
        s.ms += ms;
        found = true;
        break;
      }
    if (!found) g_stats.push_back({p.name, 1, ms});
  }
  g_pending.clear();
  if (rc) return rc;
  const int n = (int)g_stats.size();
  for (int i = 0; out && i < n && i < max_entries; ++i) {
    std::strncpy(out[i].name, g_stats[i].name.c_str(), sizeof(out[i].name) - 1);
    out[i].name[sizeof(out[i].name) - 1] = 0;
    out[i].launches = g_stats[i].n;
    out[i].total_ms = g_stats[i].ms;
  }
  if (reset) g_stats.clear();
  return n;
}

}  // extern "C"
