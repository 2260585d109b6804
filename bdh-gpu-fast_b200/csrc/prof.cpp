// Optional launch timing: between bdh_profile_begin() and bdh_profile_end() every kernel launch
// of the library is bracketed by two CUDA events recorded on its own stream, so a caller (the
// benchmark) can attribute device time to each kernel kind inside its timed region without a
// profiler. Off by default: when inactive the hooks cost one atomic load.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "bdh_sm100.h"
#include "internal.h"
#include "tma_host.h"

namespace bdh {

namespace {
struct Rec {
  int kind;
  cudaEvent_t a, b;
};
std::atomic<bool> g_on{false};
std::mutex g_mu;
std::vector<Rec> g_recs;
std::vector<cudaEvent_t> g_pool;
thread_local cudaEvent_t t_pending = nullptr;

cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}
}  // namespace

void prof_start(int kind, cudaStream_t s) {
  (void)kind;
  if (!g_on.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_mu);
  t_pending = take_event();
  if (t_pending) cudaEventRecord(t_pending, s);
}

void prof_stop(int kind, cudaStream_t s) {
  if (!g_on.load(std::memory_order_relaxed) || t_pending == nullptr) return;
  std::lock_guard<std::mutex> lk(g_mu);
  cudaEvent_t b = take_event();
  if (b == nullptr) return;
  cudaEventRecord(b, s);
  g_recs.push_back({kind, t_pending, b});
  t_pending = nullptr;
}

}  // namespace bdh

extern "C" {

int bdh_profile_begin(void) {
  std::lock_guard<std::mutex> lk(bdh::g_mu);
  for (auto& r : bdh::g_recs) {
    bdh::g_pool.push_back(r.a);
    bdh::g_pool.push_back(r.b);
  }
  bdh::g_recs.clear();
  bdh::g_on.store(true);
  return BDH_OK;
}

int bdh_profile_end(double ms[BDH_PROF_KINDS], int launches[BDH_PROF_KINDS]) {
  bdh::g_on.store(false);
  std::lock_guard<std::mutex> lk(bdh::g_mu);
  for (int k = 0; k < BDH_PROF_KINDS; ++k) {
    ms[k] = 0.0;
    launches[k] = 0;
  }
  for (auto& r : bdh::g_recs) {
    float t = 0.f;
    if (cudaEventSynchronize(r.b) != cudaSuccess || cudaEventElapsedTime(&t, r.a, r.b) != cudaSuccess) {
      bdh::set_error("bdh_profile_end: event timing failed");
      return BDH_ERR_CUDA;
    }
    if (r.kind >= 0 && r.kind < BDH_PROF_KINDS) {
      ms[r.kind] += t;
      launches[r.kind] += 1;
    }
  }
  return BDH_OK;
}

}  // extern "C"
