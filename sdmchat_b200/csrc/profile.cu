// Launch accounting and the event-based launch profiler behind sdm_kernel_launch_count / sdm_profile_*.
// Host code only.  Recording is off unless sdm_profile_begin() was called; then every launch is bracketed by two
// CUDA events on its own stream (a few microseconds of host time, no device memory).
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>
#include "kernels.cuh"

namespace sdm {

namespace {
std::atomic<int64_t> g_launches{0};
std::mutex g_mu;
bool g_recording = false;
thread_local const char* g_tag = "";

struct Rec {
  const char* kernel;
  const char* tag;
  cudaEvent_t a, b;
};
std::vector<Rec> g_recs;
std::vector<cudaEvent_t> g_pool;
size_t g_pool_used = 0;

struct Group {
  std::string kernel, tag;
  int launches;
  double ms;
};
std::vector<Group> g_groups;

cudaEvent_t take_event() {
  if (g_pool_used == g_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    g_pool.push_back(e);
  }
  return g_pool[g_pool_used++];
}
}  // namespace

LaunchScope::LaunchScope(const char* kernel, cudaStream_t st) : rec_(-1), st_(st) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_recording) return;
  cudaEvent_t a = take_event(), b = take_event();
  if (!a || !b) return;
  cudaEventRecord(a, st);
  g_recs.push_back({kernel, g_tag, a, b});
  rec_ = (int)g_recs.size() - 1;
}

LaunchScope::~LaunchScope() {
  if (rec_ < 0) return;
  std::lock_guard<std::mutex> lk(g_mu);
  if (rec_ < (int)g_recs.size()) cudaEventRecord(g_recs[rec_].b, st_);
}

OpTag::OpTag(const char* tag) : prev_(g_tag) { g_tag = tag; }
OpTag::~OpTag() { g_tag = prev_; }

}  // namespace sdm

using namespace sdm;

extern "C" {

int64_t sdm_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

sdm_status sdm_profile_begin(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_recs.clear();
  g_groups.clear();
  g_pool_used = 0;
  g_recording = true;
  return SDM_OK;
}

int sdm_profile_end(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_recording = false;
  g_groups.clear();
  for (const Rec& r : g_recs) {
    if (cudaEventSynchronize(r.b) != cudaSuccess) return -1;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) return -1;
    bool found = false;
    for (Group& g : g_groups) {
      if (g.kernel == r.kernel && g.tag == r.tag) {
        g.launches += 1;
        g.ms += ms;
        found = true;
        break;
      }
    }
    if (!found) g_groups.push_back({r.kernel, r.tag, 1, (double)ms});
  }
  g_recs.clear();
  return (int)g_groups.size();
}

sdm_status sdm_profile_group(int i, char* kernel, char* tag, int name_len, int* launches, double* total_ms) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (i < 0 || i >= (int)g_groups.size() || !kernel || !tag || name_len < 2 || !launches || !total_ms)
    return SDM_ERR_ARG;
  const Group& g = g_groups[i];
  std::strncpy(kernel, g.kernel.c_str(), name_len - 1);
  kernel[name_len - 1] = 0;
  std::strncpy(tag, g.tag.c_str(), name_len - 1);
  tag[name_len - 1] = 0;
  *launches = g.launches;
  *total_ms = g.ms;
  return SDM_OK;
}

}  // extern "C"
