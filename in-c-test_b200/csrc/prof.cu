// prof.cu -- see prof.cuh.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "prof.cuh"

#define KVL_EXPORT extern "C" __attribute__((visibility("default")))

namespace kvl {

cudaError_t smem_opt_in(const void *fn, int bytes, std::atomic<unsigned long long> &done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

namespace {

struct Rec {
  std::string name;
  cudaEvent_t a = nullptr, b = nullptr;
};

std::atomic<bool> g_on{false};
std::mutex g_mu;
std::vector<Rec> g_pending;
std::vector<cudaEvent_t> g_free;
std::map<std::string, std::pair<double, long long>> g_acc;  // ms, launches

cudaEvent_t take_event() {
  if (!g_free.empty()) {
    cudaEvent_t e = g_free.back();
    g_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void collect_locked() {
  for (Rec &r : g_pending) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      auto &acc = g_acc[r.name];
      acc.first += ms;
      acc.second += 1;
    }
    g_free.push_back(r.a);
    g_free.push_back(r.b);
  }
  g_pending.clear();
}

}  // namespace

bool prof_enabled() { return g_on.load(std::memory_order_relaxed); }

int prof_begin(const char *name, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_pending.size() > 100000) collect_locked();
  Rec r;
  r.name = name;
  r.a = take_event();
  r.b = take_event();
  if (!r.a || !r.b) return -1;
  cudaEventRecord(r.a, s);
  g_pending.push_back(r);
  return static_cast<int>(g_pending.size()) - 1;
}

void prof_end(int id, cudaStream_t s) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (id >= 0 && id < static_cast<int>(g_pending.size())) cudaEventRecord(g_pending[id].b, s);
}

}  // namespace kvl

using namespace kvl;

// Enables (1) or disables (0) per-kernel timing; enabling clears the totals.
KVL_EXPORT int kvl_mla_cuda_profile(int enable) {
  std::lock_guard<std::mutex> lk(g_mu);
  const int prev = g_on.load() ? 1 : 0;
  if (enable) {
    collect_locked();
    g_acc.clear();
  }
  g_on.store(enable != 0);
  return prev;
}

// Waits for the recorded launches and writes up to `max_entries` lines
// "name,total_ms,launches\n" into `buf` (NUL-terminated).  Returns the number
// of kernels, or -1 if `buf` is too small.
KVL_EXPORT int kvl_mla_cuda_profile_read(char *buf, size_t cap) {
  std::lock_guard<std::mutex> lk(g_mu);
  collect_locked();
  std::string s;
  for (auto &kv : g_acc) {
    char line[256];
    snprintf(line, sizeof line, "%s,%.6f,%lld\n", kv.first.c_str(), kv.second.first, kv.second.second);
    s += line;
  }
  if (!buf || s.size() + 1 > cap) return -1;
  memcpy(buf, s.c_str(), s.size() + 1);
  return static_cast<int>(g_acc.size());
}
