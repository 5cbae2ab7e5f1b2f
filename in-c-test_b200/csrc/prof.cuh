// prof.cuh -- optional per-kernel timing: when enabled, every kernel launch of
// the library is bracketed by CUDA events recorded on the launching stream, and
// kvl_mla_cuda_profile_read() reports the accumulated device time per kernel.
// Disabled (the default) it costs one relaxed atomic load per launch.
#pragma once
#include <cuda_runtime.h>

#include <atomic>

namespace kvl {

bool prof_enabled();
int prof_begin(const char *name, cudaStream_t s);  // returns a record id, or -1
void prof_end(int id, cudaStream_t s);

// Opts kernel `fn` into `bytes` of dynamic shared memory on the current device.
// The attribute belongs to each device's context, so it is set once per
// device: `done` holds one bit per device index (indices >= 64 set it on every
// launch).  Threads that race both set it, which is harmless.
cudaError_t smem_opt_in(const void *fn, int bytes, std::atomic<unsigned long long> &done);

struct ProfScope {
  int id;
  cudaStream_t s;
  // name == nullptr: never timed (launches that must not create events)
  ProfScope(const char *name, cudaStream_t st) : id(name && prof_enabled() ? prof_begin(name, st) : -1), s(st) {}
  ~ProfScope() {
    if (id >= 0) prof_end(id, s);
  }
};

}  // namespace kvl
