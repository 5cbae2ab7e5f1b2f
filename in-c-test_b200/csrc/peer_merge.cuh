// peer_merge.cuh -- the peer group of the cross-GPU split-KV combine
// (peer_merge.cu) and the fused attend + combine launcher used by mla_capi.cu.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "attend_host.cuh"

namespace kvl {
constexpr int kPeerMaxWorld = 8;
constexpr int kPeerMaxRows = 256;  // batch * num_heads

// Exchange buffer of every rank: tagged slots [2 sets][world][batch][nh] of
// peer_tagged_slot_words(R) u64 words -- R words of (call << 32 | float bits)
// (word j * 32 + l of slice z holds element 128 z + 4 l + j), then the lse word,
// then one pad word.  R is a multiple of 128.
inline long long peer_tagged_slot_words(int R) { return R + 2LL; }
inline size_t peer_buffer_bytes(int world, int batch, int nh, int R) {
  return 2ull * world * batch * nh * peer_tagged_slot_words(R) * sizeof(unsigned long long);
}
}  // namespace kvl

struct KvlMlaPeerGroup {
  int device = 0, rank = 0, world = 0, batch = 0, nh = 0, R = 0;
  long long rec = 0;  // floats of one packed record: batch * nh * (R + 1)
  float *local = nullptr;
  float *peers[kvl::kPeerMaxWorld] = {};
  uint32_t *err = nullptr;
  float *stage = nullptr;  // this rank's [batch][nh][R] ++ [batch][nh] staging record
  uint32_t epoch = 0;
  bool connected = false;
};

namespace kvl {
// The partials of an attend launched with skip_merge (plan dp), combined per
// (sequence, head) on this GPU and then across the group's GPUs into d_out /
// d_lse.  Unsplit sequences are read from g->stage (where the attend wrote them).
cudaError_t launch_attend_exchange(KvlMlaPeerGroup *g, const DevicePlan &dp, float *d_out, float *d_lse,
                                   cudaStream_t stream);
}  // namespace kvl
