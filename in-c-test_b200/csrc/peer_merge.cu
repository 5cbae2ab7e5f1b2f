// peer_merge.cu -- split-KV combine across the GPUs of one node in one kernel
// per GPU (plain peer stores over NVLink, no multicast, no NCCL):
//   kvl_mla_attend_bf16_exchange  attend this rank's KV range, then one kernel
//                                 per (sequence, head, 128-wide slice) combines
//                                 the attend's partials locally, exchanges the
//                                 slice with every peer and merges the world
//                                 slices;
//   kvl_mla_merge_exchange        the same exchange and merge for a caller that
//                                 already holds its packed (o, lse) record.
// Values travel as tagged words: every value is one 64-bit store of
// (call number << 32 | float bits), which a reader sees whole or not at all,
// so a reader polls the words it needs in its own buffer until they carry the
// current call's tag; no fence or flag round trip is needed.
//
// Exchange buffer of each GPU (cudaMalloc, shared with the peers through CUDA
// IPC handles; layout in peer_merge.cuh).  Call k uses set k & 1 and tag k; a
// rank can run at most one call ahead of a peer (its call k + 1 ends only after
// reading that peer's words of call k + 1, stored only after the peer's call k
// has merged), so the set it overwrites is never being read.  Every wait is
// bounded (2 s); a timeout sets the group's error word
// (kvl_mla_peer_group_check) and skips the merge.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>

#include "kvl/mla_cuda.h"
#include "merge_core.cuh"
#include "peer_merge.cuh"
#include "prof.cuh"
#include "sm100.cuh"

#define KVL_EXPORT extern "C" __attribute__((visibility("default")))

namespace kvl {
void set_error_text(const char *msg);  // mla_capi.cu

namespace {

constexpr int kMaxWorld = kPeerMaxWorld;
constexpr int kMaxRows = kPeerMaxRows;

__device__ __forceinline__ void st_tagged(unsigned long long *p, unsigned long long tag, float v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(tag | __float_as_uint(v)) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Grid (sequence b, head h, 128-wide slice z of R), 256 threads: combine this
// GPU's partials of (b, h, z) exactly as merge_partials_kernel does (or, for a
// sequence that is not split, read its result from the record), store the slice and the lse as
// tagged words into slot (set, rank, b, h) of every other GPU's buffer, poll
// this GPU's buffer until every peer's words of (b, h, z) carry the call's tag,
// and combine the world slices in rank order (so every GPU computes the same
// bits).  No block waits for another block of its own grid, only for its
// counterparts on the peers, which store before they wait; where the grid
// (up to 256 (b, h) pairs x 4 slices) exceeds what is resident at once, the
// lowest-numbered blocks of every GPU are resident together and finish first.
struct AttendExchangeArgs {
  unsigned long long *bufs[kMaxWorld];
  int rank, world, set;
  uint32_t epoch;
  int batch, nh, R;
  long long slot;                   // words per (set, rank, b, h) slot: R data + lse + pad
  const float *part_o, *part_lse;   // the plan's partials [P][nh][R], [P][nh]
  const MergeEntry *entries;        // split sequences (device), n_entries of them
  int n_entries;
  const float *rec_o, *rec_lse;     // the other sequences: [batch][nh][R], [batch][nh]
};

constexpr int kXThreads = 256;

__global__ void __launch_bounds__(kXThreads)
    attend_exchange_kernel(const __grid_constant__ AttendExchangeArgs a, float *out, float *lse, uint32_t *err) {
  const int b = blockIdx.x, h = blockIdx.y, z = blockIdx.z, R = a.R;
  const int lane = threadIdx.x & 31;
  // the attend grid's partials must be complete (this kernel is its programmatic dependent)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int ei = -1;
  for (int i = 0; i < a.n_entries; ++i)
    if (a.entries[i].seq == b) ei = i;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  float row_lse;
  const int d0 = z * 128 + 4 * lane;  // this lane's elements d0 .. d0 + 3 (R is a multiple of 128)
  if (ei >= 0) {
    const MergeSlice r = merge_slice(a.entries[ei], h, z, a.part_o, a.part_lse, a.nh, R, 1,
                                     static_cast<long long>(a.nh) * R, a.nh, true);
    const float inv = 1.0f / r.sum;
    v = make_float4(r.t.x * inv, r.t.y * inv, r.t.z * inv, r.t.w * inv);
    row_lse = r.m + logf(r.sum);
  } else {
    const long long bh = static_cast<long long>(b) * a.nh + h;
    if (threadIdx.x < 32) v = *reinterpret_cast<const float4 *>(a.rec_o + bh * R + d0);
    row_lse = a.rec_lse[bh];
  }
  if (threadIdx.x >= 32) return;
  // Word j * 32 + lane of the slice holds element d0 + j, so each store
  // instruction of the warp writes 256 contiguous bytes; word R holds the lse.
  const unsigned long long tag = static_cast<unsigned long long>(a.epoch) << 32;
  auto slot_of = [&](const unsigned long long *buf, int r) {
    return buf + (((static_cast<long long>(a.set) * a.world + r) * a.batch + b) * a.nh + h) * a.slot;
  };
  for (int p = 0; p < a.world; ++p) {
    if (p == a.rank) continue;
    unsigned long long *dst = const_cast<unsigned long long *>(slot_of(a.bufs[p], a.rank));
    st_tagged(dst + z * 128 + lane, tag, v.x);
    st_tagged(dst + z * 128 + 32 + lane, tag, v.y);
    st_tagged(dst + z * 128 + 64 + lane, tag, v.z);
    st_tagged(dst + z * 128 + 96 + lane, tag, v.w);
    if (lane == 0) st_tagged(dst + R, tag, row_lse);  // every slice stores the same value
  }
  // wait until every peer's words of this lane carry the tag
  const unsigned long long *mine = a.bufs[a.rank];
  bool ok = true;
  for (int r = 0; r < a.world && ok; ++r) {
    if (r == a.rank) continue;
    const unsigned long long *src = slot_of(mine, r);
    const uint64_t t0 = globaltimer();
    while (true) {
      const unsigned long long w0 = ld_tagged(src + z * 128 + lane), w1 = ld_tagged(src + z * 128 + 32 + lane),
                               w2 = ld_tagged(src + z * 128 + 64 + lane), w3 = ld_tagged(src + z * 128 + 96 + lane),
                               wl = ld_tagged(src + R);
      if (((w0 & w1 & w2 & w3 & wl) >> 32) == a.epoch && ((w0 | w1 | w2 | w3 | wl) >> 32) == a.epoch) break;
      if (globaltimer() - t0 > KVL_WAIT_LIMIT_NS) {
        atomicOr(err, ERR_TIMEOUT_FULL);
        ok = false;
        break;
      }
    }
  }
  if (!__all_sync(0xffffffffu, ok)) return;
  auto val = [](unsigned long long w) { return __uint_as_float(static_cast<uint32_t>(w)); };
  float mm = -INFINITY;
  for (int r = 0; r < a.world; ++r) mm = fmaxf(mm, r == a.rank ? row_lse : val(ld_tagged(slot_of(mine, r) + R)));
  float ss = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < a.world; ++r) {
    float4 u = v;
    float lr = row_lse;
    if (r != a.rank) {
      const unsigned long long *src = slot_of(mine, r);
      u = make_float4(val(ld_tagged(src + z * 128 + lane)), val(ld_tagged(src + z * 128 + 32 + lane)),
                      val(ld_tagged(src + z * 128 + 64 + lane)), val(ld_tagged(src + z * 128 + 96 + lane)));
      lr = val(ld_tagged(src + R));
    }
    const float w = expf(lr - mm);
    ss += w;
    acc.x = fmaf(w, u.x, acc.x);
    acc.y = fmaf(w, u.y, acc.y);
    acc.z = fmaf(w, u.z, acc.z);
    acc.w = fmaf(w, u.w, acc.w);
  }
  const float inv = 1.0f / ss;
  *reinterpret_cast<float4 *>(out + (static_cast<long long>(b) * a.nh + h) * R + d0) =
      make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  if (lse && z == 0 && lane == 0) lse[b * a.nh + h] = mm + logf(ss);
}

}  // namespace

namespace {
cudaError_t launch_exchange(KvlMlaPeerGroup *g, const MergeEntry *entries, int n_entries, const float *part_o,
                            const float *part_lse, const float *rec_o, const float *rec_lse, float *d_out,
                            float *d_lse, cudaStream_t stream) {
  AttendExchangeArgs a;
  memset(&a, 0, sizeof a);
  for (int r = 0; r < g->world; ++r) a.bufs[r] = reinterpret_cast<unsigned long long *>(g->peers[r]);
  // The tag of a call is its 32-bit number.  Buffers start zeroed, so tag 0
  // would match words nobody wrote: on wrap-around the count skips 0 and 1 and
  // resumes at 2, which keeps the two buffer sets alternating (set = epoch & 1).
  if (++g->epoch == 0u) g->epoch = 2u;
  a.rank = g->rank;
  a.world = g->world;
  a.set = static_cast<int>(g->epoch & 1u);
  a.epoch = g->epoch;
  a.batch = g->batch;
  a.nh = g->nh;
  a.R = g->R;
  a.slot = peer_tagged_slot_words(g->R);
  a.part_o = part_o;
  a.part_lse = part_lse;
  a.entries = entries;
  a.n_entries = n_entries;
  a.rec_o = rec_o;
  a.rec_lse = rec_lse;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g->batch, g->nh, g->R / 128);
  cfg.blockDim = dim3(kXThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ProfScope ps(n_entries ? "attend_exchange" : "merge_exchange", stream);
  return cudaLaunchKernelEx(&cfg, attend_exchange_kernel, a, d_out, d_lse, g->err);
}
}  // namespace

cudaError_t launch_attend_exchange(KvlMlaPeerGroup *g, const DevicePlan &dp, float *d_out, float *d_lse,
                                   cudaStream_t stream) {
  return launch_exchange(
      g, reinterpret_cast<const MergeEntry *>(static_cast<const uint8_t *>(dp.d_meta) + dp.off_merge),
      static_cast<int>(dp.host.merges.size()), dp.part_o, dp.part_lse, g->stage,
      g->stage + static_cast<long long>(g->batch) * g->nh * g->R, d_out, d_lse, stream);
}

}  // namespace kvl

namespace {
void peer_err(const char *what, cudaError_t e) {
  char buf[256];
  snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
  kvl::set_error_text(buf);
}
}  // namespace

KVL_EXPORT size_t kvl_mla_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

KVL_EXPORT int kvl_mla_peer_group_create(KvlMlaPeerGroup **group, int rank, int world, int batch, int num_heads,
                                         int kv_lora_rank, void *handle_out) {
  if (!group || !handle_out || world < 2 || world > kvl::kMaxWorld || rank < 0 || rank >= world || batch <= 0 ||
      num_heads <= 0 || kv_lora_rank <= 0 || kv_lora_rank % 128 != 0 || batch * num_heads > kvl::kMaxRows) {
    kvl::set_error_text("invalid peer group arguments");
    return -1;
  }
  KvlMlaPeerGroup *g = new KvlMlaPeerGroup();
  cudaGetDevice(&g->device);
  g->rank = rank;
  g->world = world;
  g->batch = batch;
  g->nh = num_heads;
  g->R = kv_lora_rank;
  g->rec = static_cast<long long>(batch) * num_heads * (kv_lora_rank + 1);
  const size_t bytes = kvl::peer_buffer_bytes(world, batch, num_heads, kv_lora_rank);
  cudaError_t e = cudaMalloc(&g->local, bytes);
  if (e == cudaSuccess) e = cudaMemset(g->local, 0, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&g->stage, g->rec * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&g->err, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(g->err, 0, sizeof(uint32_t));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->local);
  if (e != cudaSuccess) {
    peer_err("peer group create", e);
    cudaFree(g->local);
    cudaFree(g->stage);
    cudaFree(g->err);
    delete g;
    return -1;
  }
  memcpy(handle_out, &h, sizeof h);
  g->peers[rank] = g->local;
  *group = g;
  return 0;
}

KVL_EXPORT int kvl_mla_peer_group_connect(KvlMlaPeerGroup *g, const void *handles) {
  if (!g || !handles || g->connected) {
    kvl::set_error_text("invalid peer group connect");
    return -1;
  }
  cudaSetDevice(g->device);
  for (int r = 0; r < g->world; ++r) {
    if (r == g->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t *>(handles) + r * sizeof h, sizeof h);
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      peer_err("peer group connect (cudaIpcOpenMemHandle)", e);
      for (int q = 0; q < r; ++q)
        if (q != g->rank && g->peers[q]) cudaIpcCloseMemHandle(g->peers[q]);
      return -1;
    }
    g->peers[r] = static_cast<float *>(p);
  }
  g->connected = true;
  return 0;
}

KVL_EXPORT int kvl_mla_merge_exchange(KvlMlaPeerGroup *g, float *d_out, float *d_lse, const float *d_record,
                                      void *stream) {
  if (!g || !g->connected || !d_out || !d_record ||
      ((reinterpret_cast<uintptr_t>(d_out) | reinterpret_cast<uintptr_t>(d_record)) & 15) != 0) {
    kvl::set_error_text("invalid merge exchange arguments (d_out and d_record 16-byte aligned)");
    return -1;
  }
  const cudaError_t e =
      kvl::launch_exchange(g, nullptr, 0, nullptr, nullptr, d_record,
                           d_record + static_cast<long long>(g->batch) * g->nh * g->R, d_out, d_lse,
                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    peer_err("merge exchange launch", e);
    return -1;
  }
  return 0;
}

KVL_EXPORT int kvl_mla_peer_group_check(KvlMlaPeerGroup *g, void *stream) {
  if (!g) return -1;
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return -1;
  uint32_t err = 0;
  if (cudaMemcpy(&err, g->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (err) {
    cudaMemset(g->err, 0, 4);
    char buf[96];
    snprintf(buf, sizeof buf, "merge exchange: a peer's record did not arrive in time (0x%x)", err);
    kvl::set_error_text(buf);
    return -1;
  }
  return 0;
}

KVL_EXPORT void kvl_mla_peer_group_destroy(KvlMlaPeerGroup *g) {
  if (!g) return;
  cudaSetDevice(g->device);
  for (int r = 0; r < g->world; ++r)
    if (r != g->rank && g->peers[r]) cudaIpcCloseMemHandle(g->peers[r]);
  cudaFree(g->local);
  cudaFree(g->stage);
  cudaFree(g->err);
  delete g;
}
