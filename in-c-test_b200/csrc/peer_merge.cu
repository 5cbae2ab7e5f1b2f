// peer_merge.cu -- split-KV combine across the GPUs of one node in one kernel:
// every GPU stores its packed partial record (o [B][nh][R] ++ lse [B][nh]) into
// slot `rank` of every GPU's exchange buffer over NVLink (plain peer stores,
// no multicast), raises a flag in each, waits for the flags of all ranks in
// its own buffer, and merges the `world` records -- the NCCL all-gather plus
// merge launch of the split-KV decode (config 5) as one launch.
//
// Exchange buffer of each GPU (cudaMalloc, shared with the peers through CUDA
// IPC handles): 2 sets x world records of rec = B*nh*(R+1) floats, then flags
// [2][world] uint32.  Call k uses set k & 1 and writes flag value k; a rank can
// run at most one call ahead of a peer (call k + 1 waits for that peer's flag
// of call k + 1, written only after the peer's call k has merged), so the set
// it overwrites is never being read.  Every wait is bounded (2 s); a timeout
// sets the group's error word (kvl_mla_peer_group_check) and skips the merge.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "kvl/mla_cuda.h"
#include "prof.cuh"
#include "sm100.cuh"

#define KVL_EXPORT extern "C" __attribute__((visibility("default")))

namespace kvl {
void set_error_text(const char *msg);  // mla_capi.cu

namespace {

constexpr int kMaxWorld = 8;
constexpr int kMaxRows = 256;  // batch * num_heads per record
constexpr int kThreads = 1024;

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerArgs {
  float *bufs[kMaxWorld];  // every rank's exchange buffer (this rank's own included)
  int rank, world, set;
  uint32_t epoch;
  long long rec;           // floats per record
  int batch, nh, R;
};

__global__ void __launch_bounds__(kThreads, 1)
    peer_exchange_merge_kernel(const __grid_constant__ PeerArgs a, const float *record, float *out, float *lse,
                               uint32_t *err) {
  __shared__ int timed_out;
  if (threadIdx.x == 0) timed_out = 0;
  const long long rec = a.rec;
  // 1. this rank's record into slot `rank` of every buffer
  const bool vec = (rec & 3) == 0 && (reinterpret_cast<uintptr_t>(record) & 15) == 0;
  for (int p = 0; p < a.world; ++p) {
    float *dst = a.bufs[p] + (static_cast<long long>(a.set) * a.world + a.rank) * rec;
    if (vec) {
      for (long long i = threadIdx.x; i < rec / 4; i += blockDim.x)
        reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(record)[i];
    } else {
      for (long long i = threadIdx.x; i < rec; i += blockDim.x) dst[i] = record[i];
    }
  }
  // 2. flag `rank` of the current set in every buffer: the barrier orders every
  // thread's record stores before thread 0's system-scope fence, which orders
  // them before the flag stores (release is cumulative)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < a.world; ++p) {
      uint32_t *flags = reinterpret_cast<uint32_t *>(a.bufs[p] + 2LL * a.world * rec);
      st_release_sys(flags + a.set * a.world + a.rank, a.epoch);
    }
  }
  // 3. wait for every rank's flag in this buffer
  if (threadIdx.x < a.world) {
    const uint32_t *flags = reinterpret_cast<const uint32_t *>(a.bufs[a.rank] + 2LL * a.world * rec);
    const uint32_t *f = flags + a.set * a.world + threadIdx.x;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) != a.epoch) {
      if (globaltimer() - t0 > KVL_WAIT_LIMIT_NS) {
        atomicOr(err, ERR_TIMEOUT_FULL);
        timed_out = 1;
        break;
      }
    }
  }
  // the waiting threads' acquire loads, then the barrier, order the records
  // before every thread's reads below
  __syncthreads();
  if (timed_out) return;
  // 4. combine the world records: o = sum_r w_r o_r / sum_r w_r, w_r = exp(lse_r - max),
  // the weights once per (sequence, head) in shared memory, the outputs in float4
  __shared__ float sw[kMaxWorld * kMaxRows];
  __shared__ float sinv[kMaxRows];
  const float *base = a.bufs[a.rank] + static_cast<long long>(a.set) * a.world * rec;
  const int rows = a.batch * a.nh;  // (sequence, head) pairs, <= kMaxRows (checked at create)
  const long long olen = static_cast<long long>(rows) * a.R;
  for (int bh = threadIdx.x; bh < rows; bh += blockDim.x) {
    float m = -INFINITY;
    for (int r = 0; r < a.world; ++r) m = fmaxf(m, base[r * rec + olen + bh]);
    float sum = 0.f;
    for (int r = 0; r < a.world; ++r) {
      const float w = expf(base[r * rec + olen + bh] - m);
      sw[r * kMaxRows + bh] = w;
      sum += w;
    }
    sinv[bh] = 1.0f / sum;
    if (lse) lse[bh] = m + logf(sum);
  }
  __syncthreads();
  if ((a.R & 3) == 0 && (rec & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
    for (long long i4 = threadIdx.x; i4 < olen / 4; i4 += blockDim.x) {
      const int bh = static_cast<int>((4 * i4) / a.R);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < a.world; ++r) {
        const float w = sw[r * kMaxRows + bh];
        const float4 v = reinterpret_cast<const float4 *>(base + r * rec)[i4];
        acc.x = fmaf(w, v.x, acc.x);
        acc.y = fmaf(w, v.y, acc.y);
        acc.z = fmaf(w, v.z, acc.z);
        acc.w = fmaf(w, v.w, acc.w);
      }
      const float inv = sinv[bh];
      reinterpret_cast<float4 *>(out)[i4] = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
  } else {
    for (long long i = threadIdx.x; i < olen; i += blockDim.x) {
      const int bh = static_cast<int>(i / a.R);
      float acc = 0.f;
      for (int r = 0; r < a.world; ++r) acc = fmaf(sw[r * kMaxRows + bh], base[r * rec + i], acc);
      out[i] = acc * sinv[bh];
    }
  }
}

}  // namespace
}  // namespace kvl

struct KvlMlaPeerGroup {
  int device = 0, rank = 0, world = 0, batch = 0, nh = 0, R = 0;
  long long rec = 0;
  float *local = nullptr;
  float *peers[kvl::kMaxWorld] = {};
  uint32_t *err = nullptr;
  uint32_t epoch = 0;
  bool connected = false;
};

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
      num_heads <= 0 || kv_lora_rank <= 0 || batch * num_heads > kvl::kMaxRows) {
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
  const size_t bytes = (2ull * world * g->rec) * sizeof(float) + 2ull * world * sizeof(uint32_t);
  cudaError_t e = cudaMalloc(&g->local, bytes);
  if (e == cudaSuccess) e = cudaMemset(g->local, 0, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&g->err, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(g->err, 0, sizeof(uint32_t));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->local);
  if (e != cudaSuccess) {
    peer_err("peer group create", e);
    cudaFree(g->local);
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
  if (!g || !g->connected || !d_out || !d_record) {
    kvl::set_error_text("invalid merge exchange arguments");
    return -1;
  }
  kvl::PeerArgs a;
  memset(&a, 0, sizeof a);
  for (int r = 0; r < g->world; ++r) a.bufs[r] = g->peers[r];
  ++g->epoch;
  a.rank = g->rank;
  a.world = g->world;
  a.set = static_cast<int>(g->epoch & 1u);
  a.epoch = g->epoch;
  a.rec = g->rec;
  a.batch = g->batch;
  a.nh = g->nh;
  a.R = g->R;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  kvl::ProfScope ps("merge_exchange", s);
  kvl::peer_exchange_merge_kernel<<<1, kvl::kThreads, 0, s>>>(a, d_record, d_out, d_lse, g->err);
  const cudaError_t e = cudaGetLastError();
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
  cudaFree(g->err);
  delete g;
}
