// attend_noalloc.cu -- kvl_mla_attend_bf16_noalloc: the single-sequence
// split-KV decode attend (the tcgen05 kernel of attend_bf16.cu plus the
// partial merge) with every byte of its scratch -- the work plan, the
// per-range partial outputs, the query image and the device error word -- in a
// file-scope
// device array instead of memory allocated at call time.
//
// It exists for callers that cannot allocate device memory when they decode:
// a runtime that reserves its whole device-memory budget up front and must not
// have a library allocate behind it, or a decode loop that must not stall on
// cudaMalloc, which can synchronise the device and can fail once memory is
// fragmented.  The caller passes the inputs and outputs; the call itself
// performs no cudaMalloc, cudaFree or other allocating library routine.
//
// Limits and sharing:
//   * one sequence per call, split over at most kNoAllocMaxSplits (148) KV
//     ranges; the scratch is 4.9 MB and every GPU that loads the library keeps
//     it until the process exits;
//   * all calls share the one array, which keeps the last call's contents:
//     the device plan and the error word are rewritten at the start of every
//     call, and each call reads only the partials it wrote.  Calls that
//     overlap on the GPU (different streams or host threads, same device) race
//     on the array and must be serialised by the caller;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, once per device, with that device current);
//   * the call is synchronous: it returns once `stream` has finished the
//     attend and the error word is back on the host, so it cannot be captured
//     into a CUDA graph.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "attend_common.cuh"
#include "attend_host.cuh"
#include "kvl/mla_cuda.h"

#define KVL_EXPORT extern "C" __attribute__((visibility("default")))

namespace kvl {

cudaError_t launch_attend_bf16_unprofiled(const AttendParams &p, int grid, int batch, bool qprep,
                                         cudaStream_t stream);
cudaError_t launch_merge_unprofiled(float *out, float *lse, const float *part_o, const float *part_lse,
                                   const MergeEntry *d_entries, int n_entries, int nh, int R,
                                   cudaStream_t stream, int max_count);
void set_error_text(const char *msg);

namespace {

constexpr int kNoAllocMaxSplits = 148;

struct NoAllocPlan {
  AttendSegment segs[kNoAllocMaxSplits];
  int cta_seg[kNoAllocMaxSplits + 1];
  long long row0;
  MergeEntry merge;
  uint32_t err;
};

constexpr size_t kPlanBytes = (sizeof(NoAllocPlan) + 255) & ~size_t(255);
constexpr size_t kPartOBytes = size_t(kNoAllocMaxSplits) * kHeads * kLatent * sizeof(float);
constexpr size_t kPartLseBytes = (size_t(kNoAllocMaxSplits) * kHeads * sizeof(float) + 255) & ~size_t(255);
constexpr size_t kScratchBytes = kPlanBytes + kPartOBytes + kPartLseBytes + kQImgStride;

}  // namespace

// The scratch.  In host code this name is only a stand-in for the symbol: its
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices];

void fail(const char *fmt, long long a = 0, long long b = 0) {
  char buf[256];
  snprintf(buf, sizeof buf, fmt, a, b);
  set_error_text(buf);
}

// Device address of the scratch on `dev` (the current device); looked up once.
void *scratch_on(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) return nullptr;
    g_scratch_ptr[dev] = ptr;
  }
  return g_scratch_ptr[dev];
}

// Writes the plan of one sequence split into `splits` equal ranges of tiles
// (every range non-empty) and clears the error word.
__global__ void noalloc_plan_kernel(NoAllocPlan *plan, int seq_len, long long row0, int splits) {
  const long long tiles = (seq_len + kTileTok - 1) / kTileTok;
  for (int c = threadIdx.x; c < splits; c += blockDim.x) {
    const long long lo = tiles * c / splits, hi = tiles * (c + 1) / splits;
    AttendSegment s;
    s.seq = 0;
    s.row0 = row0;
    s.tok_begin = static_cast<int>(lo * kTileTok);
    s.tok_end = static_cast<int>(hi * kTileTok < seq_len ? hi * kTileTok : seq_len);
    s.slot = splits > 1 ? c : -1;
    plan->segs[c] = s;
    plan->cta_seg[c] = c;
  }
  if (threadIdx.x == 0) {
    plan->cta_seg[splits] = splits;
    plan->row0 = row0;
    plan->merge = MergeEntry{0, 0, splits, 1};
    plan->err = 0u;
  }
}

}  // namespace
}  // namespace kvl

using namespace kvl;

// Declared in include/kvl/mla_cuda.h.
KVL_EXPORT int kvl_mla_attend_bf16_noalloc(float *d_out, float *d_lse, const float *d_q, const uint16_t *d_kv,
                                           int64_t rows, int seq_len, int64_t seq_row0, int num_heads,
                                           int kv_lora_rank, int rope_dim, int splits, float softmax_scale,
                                           void *stream) {
  if (!d_out || !d_q || !d_kv) {
    fail("noalloc attend: null pointer argument");
    return -1;
  }
  if (num_heads != kHeads || kv_lora_rank != kLatent || rope_dim != kRope) {
    fail("noalloc attend: only the (16 heads, 512, 64) shape is supported");
    return -1;
  }
  if (seq_len <= 0 || seq_row0 < 0 || rows <= 0 || seq_row0 + seq_len > rows || rows >= (1LL << 31)) {
    fail("noalloc attend: bad sequence range (len %lld, first row %lld)", seq_len, seq_row0);
    return -1;
  }
  if (splits < 0 || splits > kNoAllocMaxSplits) {
    fail("noalloc attend: %lld splits requested; the scratch holds at most %lld", splits, kNoAllocMaxSplits);
    return -1;
  }
  if ((reinterpret_cast<uintptr_t>(d_kv) & 15) != 0) {
    fail("noalloc attend: kv pool must be 16-byte aligned");
    return -1;
  }
  if ((reinterpret_cast<uintptr_t>(d_q) & 15) != 0) {
    fail("noalloc attend: the absorbed query must be 16-byte aligned");
    return -1;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    fail("noalloc attend: no CUDA device");
    return -1;
  }
  uint8_t *scratch = static_cast<uint8_t *>(scratch_on(dev));
  if (!scratch) {
    fail("noalloc attend: cudaGetSymbolAddress of the scratch array failed on device %lld", dev);
    return -1;
  }
  if (splits == 0) {
    int sms = kNoAllocMaxSplits;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    splits = sms < kNoAllocMaxSplits ? sms : kNoAllocMaxSplits;
  }
  const long long tiles = (seq_len + kTileTok - 1) / kTileTok;
  if (splits > tiles) splits = static_cast<int>(tiles);

  NoAllocPlan *plan = reinterpret_cast<NoAllocPlan *>(scratch);
  float *part_o = reinterpret_cast<float *>(scratch + kPlanBytes);
  float *part_lse = reinterpret_cast<float *>(scratch + kPlanBytes + kPartOBytes);
  uint8_t *qimg = scratch + kPlanBytes + kPartOBytes + kPartLseBytes;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  AttendParams p;
  memset(&p, 0, sizeof p);
  if (!make_tmap_2d(&p.tm_kv, d_kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kRow, static_cast<uint64_t>(rows), kRow * 2,
                    64, kTileTok, CU_TENSOR_MAP_SWIZZLE_128B)) {
    fail("noalloc attend: tensor map encoding failed");
    return -1;
  }
  p.q = d_q;
  p.out = d_out;
  p.lse = d_lse;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.qimg = qimg;
  p.segs = plan->segs;
  p.cta_seg = plan->cta_seg;
  p.seq_row0 = &plan->row0;
  p.rows = rows;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = &plan->err;

  noalloc_plan_kernel<<<1, 160, 0, st>>>(plan, seq_len, seq_row0, splits);
  cudaError_t e = cudaGetLastError();
  // one segment per CTA: the kernel converts the query itself (no prep kernel)
  if (e == cudaSuccess) e = launch_attend_bf16_unprofiled(p, splits, 1, false, st);
  if (e == cudaSuccess && splits > 1)
    e = launch_merge_unprofiled(d_out, d_lse, part_o, part_lse, &plan->merge, 1, kHeads, kLatent, st, splits);
  // The error word comes back on the caller's stream, behind the kernels, so
  // the call waits for that stream alone (not for the legacy default stream or
  // other blocking streams of the device).
  uint32_t err = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&err, &plan->err, sizeof err, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    fail("noalloc attend: CUDA error %lld", static_cast<long long>(e));
    return -1;
  }
  if (err != 0) {
    fail("noalloc attend: kernel reported device error 0x%llx", err);
    return -1;
  }
  return 0;
}
