// attend_common.cuh -- shared definitions of the absorbed-MLA decode attend
// kernels (bf16 latent state and row-wise Q8 latent state).
//
// The attend core restated here is the inner part of the reference decode
// (src/mla_compressed_state.c:132-148, src/mla_compressed_q8_state.c:216-238):
// for every head h and cached row j
//     s_j   = (q_lat_h . latent_j + q_rope_h . rope_j) * scale
//     mix_h = sum_j softmax(s)_j * latent_j
// with all heads sharing one 576-wide cached row (512 latent + 64 rope).
//
// Work decomposition ("stream-K" over KV tiles): the KV rows of every sequence
// are cut into tiles of 128 rows; the concatenated tile list of the whole batch
// is split into equal contiguous ranges, one per CTA.  A CTA's range is a list
// of segments (one sequence each).  A segment that covers a whole sequence
// writes the normalised output directly; a piece of a split sequence writes a
// partial (o, lse) that the merge kernel combines.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#ifdef __CUDACC__
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#endif

namespace kvl {

constexpr int kHeads = 16;       // tcgen05 N (heads share one latent row)
constexpr int kLatent = 512;     // kv_lora_rank
constexpr int kRope = 64;        // qk_rope_dim
constexpr int kRow = kLatent + kRope;
// KV rows per tile = tcgen05 M of the score MMA.  A tcgen05.mma costs about
// the same (~48 cycles) at M=64 and M=128 when N is 16 (the heads), so 128
// rows per MMA halves the score-MMA count per cached row.
constexpr int kTileTok = 128;

struct AttendSegment {
  int seq;        // batch index
  int tok_begin;  // first KV row of the segment (tile aligned within the sequence)
  int tok_end;    // one past the last KV row
  int slot;       // partial slot, or -1 when the segment is the whole sequence
  long long row0; // pool row of the sequence's row 0 (so no role reads seq_row0 at a boundary)
};

// Query images.  Before the attend, a small kernel writes the absorbed query of
// every sequence in exactly the shared-memory layout the kernel's MMAs read;
// a loader warp then brings a segment's query in with one bulk copy instead of
// the softmax warps converting it at every segment start.
//   bf16 kernel: nine SW128 boxes of 16 heads x 64 dims bf16 (18432 B)
//   Q8 kernel:   int8 hi/lo parts [32][512] as four SW128 boxes (16384 B),
//                q_rope [16][64] bf16 as one SW128 box (2048 B), then the
//                per-head scale sq [16] fp32 (64 B)
constexpr uint32_t kQImgBf16Bytes = 9 * 2048;
constexpr uint32_t kQImgQ8Bytes = 4 * 4096 + 2048 + 64;
constexpr uint32_t kQImgStride = 18688;  // per sequence, a multiple of 256
static_assert(kQImgBf16Bytes <= kQImgStride && kQImgQ8Bytes <= kQImgStride, "query image stride");

struct AttendParams {
  CUtensorMap tm_kv;         // bf16 layout: [rows][576] (latent | rope)
  CUtensorMap tm_rope;       // q8 layout: rope bf16 [rows][64]
  CUtensorMap tm_lat8;       // q8 layout: latent int8 [rows][512]
  const float *latent_scale; // q8 layout: [rows]
  const float *q;            // [B][16][576] fp32 absorbed query (q_lat | q_rope)
  float *out;                // [B][16][512] fp32 normalised mix
  float *lse;                // [B][16] natural-log normaliser (may be null)
  float *part_o;             // [P][16][512]
  float *part_lse;           // [P][16]
  const AttendSegment *segs;
  const int *cta_seg;        // [grid + 1] segment ranges per CTA
  const long long *seq_row0; // [B] first pool row of each sequence
  const uint8_t *qimg;       // [B][kQImgStride] query images (written by the prep kernel)
  long long rows;            // rows in the pool
  float scale_log2;          // softmax scale * log2(e)
  uint32_t *err;             // error word (bit-or of kvl::ERR_*)
  int first_tile_alone;      // bf16 kernel: copies beyond a CTA's first tile wait for it to land
                             // (launches of few tiles per CTA, where the grid's first tiles all
                             // arrive in one burst)
  int q_after_wait;          // launched as a programmatic dependent of the kernel that writes q
                             // (a kernel that releases its dependents only after its own
                             // griddepcontrol.wait, so the KV rows are complete): the copies
                             // start at once, the first query is read after griddepcontrol.wait
};

#ifdef __CUDACC__
// Two floats as a packed bf16 pair (round to nearest even).
__device__ __forceinline__ uint32_t pack2_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&v);
}

// The fp32 absorbed query [16][576] of one sequence as nine SW128 boxes of
// bf16 (64 dims x 16 heads, 2 KB each), in two phases so that a caller can
// issue the loads, signal that they are in flight, and only then wait for
// them: query_tile_load issues every global load of thread tid (0..127) into
// v, query_tile_store converts and stores them.

constexpr int kQueryPer = kHeads * (kRow / 8) / 128;  // 9 chunks of 8 values per thread

__device__ __forceinline__ void query_tile_load(const float *qs, int tid, float4 (&v)[2 * kQueryPer]) {
#pragma unroll
  for (int i = 0; i < kQueryPer; ++i) {
    const int idx = tid + 128 * i;
    const int h = idx / (kRow / 8), c8 = idx % (kRow / 8);
    v[2 * i] = *reinterpret_cast<const float4 *>(qs + h * kRow + c8 * 8);
    v[2 * i + 1] = *reinterpret_cast<const float4 *>(qs + h * kRow + c8 * 8 + 4);
  }
}

__device__ __forceinline__ void query_tile_store(uint8_t *qd, int tid, const float4 (&v)[2 * kQueryPer]) {
#pragma unroll
  for (int i = 0; i < kQueryPer; ++i) {
    const int idx = tid + 128 * i;
    const int h = idx / (kRow / 8), c8 = idx % (kRow / 8);
    uint4 o;
    o.x = pack2_bf16(v[2 * i].x, v[2 * i].y);
    o.y = pack2_bf16(v[2 * i].z, v[2 * i].w);
    o.z = pack2_bf16(v[2 * i + 1].x, v[2 * i + 1].y);
    o.w = pack2_bf16(v[2 * i + 1].z, v[2 * i + 1].w);
    const uint32_t chunk = (c8 & 7) ^ (h & 7);  // 128-byte swizzle within the 16-row box
    *reinterpret_cast<uint4 *>(qd + (c8 >> 3) * 2048 + (h >> 3) * 1024 + (h & 7) * 128 + chunk * 16) = o;
  }
}

// Both phases at once.
__device__ __forceinline__ void load_query_tile(uint8_t *qd, const float *qs, int tid) {
  float4 v[2 * kQueryPer];
  query_tile_load(qs, tid, v);
  query_tile_store(qd, tid, v);
}
#endif

// Launches fn(p) -- a kernel taking one parameter struct -- as a programmatic
// dependent of the previous kernel on `stream`: it may start while that kernel
// drains, and must order its reads of that kernel's results with
// griddepcontrol.wait.
template <typename P>
inline cudaError_t launch_pdl(const void *fn, int grid, int threads, uint32_t smem, cudaStream_t stream, const P &p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *args[] = {const_cast<P *>(&p)};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace kvl
