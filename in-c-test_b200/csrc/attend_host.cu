// attend_host.cu -- host half of the decode attend path: TMA descriptor
// encoding, the stream-K work plan, the partial (o, lse) merge kernel, and the
// generic attend kernel used for head shapes the tcgen05 kernel does not cover
// (tiny test configurations such as the reference probes' NH=2, R=6).
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "attend_common.cuh"
#include "attend_host.cuh"
#include "merge_core.cuh"
#include "sm100.cuh"
#include "prof.cuh"

namespace kvl {

cudaError_t launch_attend_bf16(const AttendParams &p, int grid, int batch, bool qprep, cudaStream_t stream);
cudaError_t launch_attend_q8(const AttendParams &p, int grid, int batch, bool qprep, cudaStream_t stream);

// ------------------------------------------------------------------ TMA maps
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

bool make_tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, uint64_t inner,
                  uint64_t rows, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, const uint64_t dims[3],
                  const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t s[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t e[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void *>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------------ plan
int build_attend_plan(HostPlan &hp, int batch, const int *seq_len, const long long *seq_row0,
                      int max_ctas) {
  if (batch <= 0 || !seq_len || !seq_row0 || max_ctas <= 0) return -1;
  hp = HostPlan();
  hp.batch = batch;
  std::vector<long long> tiles(batch);
  long long total = 0;
  for (int b = 0; b < batch; ++b) {
    if (seq_len[b] <= 0 || seq_row0[b] < 0) return -1;
    tiles[b] = (seq_len[b] + kTileTok - 1) / kTileTok;
    total += tiles[b];
  }
  const int grid = static_cast<int>(std::min<long long>(max_ctas, total));
  hp.grid = grid;
  hp.cta_seg.assign(grid + 1, 0);
  hp.seq_row0.assign(seq_row0, seq_row0 + batch);
  hp.seq_len.assign(seq_len, seq_len + batch);
  std::vector<int> first_slot(batch, -1), nslot(batch, 0);
  int b = 0;
  long long ob = 0;  // tiles of sequence b already assigned
  for (int c = 0; c < grid; ++c) {
    hp.cta_seg[c] = static_cast<int>(hp.segs.size());
    long long remaining = (total * (c + 1)) / grid - (total * c) / grid;
    while (remaining > 0) {
      const long long take = std::min(remaining, tiles[b] - ob);
      AttendSegment s;
      s.seq = b;
      s.row0 = seq_row0[b];
      s.tok_begin = static_cast<int>(ob * kTileTok);
      s.tok_end = static_cast<int>(std::min<long long>((ob + take) * kTileTok, seq_len[b]));
      const bool whole = (ob == 0 && take == tiles[b]);
      if (whole) {
        s.slot = -1;
      } else {
        s.slot = hp.nparts++;
        if (first_slot[b] < 0) first_slot[b] = s.slot;
        ++nslot[b];
      }
      hp.segs.push_back(s);
      ob += take;
      remaining -= take;
      if (ob == tiles[b]) { ++b; ob = 0; }
    }
  }
  hp.cta_seg[grid] = static_cast<int>(hp.segs.size());
  for (int i = 0; i < batch; ++i)
    if (nslot[i] > 0) {
      hp.merges.push_back(MergeEntry{i, first_slot[i], nslot[i], 1});
      hp.max_merge_count = std::max(hp.max_merge_count, nslot[i]);
    }
  return 0;
}

// The plans of `count` single sequences side by side: sequence t is cut into
// exactly the segments, partial slots (in order) and merge entry that
// build_attend_plan gives it alone, on CTAs of its own, so one launch computes
// every sequence bit for bit as its own launch would (a block decode then
// equals its serial decode).
int build_concat_plan(HostPlan &hp, int count, const int *seq_len, const long long *seq_row0, int max_ctas) {
  if (count <= 0 || !seq_len || !seq_row0) return -1;
  hp = HostPlan();
  hp.batch = count;
  hp.seq_row0.assign(seq_row0, seq_row0 + count);
  hp.seq_len.assign(seq_len, seq_len + count);
  for (int t = 0; t < count; ++t) {
    HostPlan one;
    const long long r0 = seq_row0[t];
    if (build_attend_plan(one, 1, &seq_len[t], &r0, max_ctas) != 0) return -1;
    const int seg0 = static_cast<int>(hp.segs.size()), slot0 = hp.nparts;
    for (AttendSegment sg : one.segs) {
      sg.seq = t;
      if (sg.slot >= 0) sg.slot += slot0;
      hp.segs.push_back(sg);
    }
    for (int c = 0; c < one.grid; ++c) hp.cta_seg.push_back(seg0 + one.cta_seg[c]);
    for (MergeEntry e : one.merges) {
      e.seq = t;
      e.first += slot0;
      hp.merges.push_back(e);
    }
    hp.nparts += one.nparts;
    hp.grid += one.grid;
    hp.max_merge_count = std::max(hp.max_merge_count, one.max_merge_count);
  }
  hp.cta_seg.push_back(static_cast<int>(hp.segs.size()));
  return 0;
}

// ------------------------------------------------------------------ merge
// (merge_core.cuh holds the combine itself)
__global__ void merge_partials_kernel(float *out, float *lse, const float *part_o,
                                      const float *part_lse, const MergeEntry *entries, int nh,
                                      int R, int uniform_parts, int pb, long long rec_o, long long rec_l) {
  // entries == nullptr: sequence b combines parts b, b + B, b + 2B, ... (part-major layout)
  const MergeEntry e = entries ? entries[blockIdx.x]
                               : MergeEntry{(int)blockIdx.x, (int)blockIdx.x, uniform_parts, (int)gridDim.x};
  const int h = blockIdx.y;
  // Launched as a programmatic dependent of the attend kernel: wait until that
  // grid has completed and its partials are visible; then let the next
  // dependent kernel be scheduled.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const MergeSlice r = merge_slice(e, h, blockIdx.z, part_o, part_lse, nh, R, pb, rec_o, rec_l,
                                   (reinterpret_cast<uintptr_t>(out) & 15) == 0);
  if (lse && blockIdx.z == 0 && threadIdx.x == 0) lse[(size_t)e.seq * nh + h] = r.m + logf(r.sum);
  if (threadIdx.x < 32) {
    const float inv = 1.0f / r.sum;
    const float4 t = r.t;
    const int d0 = r.d0;
    float *dst = out + ((size_t)e.seq * nh + h) * R + d0;
    if (r.vec) {
      *reinterpret_cast<float4 *>(dst) = make_float4(t.x * inv, t.y * inv, t.z * inv, t.w * inv);
    } else {
      if (d0 < R) dst[0] = t.x * inv;
      if (d0 + 1 < R) dst[1] = t.y * inv;
      if (d0 + 2 < R) dst[2] = t.z * inv;
      if (d0 + 3 < R) dst[3] = t.w * inv;
    }
  }
}

// Entries of at most 4 parts (merge_warps == 1): one warp per (entry, head,
// 128-wide slice), eight heads per block, so a batch of short-split sequences
// does not launch one 32-thread block per head.  The arithmetic, including its
// order, is that of merge_partials_kernel with one warp, so which of the two
// runs never changes a result.
__global__ void merge_small_kernel(float *out, float *lse, const float *part_o, const float *part_lse,
                                   const MergeEntry *entries, int nh, int R, int uniform_parts, int pb,
                                   long long rec_o, long long rec_l) {
  const MergeEntry e = entries ? entries[blockIdx.x]
                               : MergeEntry{(int)blockIdx.x, (int)blockIdx.x, uniform_parts, (int)gridDim.x};
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = blockIdx.y * 8 + warp;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (h >= nh) return;
  auto o_of = [&](int q) {
    const int p = e.first + q * e.step;
    return part_o + (p / pb) * rec_o + ((size_t)(p % pb) * nh + h) * R;
  };
  float m = -INFINITY, lv = -INFINITY;
  if (lane < e.count) {
    const int p = e.first + lane * e.step;
    lv = part_lse[(p / pb) * rec_l + (size_t)(p % pb) * nh + h];
    m = lv;
  }
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const float w = lane < e.count ? expf(lv - m) : 0.f;
  float sum = w;
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lse && blockIdx.z == 0 && lane == 0) lse[(size_t)e.seq * nh + h] = m + logf(sum);
  const int d0 = blockIdx.z * 128 + 4 * lane;
  const bool vec = (R & 3) == 0 && d0 + 3 < R && (rec_o & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(part_o) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q = 0; q < e.count; ++q) {
    const float wq = __shfl_sync(0xffffffffu, w, q);
    const float *src = o_of(q) + d0;
    if (vec) {
      const float4 v = *reinterpret_cast<const float4 *>(src);
      acc.x = fmaf(wq, v.x, acc.x);
      acc.y = fmaf(wq, v.y, acc.y);
      acc.z = fmaf(wq, v.z, acc.z);
      acc.w = fmaf(wq, v.w, acc.w);
    } else {
      if (d0 < R) acc.x = fmaf(wq, src[0], acc.x);
      if (d0 + 1 < R) acc.y = fmaf(wq, src[1], acc.y);
      if (d0 + 2 < R) acc.z = fmaf(wq, src[2], acc.z);
      if (d0 + 3 < R) acc.w = fmaf(wq, src[3], acc.w);
    }
  }
  const float inv = 1.0f / sum;
  float *dst = out + ((size_t)e.seq * nh + h) * R + d0;
  if (vec) {
    *reinterpret_cast<float4 *>(dst) = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  } else {
    if (d0 < R) dst[0] = acc.x * inv;
    if (d0 + 1 < R) dst[1] = acc.y * inv;
    if (d0 + 2 < R) dst[2] = acc.z * inv;
    if (d0 + 3 < R) dst[3] = acc.w * inv;
  }
}

// Programmatic dependent launch: the merge grid may be scheduled while the
// attend grid drains (its blocks wait in griddepcontrol.wait), which hides the
// launch gap between the two.
static cudaError_t merge_launch_pdl(float *out, float *lse, const float *part_o, const float *part_lse,
                                    const MergeEntry *d_entries, int n_entries, int nh, int R,
                                    cudaStream_t stream, int max_count, int pb = 1, long long rec_o = -1,
                                    long long rec_l = -1) {
  if (rec_o < 0) rec_o = static_cast<long long>(nh) * R;
  if (rec_l < 0) rec_l = nh;
  const bool small = merge_warps(max_count) == 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = small ? dim3(n_entries, (nh + 7) / 8, (R + 127) / 128) : dim3(n_entries, nh, (R + 127) / 128);
  cfg.blockDim = dim3(small ? 256 : 32 * merge_warps(max_count));
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (small)
    return cudaLaunchKernelEx(&cfg, merge_small_kernel, out, lse, part_o, part_lse, d_entries, nh, R, max_count,
                              pb, rec_o, rec_l);
  return cudaLaunchKernelEx(&cfg, merge_partials_kernel, out, lse, part_o, part_lse, d_entries, nh, R, max_count,
                            pb, rec_o, rec_l);
}

cudaError_t launch_merge(float *out, float *lse, const float *part_o, const float *part_lse,
                         const MergeEntry *d_entries, int n_entries, int nh, int R,
                         cudaStream_t stream, int max_count) {
  // d_entries == nullptr selects the part-major layout with max_count parts per sequence.
  if (n_entries <= 0) return cudaSuccess;
  ProfScope ps("merge_partials", stream);
  return merge_launch_pdl(out, lse, part_o, part_lse, d_entries, n_entries, nh, R, stream, max_count);
}

// Packed records: part r of `parts` is [batch][nh][R] outputs followed by
// [batch][nh] lse values (one all-gather of both per rank).
cudaError_t launch_merge_packed(float *out, float *lse, const float *parts_base, int parts, int batch, int nh,
                                int R, cudaStream_t stream) {
  ProfScope ps("merge_partials", stream);
  const long long rec = static_cast<long long>(batch) * nh * (R + 1);
  return merge_launch_pdl(out, lse, parts_base, parts_base + static_cast<long long>(batch) * nh * R, nullptr,
                          batch, nh, R, stream, parts, batch, rec, rec);
}

// The merge launch without per-kernel timing (its events are created on
// demand); for the entry point that must not allocate.
cudaError_t launch_merge_unprofiled(float *out, float *lse, const float *part_o, const float *part_lse,
                                   const MergeEntry *d_entries, int n_entries, int nh, int R,
                                   cudaStream_t stream, int max_count) {
  if (n_entries <= 0) return cudaSuccess;
  return merge_launch_pdl(out, lse, part_o, part_lse, d_entries, n_entries, nh, R, stream, max_count);
}

// ------------------------------------------------------------------ generic attend
// One CTA per (head, sequence); online softmax over chunks of 1024 rows in
// fp32.  Used only when (NH, R, DR) is not the production (16, 512, 64); the
// drop-in states of such shapes keep fp32 rows (kvf), the reference's own
// state format.
template <bool Q8>
__global__ void attend_generic_kernel(float *out, float *lse, const float *q,
                                      const uint16_t *kv, const float *kvf, const int8_t *lat8,
                                      const float *lscale, const uint16_t *rope16, const long long *row0,
                                      const int *len, int nh, int R, int DR, float scale_log2) {
  constexpr int kChunk = 1024;
  const int h = blockIdx.x, b = blockIdx.y;
  extern __shared__ float sm[];
  float *qv = sm;                 // R + DR
  float *sc = qv + R + DR;        // kChunk
  float *acc = sc + kChunk;       // R
  float *red = acc + R;           // 32
  const int L = len[b];
  const long long r0 = row0[b];
  const float *qs = q + ((size_t)b * nh + h) * (R + DR);
  for (int i = threadIdx.x; i < R + DR; i += blockDim.x) qv[i] = qs[i];
  for (int i = threadIdx.x; i < R; i += blockDim.x) acc[i] = 0.f;
  __syncthreads();
  auto lat = [&](long long row, int r) -> float {
    if (Q8) return __fmul_rn((float)lat8[row * R + r], lscale[row]);
    if (kvf) return kvf[row * (R + DR) + r];
    return __bfloat162float(__ushort_as_bfloat16(kv[row * (R + DR) + r]));
  };
  auto rp = [&](long long row, int d) -> float {
    if (Q8) return __bfloat162float(__ushort_as_bfloat16(rope16[row * DR + d]));
    if (kvf) return kvf[row * (R + DR) + R + d];
    return __bfloat162float(__ushort_as_bfloat16(kv[row * (R + DR) + R + d]));
  };
  auto block_reduce = [&](float v, bool is_max) -> float {
    for (int off = 16; off > 0; off >>= 1) {
      const float o = __shfl_xor_sync(0xffffffffu, v, off);
      v = is_max ? fmaxf(v, o) : v + o;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = is_max ? -INFINITY : 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
    return r;
  };
  float m = -INFINITY, l = 0.f;
  for (int j0 = 0; j0 < L; j0 += kChunk) {
    const int n = min(kChunk, L - j0);
    float cmax = -INFINITY;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      const long long row = r0 + j0 + j;
      float s = 0.f;
      for (int r = 0; r < R; ++r) s = fmaf(qv[r], lat(row, r), s);
      for (int d = 0; d < DR; ++d) s = fmaf(qv[R + d], rp(row, d), s);
      s *= scale_log2;
      sc[j] = s;
      cmax = fmaxf(cmax, s);
    }
    cmax = block_reduce(cmax, true);
    const float mn = fmaxf(m, cmax);
    const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - mn);
    float psum = 0.f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      sc[j] = exp2f(sc[j] - mn);
      psum += sc[j];
    }
    psum = block_reduce(psum, false);
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += blockDim.x) {
      float a = acc[r] * alpha;
      for (int j = 0; j < n; ++j) a = fmaf(sc[j], lat(r0 + j0 + j, r), a);
      acc[r] = a;
    }
    l = l * alpha + psum;
    m = mn;
    __syncthreads();
  }
  float *os = out + ((size_t)b * nh + h) * R;
  for (int r = threadIdx.x; r < R; r += blockDim.x) os[r] = acc[r] / l;
  if (lse && threadIdx.x == 0) lse[(size_t)b * nh + h] = (m + log2f(l)) * 0.69314718055994531f;
}

cudaError_t launch_attend_generic(bool q8, float *out, float *lse, const float *q, const uint16_t *kv,
                                  const float *kvf, const int8_t *lat8, const float *lscale, const uint16_t *rope16,
                                  const long long *d_row0, const int *d_len, int batch, int nh,
                                  int R, int DR, float scale_log2, cudaStream_t stream) {
  const size_t sm = (size_t)(R + DR + 1024 + R + 32) * sizeof(float);
  if (sm > 48 * 1024) {
    auto f = q8 ? attend_generic_kernel<true> : attend_generic_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
  }
  dim3 grid(nh, batch);
  ProfScope ps("attend_generic", stream);
  if (q8)
    attend_generic_kernel<true><<<grid, 128, sm, stream>>>(out, lse, q, kv, nullptr, lat8, lscale, rope16,
                                                           d_row0, d_len, nh, R, DR, scale_log2);
  else
    attend_generic_kernel<false><<<grid, 128, sm, stream>>>(out, lse, q, kv, kvf, lat8, lscale, rope16, d_row0,
                                                            d_len, nh, R, DR, scale_log2);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ device plan
void DevicePlan::release() {
  cudaFree(d_meta);
  cudaFree(d_work);
  d_meta = nullptr;
  d_work = nullptr;
  meta_bytes = work_bytes = 0;
}

// Packs the host plan's arrays into one device allocation (grown on demand)
// and sizes the partial workspace.
int DevicePlan::upload(const HostPlan &hp, int nh, int R, cudaStream_t stream, void *pinned,
                       size_t pinned_bytes) {
  host = hp;
  const size_t seg_b = hp.segs.size() * sizeof(AttendSegment);
  const size_t cta_b = hp.cta_seg.size() * sizeof(int);
  const size_t row_b = hp.seq_row0.size() * sizeof(long long);
  const size_t mer_b = hp.merges.size() * sizeof(MergeEntry);
  const size_t len_b = hp.seq_len.size() * sizeof(int);
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  off_segs = 0;
  off_cta = off_segs + al(seg_b);
  off_row0 = off_cta + al(cta_b);
  off_merge = off_row0 + al(row_b);
  off_len = off_merge + al(mer_b);
  off_err = off_len + al(len_b);
  const size_t need = off_err + 256;
  if (need > meta_bytes) {
    cudaFree(d_meta);
    d_meta = nullptr;
    if (cudaMalloc(&d_meta, need) != cudaSuccess) { meta_bytes = 0; return -1; }
    meta_bytes = need;
  }
  // partial outputs and lse values, then the query images (256-byte aligned)
  const size_t part_bytes = ((size_t)std::max(hp.nparts, 1) * nh * (R + 1) * sizeof(float) + 255) & ~size_t(255);
  const size_t wneed = part_bytes + (size_t)hp.batch * kQImgStride;
  if (wneed > work_bytes) {
    cudaFree(d_work);
    d_work = nullptr;
    if (cudaMalloc(&d_work, wneed) != cudaSuccess) { work_bytes = 0; return -1; }
    work_bytes = wneed;
  }
  std::vector<uint8_t> tmp;
  uint8_t *stage = static_cast<uint8_t *>(pinned);
  if (!stage || pinned_bytes < need) {
    tmp.resize(need);
    stage = tmp.data();
  }
  std::memset(stage + off_err, 0, 256);
  if (seg_b) std::memcpy(stage + off_segs, hp.segs.data(), seg_b);
  std::memcpy(stage + off_cta, hp.cta_seg.data(), cta_b);
  std::memcpy(stage + off_row0, hp.seq_row0.data(), row_b);
  if (mer_b) std::memcpy(stage + off_merge, hp.merges.data(), mer_b);
  if (len_b) std::memcpy(stage + off_len, hp.seq_len.data(), len_b);
  cudaError_t e = cudaMemcpyAsync(d_meta, stage, need, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return -1;
  if (stage == tmp.data()) cudaStreamSynchronize(stream);  // pageable staging must outlive the copy
  part_o = static_cast<float *>(d_work);
  part_lse = part_o + (size_t)std::max(hp.nparts, 1) * nh * R;
  qimg = static_cast<uint8_t *>(d_work) + part_bytes;
  return 0;
}

int DevicePlan::launch(const AttendLaunch &a, cudaStream_t stream) const {
  const uint8_t *m = static_cast<const uint8_t *>(d_meta);
  const int nh = a.nh, R = a.R, DR = a.DR;
  const float scale_log2 = a.softmax_scale * 1.4426950408889634f;
  const bool fast = (nh == kHeads && R == kLatent && DR == kRope);
  if (!fast) {
    return launch_attend_generic(a.q8, a.out, a.lse, a.q, a.kv, a.kvf, a.lat8, a.lscale, a.rope16,
                                 reinterpret_cast<const long long *>(m + off_row0),
                                 reinterpret_cast<const int *>(m + off_len), host.batch, nh, R, DR,
                                 scale_log2, stream) == cudaSuccess
               ? 0
               : -1;
  }
  if (a.rows <= 0 || a.rows >= (1LL << 31)) return -1;
  if ((reinterpret_cast<uintptr_t>(a.q) & 15) != 0) return -1;  // the kernels read q as float4
  AttendParams p;
  std::memset(&p, 0, sizeof(p));
  if (!a.q8) {
    if ((reinterpret_cast<uintptr_t>(a.kv) & 15) != 0) return -1;
    if (!make_tmap_2d(&p.tm_kv, a.kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kRow, a.rows, kRow * 2, 64,
                      kTileTok, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
  } else {
    if (((reinterpret_cast<uintptr_t>(a.lat8) | reinterpret_cast<uintptr_t>(a.rope16) |
          reinterpret_cast<uintptr_t>(a.lscale)) & 15) != 0)
      return -1;
    if (!make_tmap_2d(&p.tm_lat8, a.lat8, CU_TENSOR_MAP_DATA_TYPE_UINT8, kLatent, a.rows, kLatent, 128,
                      kTileTok, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&p.tm_rope, a.rope16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, kRope, a.rows, kRope * 2,
                      64, kTileTok, CU_TENSOR_MAP_SWIZZLE_128B))
      return -1;
    p.latent_scale = a.lscale;
  }
  p.q = a.q;
  p.out = a.out;
  p.lse = a.lse;
  p.part_o = part_o;
  p.part_lse = part_lse;
  p.qimg = qimg;
  p.segs = reinterpret_cast<const AttendSegment *>(m + off_segs);
  p.cta_seg = reinterpret_cast<const int *>(m + off_cta);
  p.seq_row0 = reinterpret_cast<const long long *>(m + off_row0);
  p.rows = a.rows;
  p.scale_log2 = scale_log2;
  p.err = reinterpret_cast<uint32_t *>(const_cast<uint8_t *>(m + off_err));
  // few tiles per CTA: each CTA's first tile goes out before any prefetch
  long long tiles = 0;
  for (const AttendSegment &sg : host.segs) tiles += (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
  p.first_tile_alone = host.grid > 0 && tiles <= 16LL * host.grid;
  // query images are read only from a CTA's second segment on
  bool multi = false;
  for (int c = 0; c < host.grid && !multi; ++c) multi = host.cta_seg[c + 1] - host.cta_seg[c] > 1;
  // with query images the attend is already the prep kernel's dependent
  p.q_after_wait = a.q_dependent && !multi;
  cudaError_t e = a.q8 ? launch_attend_q8(p, host.grid, host.batch, multi, stream)
                       : launch_attend_bf16(p, host.grid, host.batch, multi, stream);
  if (e != cudaSuccess) return -1;
  if (!host.merges.empty() && !a.skip_merge) {
    e = launch_merge(a.out, a.lse, part_o, part_lse, reinterpret_cast<const MergeEntry *>(m + off_merge),
                     static_cast<int>(host.merges.size()), nh, R, stream, host.max_merge_count);
    if (e != cudaSuccess) return -1;
  }
  return 0;
}

uint32_t *DevicePlan::err_word() const {
  return reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(d_meta) + off_err);
}

}  // namespace kvl
