// merge_core.cuh -- the split-KV combine of one (entry, head, 128-wide slice),
// shared by the single-GPU merge kernel (attend_host.cu) and the fused
// cross-GPU combine (peer_merge.cu) so both sum in the same order.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "attend_host.cuh"

namespace kvl {

// out[seq][h][:] = sum_p w_p o_p / sum_p w_p,  w_p = exp(lse_p - max_p lse_p);
// lse[seq][h] = max + log(sum_p w_p).  Part p of an entry lives at part index
// first + p * step (each part is [16][R] floats and [16] lse values).
// Grid (entry, head, 128-wide slice of R); each lane owns 4 consecutive output
// elements and the block's warps split the entry's parts, so a part's slice is
// one coalesced 512-byte read.  The block first turns the parts' lse values
// into weights exp(lse - max) in shared memory (one pass of loads, block-wide
// reductions); each warp then keeps eight parts' slices in flight per step.
constexpr int kMergeSmemParts = 256;
// Warps that combine an entry of `count` parts: enough to split the parts (a
// few per warp), at most 8, so that a merge block (~5 KB of shared memory) fits
// beside a resident bf16 attend CTA and waits there for the attend grid to
// complete.  A function of the entry alone, so an entry's summation order does
// not depend on the other entries of the launch (a block decode merges each
// token exactly as its serial decode does).
__host__ __device__ inline int merge_warps(int count) {
  int w = 1;
  while (w < 8 && 4 * w < count) w <<= 1;
  return w;
}

// Part p lives at part_o + (p / pb) * rec_o + (p % pb) * nh * R (and the lse
// likewise with rec_l, nh): pb = 1, rec_o = nh * R, rec_l = nh for the
// part-major arrays; pb = batch for packed records [batch][nh][R] ++ [batch][nh].
// merge_slice combines slice z (elements [128 z, 128 z + 128)) of head h of
// entry e with the block's first merge_warps(e.count) warps (the block has at
// least that many).  On return every thread holds m (max lse) and sum (sum of
// the weights); lane l of warp 0 holds t, the unnormalised weighted sum of the
// elements d0 = 128 z + 4 l .. d0 + 3, and vec says whether they were read as
// one float4 (R, rec_o and part_o 4-float aligned, d0 + 3 < R, out_aligned).
struct MergeSlice {
  float4 t;
  float m, sum;
  int d0;
  bool vec;
};

__device__ __forceinline__ MergeSlice merge_slice(const MergeEntry e, int h, int z, const float *part_o,
                                                  const float *part_lse, int nh, int R, int pb, long long rec_o,
                                                  long long rec_l, bool out_aligned) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = min(static_cast<int>(blockDim.x >> 5), merge_warps(e.count));  // warps >= nw only sync
  const bool act = warp < nw;
  __shared__ float4 red[8][32];
  __shared__ float wts[kMergeSmemParts];
  __shared__ float rs[8];
  auto part_of = [&](int q) { return e.first + q * e.step; };
  auto lse_of = [&](int q) {
    const int p = part_of(q);
    return part_lse[(p / pb) * rec_l + (size_t)(p % pb) * nh + h];
  };
  auto o_of = [&](int q) {
    const int p = part_of(q);
    return part_o + (p / pb) * rec_o + ((size_t)(p % pb) * nh + h) * R;
  };
  float m = -INFINITY;
  for (int q = threadIdx.x; act && q < e.count; q += 32 * nw) {
    const float v = lse_of(q);
    if (q < kMergeSmemParts) wts[q] = v;
    m = fmaxf(m, v);
  }
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0 && act) rs[warp] = m;
  __syncthreads();
  m = rs[0];
  for (int i = 1; i < nw; ++i) m = fmaxf(m, rs[i]);
  __syncthreads();
  float sum = 0.f;
  for (int q = threadIdx.x; act && q < e.count; q += 32 * nw) {
    const float w = expf((q < kMergeSmemParts ? wts[q] : lse_of(q)) - m);
    if (q < kMergeSmemParts) wts[q] = w;
    sum += w;
  }
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0 && act) rs[warp] = sum;
  __syncthreads();
  sum = 0.f;
  for (int i = 0; i < nw; ++i) sum += rs[i];
  const int d0 = z * 128 + 4 * lane;
  const bool vec = out_aligned && (R & 3) == 0 && d0 + 3 < R && (rec_o & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(part_o) & 15) == 0;
  auto weight = [&](int q) { return q < kMergeSmemParts ? wts[q] : expf(lse_of(q) - m); };
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (vec) {
    for (int q0 = warp; act && q0 < e.count; q0 += 8 * nw) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = q0 + j * nw;
        v[j] = q < e.count ? *reinterpret_cast<const float4 *>(o_of(q) + d0) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = q0 + j * nw;
        if (q < e.count) {
          const float w = weight(q);
          acc.x = fmaf(w, v[j].x, acc.x);
          acc.y = fmaf(w, v[j].y, acc.y);
          acc.z = fmaf(w, v[j].z, acc.z);
          acc.w = fmaf(w, v[j].w, acc.w);
        }
      }
    }
  } else {
    for (int q = warp; act && q < e.count; q += nw) {
      const float w = weight(q);
      const float *src = o_of(q) + d0;
      if (d0 < R) acc.x = fmaf(w, src[0], acc.x);
      if (d0 + 1 < R) acc.y = fmaf(w, src[1], acc.y);
      if (d0 + 2 < R) acc.z = fmaf(w, src[2], acc.z);
      if (d0 + 3 < R) acc.w = fmaf(w, src[3], acc.w);
    }
  }
  if (act) red[warp][lane] = acc;
  __syncthreads();
  MergeSlice r;
  r.m = m;
  r.sum = sum;
  r.d0 = d0;
  r.vec = vec;
  r.t = make_float4(0.f, 0.f, 0.f, 0.f);
  if (warp == 0) {
    float4 t = red[0][lane];
    for (int i = 1; i < nw; ++i) {
      const float4 u = red[i][lane];
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    r.t = t;
  }
  return r;
}

}  // namespace kvl
