// mla_kernels.cu -- the small kernels around the attend core of one absorbed
// MLA decode step (src/mla_compressed_state.c:86-161):
//   gemv_bf16      y = W x for the q_proj / kv_a_proj / o_proj projections
//                  (src/ops.c:53-66; fp32 accumulation; kv_a_proj in the AVX2
//                  build's exact summation order, src/ops.c:31-50)
//   append_*       RMSNorm of the latent (src/ops.c:76-83) and interleaved
//                  RoPE of the rope slice (src/mla_compressed_state.c:8-22),
//                  stored as a bf16 state row or quantised into the Q8 state
//                  (src/mla_compressed_q8_state.c:9-16, 34-55, 111-127)
//   absorb         q_lat = W_UK^T q_nope per head and RoPE of q_pe
//                  (src/mla_compressed_state.c:119-131)
//   vup            head_out = W_UV mix per head (src/mla_compressed_state.c:149-155)
//
// The float arithmetic of RMSNorm, RoPE and the quantiser uses explicitly
// rounded intrinsics (no FMA contraction) and double-precision angles, so the
// Q8 rows are bit-identical to the reference's given the same fp32 inputs.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "mla_kernels.cuh"
#include "pdl.cuh"
#include "prof.cuh"

namespace kvl {

__device__ __forceinline__ float bf16f(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }

// src/mla_compressed_q8_state.c:9-16: RNE, Inf/NaN keep their high half.
__device__ __forceinline__ uint16_t f32_to_bf16_rne_ref(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7f800000u) != 0x7f800000u) u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

template <typename T>
__device__ __forceinline__ T block_sum(T v, T *red) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  T r = 0;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) r += red[i];
  return r;
}

__device__ __forceinline__ float block_max(float v, float *red) {
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < static_cast<int>(blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
  return r;
}

// The block's threads pull [p, p + bytes) into L2, one 128-byte line each.  The
// matvec kernels run it on their weight rows before pdl_wait(): weights are
// never written by a kernel of a decode step, so the rows stream in while the
// previous kernel drains.
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(127);
  const uintptr_t a1 = reinterpret_cast<uintptr_t>(p) + bytes;
  for (uintptr_t a = a0 + 128 * static_cast<uintptr_t>(threadIdx.x); a < a1; a += 128 * static_cast<uintptr_t>(blockDim.x))
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
}

// A warp pulls one row [p, p + bytes) into L2.
__device__ __forceinline__ void prefetch_row_l2(const void *p, size_t bytes, int lane) {
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(127);
  const uintptr_t a1 = reinterpret_cast<uintptr_t>(p) + bytes;
  for (uintptr_t a = a0 + 128 * static_cast<uintptr_t>(lane); a < a1; a += 128 * 32)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
}

// --------------------------------------------------------------------- gemv
// One warp per output row, NB tokens per block share each weight load.  The
// per-row reduction order depends only on `in`, so a row's result is the same
// whichever tokens it is batched with.
template <int NB>
__global__ void gemv_bf16_kernel(float *y, const float *x, const uint16_t *W, int in, int out, int n) {
  extern __shared__ float xs[];  // [NB][in]
  if (blockIdx.y == 0 && blockIdx.x * 8 < out)
    prefetch_l2(W + static_cast<size_t>(blockIdx.x) * 8 * in, static_cast<size_t>(min(8, out - blockIdx.x * 8)) * in * 2);
  pdl_wait();
  pdl_trigger();
  const int t0 = blockIdx.y * NB;
  const int nb = min(NB, n - t0);
  for (int i = threadIdx.x; i < nb * in; i += blockDim.x) xs[i] = x[static_cast<size_t>(t0) * in + i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * 8 + warp;
  if (o >= out) return;
  const uint16_t *row = W + static_cast<size_t>(o) * in;
  float acc[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = 0.f;
  const bool vec = ((in & 7) == 0) && ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  if (vec) {
    // eight 16-byte loads per lane in flight before their FMAs (the row is a
    // few KB: one load at a time left each warp waiting on HBM latency); the
    // lane still sums its words in the order i8 = lane, lane + 32, ...
    const int n8 = in >> 3;
    constexpr int kPre = 8;
    for (int base = lane; base < n8; base += 32 * kPre) {
      uint4 wv[kPre];
#pragma unroll
      for (int j = 0; j < kPre; ++j)
        if (base + 32 * j < n8) wv[j] = *reinterpret_cast<const uint4 *>(row + (base + 32 * j) * 8);
#pragma unroll
      for (int j = 0; j < kPre; ++j) {
        const int i8 = base + 32 * j;
        if (i8 >= n8) break;
        const uint32_t wr[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
        float wf[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          wf[2 * k] = __uint_as_float(wr[k] << 16);
          wf[2 * k + 1] = __uint_as_float(wr[k] & 0xffff0000u);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          if (b < nb) {
            const float *xb = xs + b * in + i8 * 8;
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[b] = fmaf(wf[k], xb[k], acc[b]);
          }
        }
      }
    }
  } else {
    for (int i = lane; i < in; i += 32) {
      const float wf = bf16f(row[i]);
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (b < nb) acc[b] = fmaf(wf, xs[b * in + i], acc[b]);
    }
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    float v = acc[b];
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (lane == 0 && b < nb) y[static_cast<size_t>(t0 + b) * out + o] = v;
  }
}

// The kv_a_proj rows become state rows, so that product follows the
// summation order of the reference's AVX2 matvec (src/ops.c:31-50) and a
// stored row is the reference's bit for bit: eight fp32 accumulators, the one
// for i = l (mod 8) adding the rounded products w_i * x_i (a multiply, then an
// add: that build has no FMA) in increasing i; then
// ((a0 + a4) + (a1 + a5)) + ((a2 + a6) + (a3 + a7)); then the products of a
// tail past the last multiple of 8, added in order.  A warp per output row: it
// copies the row to shared memory with coalesced 16-byte loads, then lane
// 8 b + l runs accumulator l of token b of the block.
constexpr int kExactTok = 4;
constexpr int kExactWarps = 8;

__global__ void __launch_bounds__(32 * kExactWarps) gemv_bf16_exact_kernel(float *y, const float *x,
                                                                           const uint16_t *W, int in, int out,
                                                                           int n) {
  extern __shared__ float xs[];                                       // [kExactTok][in]
  uint16_t *rows = reinterpret_cast<uint16_t *>(xs + kExactTok * in);  // [kExactWarps][in]
  if (blockIdx.y == 0 && blockIdx.x * kExactWarps < out)
    prefetch_l2(W + static_cast<size_t>(blockIdx.x) * kExactWarps * in,
                static_cast<size_t>(min(kExactWarps, out - blockIdx.x * kExactWarps)) * in * 2);
  pdl_wait();
  pdl_trigger();
  const int t0 = blockIdx.y * kExactTok;
  const int nb = min(kExactTok, n - t0);
  for (int i = threadIdx.x; i < nb * in; i += blockDim.x) xs[i] = x[static_cast<size_t>(t0) * in + i];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o = blockIdx.x * kExactWarps + warp;
  uint16_t *wr = rows + static_cast<size_t>(warp) * in;
  if (o < out) {
    const uint16_t *row = W + static_cast<size_t>(o) * in;
    if ((in & 7) == 0 && ((reinterpret_cast<uintptr_t>(row) | reinterpret_cast<uintptr_t>(wr)) & 15) == 0) {
      const int n8 = in >> 3;
      constexpr int kPre = 8;
      for (int base = lane; base < n8; base += 32 * kPre) {
        uint4 v[kPre];
#pragma unroll
        for (int j = 0; j < kPre; ++j)
          if (base + 32 * j < n8) v[j] = *reinterpret_cast<const uint4 *>(row + (base + 32 * j) * 8);
#pragma unroll
        for (int j = 0; j < kPre; ++j)
          if (base + 32 * j < n8) *reinterpret_cast<uint4 *>(wr + (base + 32 * j) * 8) = v[j];
      }
    } else {
      for (int i = lane; i < in; i += 32) wr[i] = row[i];
    }
  }
  __syncthreads();
  if (o >= out) return;
  const int b = lane >> 3, l = lane & 7;
  const int n8 = in >> 3;
  const float *xb = xs + min(b, kExactTok - 1) * in;
  float a = 0.f;
  if (b < nb) {
#pragma unroll 8
    for (int k = 0; k < n8; ++k) a = __fadd_rn(a, __fmul_rn(bf16f(wr[8 * k + l]), xb[8 * k + l]));
  }
  // the horizontal sum within each group of eight lanes (lane l of the group
  // holds accumulator l)
  const float s1 = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));    // l < 4: a_l + a_{l+4}
  const float s2 = __fadd_rn(s1, __shfl_down_sync(0xffffffffu, s1, 1));  // l = 0, 2: pairs of those
  float tot = __fadd_rn(s2, __shfl_down_sync(0xffffffffu, s2, 2));       // l = 0: the total
  if (l == 0 && b < nb) {
    for (int i = 8 * n8; i < in; ++i) tot = __fadd_rn(tot, __fmul_rn(bf16f(wr[i]), xb[i]));
    y[static_cast<size_t>(t0 + b) * out + o] = tot;
  }
}

cudaError_t gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int n, cudaStream_t s,
                      bool ref_order) {
  if (n <= 0) return cudaSuccess;
  if (ref_order) {
    const size_t sm = static_cast<size_t>(in) * (kExactTok * sizeof(float) + kExactWarps * sizeof(uint16_t));
    if (sm > 227 * 1024) return cudaErrorInvalidValue;
    if (sm > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(gemv_bf16_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(sm));
      if (e != cudaSuccess) return e;
    }
    dim3 grid((out + kExactWarps - 1) / kExactWarps, (n + kExactTok - 1) / kExactTok);
    ProfScope ps("gemv_bf16", s);
    return launch_dependent(gemv_bf16_exact_kernel, grid, dim3(32 * kExactWarps), sm, s, y, x, W, in, out, n);
  }
  constexpr int NB = 4;
  const size_t sm = static_cast<size_t>(NB) * in * sizeof(float);
  if (sm > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(gemv_bf16_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(sm));
    if (e != cudaSuccess) return e;
  }
  dim3 grid((out + 7) / 8, (n + NB - 1) / NB);
  ProfScope ps("gemv_bf16", s);
  return launch_dependent(gemv_bf16_kernel<NB>, grid, dim3(256), sm, s, y, x, W, in, out, n);
}

// --------------------------------------------------------------------- rope / rmsnorm
// src/mla_compressed_state.c:8-22: angle in double, cos/sin rounded to float,
// rotation in float with separately rounded products.
__device__ __forceinline__ void rope_cos_sin(int i, int dim, int pos, float theta, float &c, float &s) {
  const double inv_freq = pow(static_cast<double>(theta), -(static_cast<double>(2 * i) / static_cast<double>(dim)));
  const double ang = static_cast<double>(pos) * inv_freq;
  double sn, cn;
  sincos(ang, &sn, &cn);
  c = static_cast<float>(cn);
  s = static_cast<float>(sn);
}
__device__ __forceinline__ void rope_rotate(float a, float b, float c, float s, float &lo, float &hi) {
  lo = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
  hi = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}
__device__ __forceinline__ void rope_pair(float a, float b, int i, int dim, int pos, float theta, float &lo,
                                          float &hi) {
  float c, s;
  rope_cos_sin(i, dim, pos, theta, c, s);
  rope_rotate(a, b, c, s, lo, hi);
}

// RMSNorm of ka[0:R] into lat (shared memory), src/ops.c:76-83.
__device__ void rmsnorm_row(float *lat, const float *ka, const uint16_t *w, int R, float eps, double *dred) {
  double ss = 0.0;
  for (int i = threadIdx.x; i < R; i += blockDim.x) ss += static_cast<double>(ka[i]) * static_cast<double>(ka[i]);
  ss = block_sum<double>(ss, dred);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ss / static_cast<double>(R)), eps)));
  for (int i = threadIdx.x; i < R; i += blockDim.x) lat[i] = __fmul_rn(__fmul_rn(ka[i], inv), bf16f(w[i]));
  __syncthreads();
}

// bf16 state row [R latent | DR rope] at row (row0 + pos0 + t) of `kv` for each
// of the n tokens; ka is [n][R + DR] (kv_a_proj output), or `parts` split-K
// partials of it (stride part_stride floats) added in order 0, 1, ...
// rows_f32 (optional) receives the fp32 row before bf16 rounding.
// dst[i] = src[i] + src[stride + i] + ... (parts terms, in order) for one row of
// n values, by the block: four values per thread per step, with up to eight
// parts' loads in flight at once.
__device__ __forceinline__ void sum_parts_row(float *dst, const float *src, int n, int parts, long long stride) {
  constexpr int kMaxP = 8;
  const bool vec = ((n | stride) & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  if (vec) {
    for (int i = 4 * threadIdx.x; i < n; i += 4 * blockDim.x) {
      float4 u[kMaxP];
#pragma unroll
      for (int pp = 0; pp < kMaxP; ++pp)
        if (pp == 0 || pp < parts) u[pp] = *reinterpret_cast<const float4 *>(src + pp * stride + i);
      float4 v = u[0];
#pragma unroll
      for (int pp = 1; pp < kMaxP; ++pp)
        if (pp < parts) {
          v.x += u[pp].x;
          v.y += u[pp].y;
          v.z += u[pp].z;
          v.w += u[pp].w;
        }
      for (int pp = kMaxP; pp < parts; ++pp) {
        const float4 w = *reinterpret_cast<const float4 *>(src + pp * stride + i);
        v.x += w.x;
        v.y += w.y;
        v.z += w.z;
        v.w += w.w;
      }
      dst[i] = v.x;
      dst[i + 1] = v.y;
      dst[i + 2] = v.z;
      dst[i + 3] = v.w;
    }
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float v = src[i];
      for (int pp = 1; pp < parts; ++pp) v += src[pp * stride + i];
      dst[i] = v;
    }
  }
}

__global__ void append_bf16_kernel(uint16_t *kv, long long row0, const float *ka, const uint16_t *norm_w, int R,
                                   int DR, int pos0, float eps, float theta, float *rows_f32,
                                   const long long *row_of, const int *pos_of, int parts, long long part_stride) {
  extern __shared__ float sh[];
  float *lat = sh;
  double *dred = reinterpret_cast<double *>(sh + ((R + 1) & ~1));
  float *ksum = reinterpret_cast<float *>(dred + 32) + 32;  // [R + DR] when parts > 1
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const float *kt = ka + static_cast<size_t>(t) * (R + DR);
  if (parts > 1) {
    sum_parts_row(ksum, kt, R + DR, parts, part_stride);
    __syncthreads();
    kt = ksum;
  }
  rmsnorm_row(lat, kt, norm_w, R, eps, dred);
  const int pos = pos_of ? pos_of[t] : pos0 + t;
  const long long row = row_of ? row_of[t] : row0 + pos0 + t;
  uint16_t *dst = kv + static_cast<size_t>(row) * (R + DR);
  float *df = rows_f32 ? rows_f32 + static_cast<size_t>(t) * (R + DR) : nullptr;
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    dst[i] = __bfloat16_as_ushort(__float2bfloat16_rn(lat[i]));
    if (df) df[i] = lat[i];
  }
  const int half = DR / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float lo, hi;
    rope_pair(kt[R + 2 * i], kt[R + 2 * i + 1], i, DR, pos, theta, lo, hi);
    dst[R + i] = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
    dst[R + half + i] = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
    if (df) { df[R + i] = lo; df[R + half + i] = hi; }
  }
}

// Prefill form of append_bf16 for the Kimi shape (R = 512, DR = 64): one warp
// per token, rows [0, n) of `pool`, RoPE cos/sin from a [n][32] table built by
// rope_table_kernel with the same double-angle arithmetic as rope_pair.  The
// same operations as append_bf16 (double sum of squares, float scale, float
// rotation without contraction); only the order of the double sum differs.
__global__ void append_rows_bf16_kernel(uint16_t *pool, const float *ka, const uint16_t *norm_w,
                                        const float2 *cs, int n, float eps, int parts, long long part_stride) {
  constexpr int R = 512, DR = 64;
  pdl_wait();
  pdl_trigger();
  const int warp = static_cast<int>((blockIdx.x * static_cast<unsigned>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const float *kt = ka + static_cast<size_t>(warp) * (R + DR);
  float4 v[4];
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = reinterpret_cast<const float4 *>(kt)[lane + 32 * k];
    for (int z = 1; z < parts; ++z) {  // split-K partial products, summed in order
      const float4 u = reinterpret_cast<const float4 *>(kt + z * part_stride)[lane + 32 * k];
      v[k].x += u.x;
      v[k].y += u.y;
      v[k].z += u.z;
      v[k].w += u.w;
    }
    ss += static_cast<double>(v[k].x) * static_cast<double>(v[k].x);
    ss += static_cast<double>(v[k].y) * static_cast<double>(v[k].y);
    ss += static_cast<double>(v[k].z) * static_cast<double>(v[k].z);
    ss += static_cast<double>(v[k].w) * static_cast<double>(v[k].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(ss / static_cast<double>(R)), eps)));
  uint16_t *dst = pool + static_cast<size_t>(warp) * (R + DR);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int c = 4 * (lane + 32 * k);
    const uint2 w = *reinterpret_cast<const uint2 *>(norm_w + c);
    const float y0 = __fmul_rn(__fmul_rn(v[k].x, inv), __uint_as_float(w.x << 16));
    const float y1 = __fmul_rn(__fmul_rn(v[k].y, inv), __uint_as_float(w.x & 0xffff0000u));
    const float y2 = __fmul_rn(__fmul_rn(v[k].z, inv), __uint_as_float(w.y << 16));
    const float y3 = __fmul_rn(__fmul_rn(v[k].w, inv), __uint_as_float(w.y & 0xffff0000u));
    uint2 o;
    o.x = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(y0))) |
          (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(y1))) << 16);
    o.y = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(y2))) |
          (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(y3))) << 16);
    *reinterpret_cast<uint2 *>(dst + c) = o;
  }
  // rope pair (2i, 2i+1) -> (i, 32 + i), i = lane
  float2 ab = reinterpret_cast<const float2 *>(kt + R)[lane];
  for (int z = 1; z < parts; ++z) {
    const float2 u = reinterpret_cast<const float2 *>(kt + z * part_stride + R)[lane];
    ab.x += u.x;
    ab.y += u.y;
  }
  const float2 t = cs[static_cast<size_t>(warp) * (DR / 2) + lane];
  const float lo = __fsub_rn(__fmul_rn(ab.x, t.x), __fmul_rn(ab.y, t.y));
  const float hi = __fadd_rn(__fmul_rn(ab.y, t.x), __fmul_rn(ab.x, t.y));
  dst[R + lane] = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  dst[R + DR / 2 + lane] = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
}

cudaError_t append_rows_bf16(uint16_t *pool, const float *ka, const uint16_t *norm_w, const float2 *cs, int n,
                             float eps, cudaStream_t s, int parts, long long part_stride) {
  if (n <= 0) return cudaSuccess;
  if (parts < 1) return cudaErrorInvalidValue;
  ProfScope ps("append_bf16", s);
  return launch_dependent(append_rows_bf16_kernel, dim3((n + 7) / 8), dim3(256), 0, s, pool, ka, norm_w, cs, n, eps,
                          parts, part_stride);
}

// q = sum of split-K partial products [parts][n][16 * 192] fp32 with RoPE on
// each head's last 64 columns, bf16 [n][16][192]: the arithmetic of the
// q_proj GEMM's EPI_QROPE epilogue (pair (2i, 2i + 1) -> (i, 32 + i)).  One
// warp per (row, head): lane l sums nope columns 4l .. 4l + 3 and rope pair l.
__global__ void sum_parts_qrope_kernel(uint16_t *q, const float *parts, int np, long long stride,
                                       const float2 *cs, int n) {
  const int wid = static_cast<int>((blockIdx.x * static_cast<unsigned>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= n * 16) return;
  const int row = wid >> 4, head = wid & 15;
  const float *src = parts + static_cast<size_t>(row) * (16 * 192) + head * 192;
  float4 a = *reinterpret_cast<const float4 *>(src + 4 * lane);
  float2 r = *reinterpret_cast<const float2 *>(src + 128 + 2 * lane);
  for (int z = 1; z < np; ++z) {
    const float4 u = *reinterpret_cast<const float4 *>(src + z * stride + 4 * lane);
    const float2 v = *reinterpret_cast<const float2 *>(src + z * stride + 128 + 2 * lane);
    a.x += u.x;
    a.y += u.y;
    a.z += u.z;
    a.w += u.w;
    r.x += v.x;
    r.y += v.y;
  }
  __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(q) + static_cast<size_t>(row) * (16 * 192) + head * 192;
  uint2 o;
  o.x = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a.x))) |
        (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a.y))) << 16);
  o.y = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a.z))) |
        (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a.w))) << 16);
  *reinterpret_cast<uint2 *>(dst + 4 * lane) = o;
  const float2 t = cs[static_cast<size_t>(row) * 32 + lane];
  dst[128 + lane] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(r.x, t.x), __fmul_rn(r.y, t.y)));
  dst[160 + lane] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(r.y, t.x), __fmul_rn(r.x, t.y)));
}

cudaError_t sum_parts_qrope(uint16_t *q, const float *parts, int np, long long stride, const float2 *cs, int n,
                            cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (np < 1) return cudaErrorInvalidValue;
  ProfScope ps("sum_qrope", s);
  sum_parts_qrope_kernel<<<(n * 16 + 7) / 8, 256, 0, s>>>(q, parts, np, stride, cs, n);
  return cudaGetLastError();
}

// src/mla_compressed_q8_state.c:34-55 for one row held in shared memory.
__device__ void quantize_row(int8_t *q, float *scale_out, const float *lat, int R, float *fred) {
  float amax = 0.f;
  for (int i = threadIdx.x; i < R; i += blockDim.x) amax = fmaxf(amax, fabsf(lat[i]));
  amax = block_max(amax, fred);
  if (!(amax > 0.0f) || !isfinite(amax)) {
    for (int i = threadIdx.x; i < R; i += blockDim.x) q[i] = 0;
    if (threadIdx.x == 0) *scale_out = 1.0f;
    return;
  }
  const float scale = __fdiv_rn(amax, 127.0f);
  const float inv = __fdiv_rn(1.0f, scale);
  for (int i = threadIdx.x; i < R; i += blockDim.x) {
    const float r = roundf(__fmul_rn(lat[i], inv));
    // A NaN element of a finite row passes the reference's clamp unchanged and
    // its (int8_t) conversion on x86-64 keeps the low byte of INT32_MIN: 0.
    q[i] = isnan(r) ? static_cast<int8_t>(0) : static_cast<int8_t>(fminf(fmaxf(r, -127.0f), 127.0f));
  }
  if (threadIdx.x == 0) *scale_out = scale;
}

// Q8 state row (int8 latent, fp32 scale, bf16 rope) for each of the n tokens,
// at the rows append_bf16 would use; ka as for append_bf16 (optionally
// `parts` split-K partials added in order).
__global__ void append_q8_kernel(int8_t *lat8, float *lscale, uint16_t *rope16, long long row0, const float *ka,
                                 const uint16_t *norm_w, int R, int DR, int pos0, float eps, float theta,
                                 const long long *row_of, const int *pos_of, int parts, long long part_stride) {
  extern __shared__ float sh[];
  float *lat = sh;
  double *dred = reinterpret_cast<double *>(sh + ((R + 1) & ~1));
  float *fred = reinterpret_cast<float *>(dred + 32);
  float *ksum = fred + 32;  // [R + DR] when parts > 1
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int pos = pos_of ? pos_of[t] : pos0 + t;
  const long long row = row_of ? row_of[t] : row0 + pos0 + t;
  const float *kt = ka + static_cast<size_t>(t) * (R + DR);
  if (parts > 1) {
    sum_parts_row(ksum, kt, R + DR, parts, part_stride);
    __syncthreads();
    kt = ksum;
  }
  rmsnorm_row(lat, kt, norm_w, R, eps, dred);
  quantize_row(lat8 + static_cast<size_t>(row) * R, lscale + row, lat, R, fred);
  const int half = DR / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float lo, hi;
    rope_pair(kt[R + 2 * i], kt[R + 2 * i + 1], i, DR, pos, theta, lo, hi);
    rope16[static_cast<size_t>(row) * DR + i] = f32_to_bf16_rne_ref(lo);
    rope16[static_cast<size_t>(row) * DR + half + i] = f32_to_bf16_rne_ref(hi);
  }
}

static size_t append_smem(int R) { return static_cast<size_t>((R + 1) & ~1) * 4 + 32 * 8 + 32 * 4; }
static size_t append_smem_parts(int R, int DR) { return append_smem(R) + static_cast<size_t>(R + DR) * 4; }

cudaError_t append_bf16(uint16_t *kv, long long row0, const float *ka, const uint16_t *norm_w, int n, int R,
                        int DR, int pos0, float eps, float theta, float *rows_f32, cudaStream_t s,
                        const long long *row_of, const int *pos_of, int parts, long long part_stride) {
  if (n <= 0) return cudaSuccess;
  ProfScope ps("append_bf16", s);
  const size_t sm = parts > 1 ? append_smem_parts(R, DR) : append_smem(R);
  return launch_dependent(append_bf16_kernel, dim3(n), dim3(128), sm, s, kv, row0, ka, norm_w, R, DR, pos0, eps, theta,
                          rows_f32, row_of, pos_of, parts, part_stride);
}

cudaError_t append_q8(int8_t *lat8, float *lscale, uint16_t *rope16, long long row0, const float *ka,
                      const uint16_t *norm_w, int n, int R, int DR, int pos0, float eps, float theta,
                      cudaStream_t s, const long long *row_of, const int *pos_of, int parts, long long part_stride) {
  if (n <= 0) return cudaSuccess;
  ProfScope ps("append_q8", s);
  const size_t sm = parts > 1 ? append_smem_parts(R, DR) : append_smem(R);
  return launch_dependent(append_q8_kernel, dim3(n), dim3(128), sm, s, lat8, lscale, rope16, row0, ka, norm_w, R, DR,
                          pos0, eps, theta, row_of, pos_of, parts, part_stride);
}

// --------------------------------------------------------------------- absorb / vup
// qabs[t][h] = [ W_UK[h]^T q_nope[t][h] (R values) | rope(q_pe[t][h]) (DR values) ]
__global__ void absorb_kernel(float *qabs, const float *q, const uint16_t *kvb, int NH, int DN, int DV, int DR,
                              int R, int pos0, float theta, const int *pos_of) {
  extern __shared__ float qn[];
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, t = blockIdx.y;
  const float *qh = q + (static_cast<size_t>(t) * NH + h) * (DN + DR);
  for (int d = threadIdx.x; d < DN; d += blockDim.x) qn[d] = qh[d];
  __syncthreads();
  float *dst = qabs + (static_cast<size_t>(t) * NH + h) * (R + DR);
  const uint16_t *wh = kvb + static_cast<size_t>(h) * (DN + DV) * R;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    float acc = 0.f;
    for (int d = 0; d < DN; ++d) acc = fmaf(bf16f(wh[static_cast<size_t>(d) * R + r]), qn[d], acc);
    dst[r] = acc;
  }
  const int half = DR / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float lo, hi;
    rope_pair(qh[DN + 2 * i], qh[DN + 2 * i + 1], i, DR, pos_of ? pos_of[t] : pos0 + t, theta, lo, hi);
    dst[R + i] = lo;
    dst[R + half + i] = hi;
  }
}

// The same product with R split into 64-wide blocks (grid NH x R/64 x n): warp
// g of a block sums dims d in [g DN/8, (g + 1) DN/8) for two columns per lane
// (one 4-byte load of a bf16 pair, 128 contiguous bytes per warp), and the
// eight partial sums are added in warp order.  R % 64 == 0, DN % 8 == 0.
__global__ void __launch_bounds__(256) absorb_r64_kernel(float *qabs, const float *q, const uint16_t *kvb, int NH,
                                                         int DN, int DV, int DR, int R, int pos0, float theta,
                                                         const int *pos_of) {
  __shared__ float part[8][64];
  const int h = blockIdx.x, rb = blockIdx.y, t = blockIdx.z;
  const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (t == 0)
    for (int d = threadIdx.x; d < DN; d += blockDim.x)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(kvb + (static_cast<size_t>(h) * (DN + DV) + d) * R + 64 * rb));
  pdl_wait();
  pdl_trigger();
  const float *qh = q + (static_cast<size_t>(t) * NH + h) * (DN + DR);
  const uint16_t *wh = kvb + static_cast<size_t>(h) * (DN + DV) * R + 64 * rb + 2 * lane;
  const int dpg = DN / 8;
  float a0 = 0.f, a1 = 0.f;
  for (int k = 0; k < dpg; ++k) {
    const int d = g * dpg + k;
    const uint32_t w2 = *reinterpret_cast<const uint32_t *>(wh + static_cast<size_t>(d) * R);
    const float qd = qh[d];
    a0 = fmaf(__uint_as_float(w2 << 16), qd, a0);
    a1 = fmaf(__uint_as_float(w2 & 0xffff0000u), qd, a1);
  }
  part[g][2 * lane] = a0;
  part[g][2 * lane + 1] = a1;
  __syncthreads();
  float *dst = qabs + (static_cast<size_t>(t) * NH + h) * (R + DR);
  if (threadIdx.x < 64) {
    float acc = part[0][threadIdx.x];
#pragma unroll
    for (int i = 1; i < 8; ++i) acc += part[i][threadIdx.x];
    dst[64 * rb + threadIdx.x] = acc;
  }
  if (rb == 0) {
    const int half = DR / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      float lo, hi;
      rope_pair(qh[DN + 2 * i], qh[DN + 2 * i + 1], i, DR, pos_of ? pos_of[t] : pos0 + t, theta, lo, hi);
      dst[R + i] = lo;
      dst[R + half + i] = hi;
    }
  }
}

cudaError_t absorb(float *qabs, const float *q, const uint16_t *kvb, int n, int NH, int DN, int DV, int DR, int R,
                   int pos0, float theta, cudaStream_t s, const int *pos_of) {
  if (n <= 0) return cudaSuccess;
  ProfScope ps("absorb", s);
  if (R % 64 == 0 && DN % 8 == 0 && (reinterpret_cast<uintptr_t>(kvb) & 3) == 0) {
    return launch_dependent(absorb_r64_kernel, dim3(NH, R / 64, n), dim3(256), 0, s, qabs, q, kvb, NH, DN, DV, DR, R,
                            pos0, theta, pos_of);
  }
  return launch_dependent(absorb_kernel, dim3(NH, n), dim3(256), DN * sizeof(float), s, qabs, q, kvb, NH, DN, DV, DR,
                          R, pos0, theta, pos_of);
}

// ho[t][h*DV + d] = sum_r W_UV[h][d][r] * mix[t][h][r]; one warp per (h, d).
__global__ void vup_kernel(float *ho, const float *mix, const uint16_t *kvb, int NH, int DN, int DV, int R) {
  const int t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = blockIdx.x * 8 + warp;
  if (t == 0 && hd < NH * DV)
    prefetch_row_l2(kvb + (static_cast<size_t>(hd / DV) * (DN + DV) + DN + hd % DV) * R, static_cast<size_t>(R) * 2,
                    lane);
  pdl_wait();
  pdl_trigger();
  if (hd >= NH * DV) return;
  const int h = hd / DV, d = hd % DV;
  const uint16_t *row = kvb + (static_cast<size_t>(h) * (DN + DV) + DN + d) * R;
  const float *m = mix + (static_cast<size_t>(t) * NH + h) * R;
  float acc = 0.f;
  if ((R & 7) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    for (int i8 = lane; i8 < R / 8; i8 += 32) {
      const uint4 wv = *reinterpret_cast<const uint4 *>(row + i8 * 8);
      const uint32_t wr[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc = fmaf(__uint_as_float(wr[k] << 16), m[i8 * 8 + 2 * k], acc);
        acc = fmaf(__uint_as_float(wr[k] & 0xffff0000u), m[i8 * 8 + 2 * k + 1], acc);
      }
    }
  } else {
    for (int i = lane; i < R; i += 32) acc = fmaf(bf16f(row[i]), m[i], acc);
  }
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) ho[static_cast<size_t>(t) * NH * DV + hd] = acc;
}

cudaError_t vup(float *ho, const float *mix, const uint16_t *kvb, int n, int NH, int DN, int DV, int R,
                cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  ProfScope ps("vup", s);
  return launch_dependent(vup_kernel, dim3((NH * DV + 7) / 8, n), dim3(256), 0, s, ho, mix, kvb, NH, DN, DV, R);
}

// Tensor-core decode step helpers (batches of sequences).
// q: `parts` split-K partial products [part][t][h][DN + DR] fp32 (stride
// part_stride floats), added in order -> qn [h][t][DN] bf16 (head-major: the A
// operand of the per-head q_nope . W_UK product) and the rotated rope part of
// qabs [t][h][R + DR] (the rope of absorb_kernel, same arithmetic).  Block
// (t, y) takes heads kQsHeads y .. + kQsHeads - 1 of token t: four consecutive
// q_nope values per thread (all of a thread's partial loads in flight at
// once), then one rope pair per thread; cos/sin once per block.
constexpr int kQsHeads = 4;

__global__ void __launch_bounds__(128) q_split_kernel(uint16_t *qn, float *qabs, const float *q, int parts,
                                                      long long part_stride, int n, int NH, int DN, int DR, int R,
                                                      float theta, const int *pos_of) {
  __shared__ float2 cs[128];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, h0 = blockIdx.y * kQsHeads, half = DR / 2, QD = DN + DR;
  const int nh = min(kQsHeads, NH - h0);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float c, sn;
    rope_cos_sin(i, DR, pos_of[t], theta, c, sn);
    cs[i] = make_float2(c, sn);
  }
  const float *qt = q + static_cast<size_t>(t) * NH * QD;
  const bool vec = (DN & 3) == 0 && (QD & 3) == 0 && (part_stride & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(q) & 15) == 0;
  if (vec) {
    for (int idx = threadIdx.x; idx < nh * (DN / 4); idx += blockDim.x) {
      const int h = h0 + idx / (DN / 4), d = 4 * (idx % (DN / 4));
      const float *src = qt + h * QD + d;
      float4 v = *reinterpret_cast<const float4 *>(src);
      for (int pp = 1; pp < parts; ++pp) {
        const float4 u = *reinterpret_cast<const float4 *>(src + pp * part_stride);
        v.x += u.x;
        v.y += u.y;
        v.z += u.z;
        v.w += u.w;
      }
      const __nv_bfloat162 lo2 = __floats2bfloat162_rn(v.x, v.y), hi2 = __floats2bfloat162_rn(v.z, v.w);
      uint2 o;
      o.x = *reinterpret_cast<const uint32_t *>(&lo2);
      o.y = *reinterpret_cast<const uint32_t *>(&hi2);
      *reinterpret_cast<uint2 *>(qn + (static_cast<size_t>(h) * n + t) * DN + d) = o;
    }
  } else {
    for (int idx = threadIdx.x; idx < nh * DN; idx += blockDim.x) {
      const int h = h0 + idx / DN, d = idx % DN;
      float v = qt[h * QD + d];
      for (int pp = 1; pp < parts; ++pp) v += qt[pp * part_stride + h * QD + d];
      qn[(static_cast<size_t>(h) * n + t) * DN + d] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nh * half; idx += blockDim.x) {
    const int h = h0 + idx / half, i = idx % half;
    const float *src = qt + h * QD + DN + 2 * i;
    float a = src[0], b = src[1];
    for (int pp = 1; pp < parts; ++pp) {
      a += src[pp * part_stride];
      b += src[pp * part_stride + 1];
    }
    float lo, hi;
    rope_rotate(a, b, cs[i].x, cs[i].y, lo, hi);
    float *dst = qabs + (static_cast<size_t>(t) * NH + h) * (R + DR);
    dst[R + i] = lo;
    dst[R + half + i] = hi;
  }
}

cudaError_t q_split(uint16_t *qn, float *qabs, const float *q, int parts, long long part_stride, int n, int NH,
                    int DN, int DR, int R, float theta, const int *pos_of, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (DR / 2 > 128) return cudaErrorInvalidValue;
  ProfScope ps("q_split", s);
  return launch_dependent(q_split_kernel, dim3(n, (NH + kQsHeads - 1) / kQsHeads), dim3(128), 0, s, qn, qabs, q, parts,
                          part_stride, n, NH, DN, DR, R, theta, pos_of);
}

// dst[i] = src[i] + src[stride + i] + ... (parts terms, in order), fp32.
__global__ void sum_parts_kernel(float *dst, const float *src, int parts, long long stride, long long n) {
  pdl_wait();
  pdl_trigger();
  const bool vec = ((n | stride) & 3) == 0 && ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) &
                                               15) == 0;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
  if (vec) {
    constexpr int kMaxP = 8;  // up to eight parts' loads in flight at once, then added in order
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n / 4; i += step) {
      float4 u[kMaxP];
#pragma unroll
      for (int pp = 0; pp < kMaxP; ++pp)
        if (pp == 0 || pp < parts) u[pp] = reinterpret_cast<const float4 *>(src + pp * stride)[i];
      float4 v = u[0];
#pragma unroll
      for (int pp = 1; pp < kMaxP; ++pp)
        if (pp < parts) {
          v.x += u[pp].x;
          v.y += u[pp].y;
          v.z += u[pp].z;
          v.w += u[pp].w;
        }
      for (int pp = kMaxP; pp < parts; ++pp) {
        const float4 w = reinterpret_cast<const float4 *>(src + pp * stride)[i];
        v.x += w.x;
        v.y += w.y;
        v.z += w.z;
        v.w += w.w;
      }
      reinterpret_cast<float4 *>(dst)[i] = v;
    }
  } else {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += step) {
      float v = src[i];
      for (int pp = 1; pp < parts; ++pp) v += src[pp * stride + i];
      dst[i] = v;
    }
  }
}

cudaError_t sum_parts(float *dst, const float *src, int parts, long long stride, long long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const long long work = (n + 3) / 4;
  const int grid = static_cast<int>((work + 255) / 256 < 148 * 8 ? (work + 255) / 256 : 148 * 8);
  ProfScope ps("sum_parts", s);
  return launch_dependent(sum_parts_kernel, dim3(grid), dim3(256), 0, s, dst, src, parts, stride, n);
}

// mix [t][h][R] fp32 -> [h][t][R] bf16 (round to nearest even), the
// head-major A operand of the per-head mix . W_UV^T product (R % 4 == 0).
__global__ void mix_heads_bf16_kernel(uint16_t *out, const float *mix, int n, int NH, int R) {
  pdl_wait();
  pdl_trigger();
  const int r4n = R / 4;
  const long long total = static_cast<long long>(n) * NH * r4n;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r4 = static_cast<int>(i % r4n);
    const long long tr = i / r4n;
    const int h = static_cast<int>(tr % NH), t = static_cast<int>(tr / NH);
    const float4 v = reinterpret_cast<const float4 *>(mix)[i];
    uint2 o;
    o.x = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v.x))) |
          (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v.y))) << 16);
    o.y = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v.z))) |
          (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v.w))) << 16);
    *reinterpret_cast<uint2 *>(out + (static_cast<size_t>(h) * n + t) * R + 4 * r4) = o;
  }
}

cudaError_t mix_heads_bf16(uint16_t *out, const float *mix, int n, int NH, int R, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (R % 4 != 0 || ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(mix)) & 15) != 0)
    return cudaErrorInvalidValue;
  const long long total = static_cast<long long>(n) * NH * (R / 4);
  const int grid = static_cast<int>((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
  ProfScope ps("mix_heads_bf16", s);
  return launch_dependent(mix_heads_bf16_kernel, dim3(grid), dim3(256), 0, s, out, mix, n, NH, R);
}

// --------------------------------------------------------------------- Q8 helpers
__global__ void quantize_rows_kernel(int8_t *q, float *scale, const float *x, int R) {
  extern __shared__ float sh[];
  float *row = sh;
  float *fred = sh + R;
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < R; i += blockDim.x) row[i] = x[static_cast<size_t>(t) * R + i];
  __syncthreads();
  quantize_row(q + static_cast<size_t>(t) * R, scale + t, row, R, fred);
}

cudaError_t quantize_rows(int8_t *q, float *scale, const float *x, int rows, int R, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  quantize_rows_kernel<<<rows, 128, (R + 32) * sizeof(float), s>>>(q, scale, x, R);
  return cudaGetLastError();
}

// src/mla_compressed_q8_state.c:57-61: one float multiply per element.
__global__ void dequant_kernel(float *out, const int8_t *q, const float *scale, long long rows, int R) {
  const long long n = rows * R;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = __fmul_rn(static_cast<float>(q[i]), scale[i / R]);
}

cudaError_t dequant(float *out, const int8_t *q, const float *scale, long long rows, int R, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  const long long n = rows * R;
  const int grid = static_cast<int>((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  dequant_kernel<<<grid, 256, 0, s>>>(out, q, scale, rows, R);
  return cudaGetLastError();
}

__global__ void bf16_rne_kernel(uint16_t *out, const float *x, long long n) {
  pdl_wait();
  pdl_trigger();
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
  const bool vec = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 7) == 0;
  if (vec) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n / 4; i += step) {
      const float4 v = reinterpret_cast<const float4 *>(x)[i];
      uint2 o;
      o.x = static_cast<uint32_t>(f32_to_bf16_rne_ref(v.x)) | (static_cast<uint32_t>(f32_to_bf16_rne_ref(v.y)) << 16);
      o.y = static_cast<uint32_t>(f32_to_bf16_rne_ref(v.z)) | (static_cast<uint32_t>(f32_to_bf16_rne_ref(v.w)) << 16);
      reinterpret_cast<uint2 *>(out)[i] = o;
    }
  } else {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += step)
      out[i] = f32_to_bf16_rne_ref(x[i]);
  }
}

cudaError_t bf16_rne(uint16_t *out, const float *x, long long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  ProfScope ps("bf16_rne", s);
  const long long work = (n + 3) / 4;
  const int grid = static_cast<int>((work + 255) / 256 < 148 * 8 ? (work + 255) / 256 : 148 * 8);
  return launch_dependent(bf16_rne_kernel, dim3(grid), dim3(256), 0, s, out, x, n);
}

// bf16 state row -> fp32 (the host mirror of the reference's fp32 state).
__global__ void bf16_to_f32_kernel(float *out, const uint16_t *x, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = bf16f(x[i]);
}

cudaError_t bf16_to_f32(float *out, const uint16_t *x, long long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int grid = static_cast<int>((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  ProfScope ps("bf16_to_f32", s);
  bf16_to_f32_kernel<<<grid, 256, 0, s>>>(out, x, n);
  return cudaGetLastError();
}

__global__ void f32_to_bf16_kernel(uint16_t *out, const float *x, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(x[i]));
}

cudaError_t f32_to_bf16(uint16_t *out, const float *x, long long n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int grid = static_cast<int>((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  f32_to_bf16_kernel<<<grid, 256, 0, s>>>(out, x, n);
  return cudaGetLastError();
}

}  // namespace kvl
