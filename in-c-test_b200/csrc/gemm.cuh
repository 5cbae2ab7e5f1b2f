// gemm.cuh -- tcgen05 GEMM (C = A . B^T, bf16 in, fp32 accumulate) used by the
// prefill projections; see gemm.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kvl {

enum : int { EPI_F32 = 0, EPI_BF16 = 1, EPI_QROPE = 2 };

struct GemmParams {
  CUtensorMap tm_a;     // A [M][K] bf16, box 64 x 128
  CUtensorMap tm_b;     // B [N][K] bf16, box 64 x BN
  int M, N, K;
  void *c;              // output, row-major with leading dimension ldc (elements)
  int ldc;
  const float2 *rope_cs;  // EPI_QROPE: cos/sin table [M][32]
  uint32_t *err;
  // batch > 1: `batch` independent products (1-SM kernel, EPI_F32/EPI_BF16):
  // both tensor maps are 3D {K, rows, batch} (box {64, rows, 1}) and product z
  // writes c + z * c_bstride (elements).  batch <= 1: 2D maps, one product.
  int batch;
  long long c_bstride;
  // ksplit > 1 (2D maps, EPI_F32, K steps divisible by ksplit): split-K, part z
  // of the K range writes its fp32 partial product to c + z * c_bstride.
  int ksplit;
  // zz_world > 0 (CTA-pair form): A's rows are the context-parallel all-gather
  // [world][2][c][K] (rank p's chunks p and 2 world - 1 - p), read in prompt
  // order: logical 128-row tile t of chunk j = t / zz_c128 is physical tile
  // (j < world ? 2j : 2 (2 world - 1 - j) + 1) * zz_c128 + t % zz_c128.
  int zz_world, zz_c128;
  // 1-SM kernel: B is a weight that no kernel before it on the stream writes;
  // the CTA's B boxes are prefetched into L2 before griddepcontrol.wait
  int prefetch_b;
  // 1-SM kernel, batch > 1: B is stored MN-major ([K][N] per product, N
  // contiguous; 3D map {N, K, batch}, box {64, 64, 1}), BN / 64 boxes per stage
  int b_mn;
};

// The physical 128-row tile of logical tile t in the zigzag all-gather layout
// (tiles past the 2 * world chunks map to themselves).
__host__ __device__ __forceinline__ int zigzag_tile(int t, int world, int c128) {
  if (world <= 0) return t;
  const int j = t / c128;
  if (j >= 2 * world) return t;
  return (j < world ? 2 * j : 2 * (2 * world - 1 - j) + 1) * c128 + t % c128;
}

// `name` labels the launch in the per-kernel profile (a string literal).
// `dependent`: launched as a programmatic dependent of the previous kernel on
// the stream (the kernel orders all its global accesses after
// griddepcontrol.wait, so any predecessor is safe).
cudaError_t launch_gemm(const GemmParams &p, int bn, int epi, int sms, cudaStream_t stream,
                        const char *name = nullptr, bool dependent = false);
// CTA-pair (2-SM) form, 256 x bn tiles: B's tensor map box is {64, bn / 2}.
cudaError_t launch_gemm_pair(const GemmParams &p, int bn, int epi, int sms, cudaStream_t stream,
                             const char *name = nullptr, bool dependent = false);
cudaError_t launch_rope_table(float2 *cs, int rows, int dim, float theta, cudaStream_t stream);
// Table rows of two position ranges: row j < split is position pos_a + j, row
// j >= split position pos_b + j - split.
cudaError_t launch_rope_table_rows(float2 *cs, int rows, int dim, float theta, int split, int pos_a, int pos_b,
                                   cudaStream_t stream);

}  // namespace kvl
