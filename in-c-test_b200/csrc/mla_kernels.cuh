// mla_kernels.cuh -- launchers of the decode-step kernels in mla_kernels.cu.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace kvl {

// ref_order: sum in the reference AVX2 matvec's order (bit-identical rows;
// used for kv_a_proj, whose output becomes the stored state row).
cudaError_t gemv_bf16(float *y, const float *x, const uint16_t *W, int in, int out, int n, cudaStream_t s,
                      bool ref_order = false);
cudaError_t append_bf16(uint16_t *kv, long long row0, const float *ka, const uint16_t *norm_w, int n, int R,
                        int DR, int pos0, float eps, float theta, float *rows_f32, cudaStream_t s,
                        const long long *row_of = nullptr, const int *pos_of = nullptr, int parts = 1,
                        long long part_stride = 0);
cudaError_t append_q8(int8_t *lat8, float *lscale, uint16_t *rope16, long long row0, const float *ka,
                      const uint16_t *norm_w, int n, int R, int DR, int pos0, float eps, float theta,
                      cudaStream_t s, const long long *row_of = nullptr, const int *pos_of = nullptr,
                      int parts = 1, long long part_stride = 0);
// Prefill rows [0, n) of a bf16 [n][576] pool (Kimi shape), RoPE from a [n][32] cos/sin table.
// parts > 1: ka holds split-K partial products `part_stride` floats apart,
// summed in order before the normalisation.
cudaError_t append_rows_bf16(uint16_t *pool, const float *ka, const uint16_t *norm_w, const float2 *cs, int n,
                             float eps, cudaStream_t s, int parts = 1, long long part_stride = 0);
// q bf16 [n][16][192] = the sum of `np` fp32 partial products [n][16 * 192]
// (`stride` floats apart) with RoPE (cos/sin cs [n][32]) on each head's last
// 64 columns, as the q_proj GEMM's EPI_QROPE epilogue computes it.
cudaError_t sum_parts_qrope(uint16_t *q, const float *parts, int np, long long stride, const float2 *cs, int n,
                            cudaStream_t s);
cudaError_t absorb(float *qabs, const float *q, const uint16_t *kvb, int n, int NH, int DN, int DV, int DR, int R,
                   int pos0, float theta, cudaStream_t s, const int *pos_of = nullptr);
cudaError_t vup(float *ho, const float *mix, const uint16_t *kvb, int n, int NH, int DN, int DV, int R,
                cudaStream_t s);
cudaError_t q_split(uint16_t *qn, float *qabs, const float *q, int parts, long long part_stride, int n, int NH,
                    int DN, int DR, int R, float theta, const int *pos_of, cudaStream_t s);
cudaError_t sum_parts(float *dst, const float *src, int parts, long long stride, long long n, cudaStream_t s);
cudaError_t mix_heads_bf16(uint16_t *out, const float *mix, int n, int NH, int R, cudaStream_t s);
cudaError_t quantize_rows(int8_t *q, float *scale, const float *x, int rows, int R, cudaStream_t s);
cudaError_t dequant(float *out, const int8_t *q, const float *scale, long long rows, int R, cudaStream_t s);
cudaError_t bf16_rne(uint16_t *out, const float *x, long long n, cudaStream_t s);
cudaError_t bf16_to_f32(float *out, const uint16_t *x, long long n, cudaStream_t s);
cudaError_t f32_to_bf16(uint16_t *out, const float *x, long long n, cudaStream_t s);

}  // namespace kvl
