// gemm.cu -- persistent tcgen05 GEMM for the MLA projections on sm_100a:
//     C[M x N] = A[M x K] . B[N x K]^T      (A, B bf16, K-major; fp32 accumulate)
// i.e. y = x W^T for the row-major weights of the reference (KvlMlaBF16).
//
// Tile 128 x BN (BN = 256 or 192), K step 64; a 4-stage TMA ring (SW128 boxes),
// one thread issuing tcgen05.mma (M=128, N=BN, K=16), the accumulator
// double-buffered in tensor memory so the epilogue of one tile overlaps the
// MMAs of the next.  Epilogues:
//   EPI_F32    C fp32 row-major (ldc elements)
//   EPI_BF16   C bf16 row-major
//   EPI_QROPE  BN = 192 = one head of q_proj (128 nope + 64 rope columns): the
//              rope half is rotated as src/mla_prefill_streaming.c:15-29 does
//              (pairs (2i, 2i+1) -> i, 32 + i) with cos/sin from a table of
//              float2 [rows][32] (position = row), and the head is stored bf16.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2-5 epilogue (TMEM subpartition = warp % 4).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "gemm.cuh"
#include "prof.cuh"
#include "sm100.cuh"

namespace kvl {
namespace gemmk {

constexpr int kStages = 4;
constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB

template <int BN>
struct Layout {
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t OFF_BAR = kStages * kStageBytes;
  static constexpr uint32_t kSmem = OFF_BAR + 256 + 1024;
  static constexpr uint32_t kTmemCols = 512;
};

struct Bars {
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

}  // namespace gemmk

using namespace gemmk;

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1) gemm_bf16_tn_kernel(const __grid_constant__ GemmParams p) {
  using L = Layout<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars *B = reinterpret_cast<Bars *>(smem + L::OFF_BAR);
  const uint32_t s_base = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int *abort = &B->abort;
  const int tiles_m = (p.M + kBM - 1) / kBM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int ksteps = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&B->full[i], 1);
      mbar_init(&B->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->acc_full[i], 1);
      mbar_init(&B->acc_empty[i], 4);
    }
    mbar_init(&B->drain, 1);
    B->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&B->tmem_base, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int mb = tile % tiles_m, nb = tile / tiles_m;  // consecutive CTAs share the B tile
        for (int ks = 0; ks < ksteps && ok; ++ks, ++it) {
          const uint32_t s = it % kStages;
          ok = mbar_wait(&B->empty[s], ((it / kStages) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
          if (!ok) break;
          uint8_t *st = smem + s * L::kStageBytes;
          mbar_arrive_expect_tx(&B->full[s], L::kStageBytes);
          tma_load_2d(st, &p.tm_a, &B->full[s], ks * kBK, mb * kBM);
          tma_load_2d(st + kABytes, &p.tm_b, &B->full[s], ks * kBK, nb * BN);
        }
      }
      if (!ok) {
        for (uint32_t s = 0; s < kStages && s < it; ++s) {
          const uint32_t last = s + kStages * ((it - 1 - s) / kStages);
          drain_wait(&B->full[s], (last / kStages) & 1, p.err);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(1, 1, 0, 0, kBM, BN);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++lt) {
        const uint32_t ab = lt & 1;
        ok = mbar_wait(&B->acc_empty[ab], ((lt >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
        tc_fence_after();
        for (int ks = 0; ks < ksteps && ok; ++ks, ++it) {
          const uint32_t s = it % kStages;
          ok = mbar_wait(&B->full[s], (it / kStages) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_addr = s_base + s * L::kStageBytes;
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_f16_ss(tmem + ab * 256, smem_desc(a_addr + kk * 32, 16, 1024, LAYOUT_SW128),
                       smem_desc(b_addr + kk * 32, 16, 1024, LAYOUT_SW128), idesc, (ks | kk) ? 1u : 0u);
          mma_commit(&B->empty[s]);
        }
        if (ok) mma_commit(&B->acc_full[ab]);
      }
      mma_commit(&B->drain);
      drain_wait(&B->drain, 0, p.err);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int sub = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * sub) << 16;
    uint32_t lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
      const int mb = tile % tiles_m, nb = tile / tiles_m;
      const uint32_t ab = lt & 1;
      bool bad = !mbar_wait(&B->acc_full[ab], (lt >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
      if (__any_sync(0xffffffffu, bad)) break;
      tc_fence_after();
      const int row = mb * kBM + 32 * sub + lane;
      const bool row_ok = row < p.M;
      const uint32_t tbase = tmem + ab * 256 + lane_base;
      if constexpr (EPI == EPI_QROPE) {
        // one head: 128 nope columns then 64 interleaved rope columns
        __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(p.c) + static_cast<size_t>(row) * p.ldc + nb * BN;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_ld32(tbase + 32 * c, v);
          tmem_wait_ld();
          if (row_ok) {
#pragma unroll
            for (int k = 0; k < 32; k += 8) {
              uint4 o;
              o.x = pack_bf16(v[k], v[k + 1]);
              o.y = pack_bf16(v[k + 2], v[k + 3]);
              o.z = pack_bf16(v[k + 4], v[k + 5]);
              o.w = pack_bf16(v[k + 6], v[k + 7]);
              *reinterpret_cast<uint4 *>(dst + 32 * c + k) = o;
            }
          }
        }
        float r[64];
        tmem_ld32(tbase + 128, r);
        tmem_ld32(tbase + 160, r + 32);
        tmem_wait_ld();
        if (row_ok) {
          const float2 *cs = p.rope_cs + static_cast<size_t>(row) * 32;
          float outv[64];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float2 t = cs[i];
            const float a = r[2 * i], b = r[2 * i + 1];
            outv[i] = __fsub_rn(__fmul_rn(a, t.x), __fmul_rn(b, t.y));
            outv[32 + i] = __fadd_rn(__fmul_rn(b, t.x), __fmul_rn(a, t.y));
          }
#pragma unroll
          for (int k = 0; k < 64; k += 8) {
            uint4 o;
            o.x = pack_bf16(outv[k], outv[k + 1]);
            o.y = pack_bf16(outv[k + 2], outv[k + 3]);
            o.z = pack_bf16(outv[k + 4], outv[k + 5]);
            o.w = pack_bf16(outv[k + 6], outv[k + 7]);
            *reinterpret_cast<uint4 *>(dst + 128 + k) = o;
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float v[32];
          tmem_ld32(tbase + 32 * c, v);
          tmem_wait_ld();
          const int col0 = nb * BN + 32 * c;
          if (row_ok && col0 < p.N) {
            const bool full = col0 + 32 <= p.N;
            if constexpr (EPI == EPI_F32) {
              float *dst = static_cast<float *>(p.c) + static_cast<size_t>(row) * p.ldc + col0;
              if (full) {
#pragma unroll
                for (int k = 0; k < 32; k += 4)
                  *reinterpret_cast<float4 *>(dst + k) = make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
              } else {
#pragma unroll
                for (int k = 0; k < 32; ++k)
                  if (col0 + k < p.N) dst[k] = v[k];
              }
            } else {
              __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(p.c) + static_cast<size_t>(row) * p.ldc + col0;
              if (full) {
#pragma unroll
                for (int k = 0; k < 32; k += 8) {
                  uint4 o;
                  o.x = pack_bf16(v[k], v[k + 1]);
                  o.y = pack_bf16(v[k + 2], v[k + 3]);
                  o.z = pack_bf16(v[k + 4], v[k + 5]);
                  o.w = pack_bf16(v[k + 6], v[k + 7]);
                  *reinterpret_cast<uint4 *>(dst + k) = o;
                }
              } else {
#pragma unroll
                for (int k = 0; k < 32; ++k)
                  if (col0 + k < p.N) dst[k] = __float2bfloat16_rn(v[k]);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Layout<BN>::kTmemCols);
  }
}

template <int BN, int EPI>
static cudaError_t launch_gemm_t(const GemmParams &p, int sms, cudaStream_t stream, const char *name) {
  using L = Layout<BN>;
  cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tn_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kSmem);
  if (e != cudaSuccess) return e;
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN);
  const int grid = tiles < sms ? tiles : sms;
  ProfScope ps(name, stream);
  gemm_bf16_tn_kernel<BN, EPI><<<grid, 192, L::kSmem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmParams &p, int bn, int epi, int sms, cudaStream_t stream) {
  if (epi == EPI_QROPE) return bn == 192 ? launch_gemm_t<192, EPI_QROPE>(p, sms, stream, "gemm_qrope") : cudaErrorInvalidValue;
  if (bn == 256) {
    if (epi == EPI_F32) return launch_gemm_t<256, EPI_F32>(p, sms, stream, "gemm_bf16");
    if (epi == EPI_BF16) return launch_gemm_t<256, EPI_BF16>(p, sms, stream, "gemm_bf16");
  } else if (bn == 192) {
    if (epi == EPI_F32) return launch_gemm_t<192, EPI_F32>(p, sms, stream, "gemm_bf16");
    if (epi == EPI_BF16) return launch_gemm_t<192, EPI_BF16>(p, sms, stream, "gemm_bf16");
  }
  return cudaErrorInvalidValue;
}

// cos/sin of pos * theta^(-2i/dim) for i < dim/2 and pos < rows: the angle
// arithmetic of src/mla_compressed_state.c:8-22 (double angle, float result).
__global__ void rope_table_kernel(float2 *cs, int rows, int dim, float theta) {
  const int half = dim / 2;
  const long long n = static_cast<long long>(rows) * half;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int pos = static_cast<int>(i / half), k = static_cast<int>(i % half);
    const double inv_freq = pow(static_cast<double>(theta), -(static_cast<double>(2 * k) / static_cast<double>(dim)));
    const double ang = static_cast<double>(pos) * inv_freq;
    cs[i] = make_float2(static_cast<float>(cos(ang)), static_cast<float>(sin(ang)));
  }
}

cudaError_t launch_rope_table(float2 *cs, int rows, int dim, float theta, cudaStream_t stream) {
  const long long n = static_cast<long long>(rows) * (dim / 2);
  const int grid = static_cast<int>((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
  ProfScope ps("rope_table", stream);
  rope_table_kernel<<<grid, 256, 0, stream>>>(cs, rows, dim, theta);
  return cudaGetLastError();
}

}  // namespace kvl
