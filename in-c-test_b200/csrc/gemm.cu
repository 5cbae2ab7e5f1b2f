// gemm.cu -- persistent tcgen05 GEMM for the MLA projections on sm_100a:
//     C[M x N] = A[M x K] . B[N x K]^T      (A, B bf16, K-major; fp32 accumulate)
// i.e. y = x W^T for the row-major weights of the reference (KvlMlaBF16).
//
// Tile 128 x BN (BN = 256, 192 or 128), K step 64; a 4-stage TMA ring (SW128 boxes),
// one thread issuing tcgen05.mma (M=128, N=BN, K=16), the accumulator
// double-buffered in tensor memory so the epilogue of one tile overlaps the
// MMAs of the next.  Epilogues:
//   EPI_F32    C fp32 row-major (ldc elements)
//   EPI_BF16   C bf16 row-major
//   EPI_QROPE  q_proj: heads of 192 columns (128 nope + 64 rope); each rope
//              group is rotated as src/mla_prefill_streaming.c:15-29 does
//              (pairs (2i, 2i+1) -> i, 32 + i) with cos/sin from a table of
//              float2 [rows][32] (position = row); stored bf16.
// Batched mode (GemmParams::batch > 1): independent products over a third
// tensor-map coordinate, e.g. the per-head absorbed-decode products
// q_nope . W_UK and mix . W_UV^T for a batch of sequences.  Split-K mode
// (GemmParams::ksplit > 1): fp32 partial products of K ranges, summed by the
// consumer (kv_a_proj, whose 576 output columns give too few tiles to fill
// the SMs otherwise).
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2-5 epilogue (TMEM subpartition = warp % 4).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "gemm.cuh"
#include "prof.cuh"
#include "pdl.cuh"
#include "sm100.cuh"

namespace kvl {
namespace gemmk {

constexpr int kStages = 4;
constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kBMnBox = kBK * 64 * 2;     // MN-major B box: 64 K rows x 64 N columns, 8 KB

template <int BN>
struct Layout {
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t OFF_BAR = kStages * kStageBytes;
  static constexpr uint32_t kSmem = OFF_BAR + 256 + 1024;
  // two accumulators of kAccCols columns; narrow tiles take less tensor memory so
  // that two CTAs that share an SM (BN = 64: 97 KB of shared memory each) do not
  // wait for each other's allocation
  static constexpr uint32_t kAccCols = BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr uint32_t kTmemCols = 2 * kAccCols;
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

// One accumulator tile row per thread: TMEM lanes of this warp's quarter,
// BN fp32 columns -> the epilogue's output row `row`, columns nb * BN + ...
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmParams &p, uint32_t tbase, int row, bool row_ok, int nb,
                                              long long cofs = 0) {
  if constexpr (EPI == EPI_QROPE) {
    // 64-column groups: a head is 192 columns (128 nope, then 64 rope), and
    // the tile edges (multiples of BN = 192 or 256) never split a rope group
    __nv_bfloat16 *dst_row = static_cast<__nv_bfloat16 *>(p.c) + static_cast<size_t>(row) * p.ldc;
#pragma unroll 1
    for (int g = 0; g < BN / 64; ++g) {
      const int col0 = nb * BN + 64 * g;
      if (col0 >= p.N) break;
      float r[64];
      tmem_ld32(tbase + 64 * g, r);
      tmem_ld32(tbase + 64 * g + 32, r + 32);
      tmem_wait_ld();
      if (!row_ok) continue;
      __nv_bfloat16 *dst = dst_row + col0;
      if (col0 % 192 == 128) {
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
        for (int k = 0; k < 64; ++k) r[k] = outv[k];
      }
#pragma unroll
      for (int k = 0; k < 64; k += 8) {
        uint4 o;
        o.x = pack_bf16(r[k], r[k + 1]);
        o.y = pack_bf16(r[k + 2], r[k + 3]);
        o.z = pack_bf16(r[k + 4], r[k + 5]);
        o.w = pack_bf16(r[k + 6], r[k + 7]);
        *reinterpret_cast<uint4 *>(dst + k) = o;
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
          float *dst = static_cast<float *>(p.c) + cofs + static_cast<size_t>(row) * p.ldc + col0;
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
          __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(p.c) + cofs + static_cast<size_t>(row) * p.ldc + col0;
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
}

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
  const int tiles_mn = tiles_m * tiles_n;
  const bool batched = p.batch > 1;
  const int nsplit = p.ksplit > 1 ? p.ksplit : 1;
  const int tiles = tiles_mn * (batched ? p.batch : nsplit);
  const int ksteps = (p.K + kBK - 1) / kBK;
  const int kc = ksteps / nsplit;  // K steps per split (the launcher checks divisibility)

  if (p.prefetch_b && threadIdx.x == 0) {
    // the weight boxes of all this CTA's tiles stream into L2 while the
    // previous kernel on the stream drains
    tma_prefetch_desc(&p.tm_b);
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      const int z = tile / tiles_mn, nb = (tile % tiles_mn) / tiles_m;
      const int kbeg = batched ? 0 : z * kc;
      for (int ks = kbeg; ks < kbeg + kc; ++ks) {
        if (batched && p.b_mn) {
          for (int j = 0; j < BN / 64; ++j) tma_prefetch_l2_3d(&p.tm_b, nb * BN + 64 * j, ks * kBK, z);
        } else if (batched) {
          tma_prefetch_l2_3d(&p.tm_b, ks * kBK, nb * BN, z);
        } else {
          tma_prefetch_l2_2d(&p.tm_b, ks * kBK, nb * BN);
        }
      }
    }
  }
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
  // as a programmatic dependent: the set-up above overlaps the previous
  // kernel's tail; every global access (loads, epilogue stores) comes after
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int z = tile / tiles_mn, t = tile % tiles_mn;
        const int mb = t % tiles_m, nb = t / tiles_m;  // consecutive CTAs share the B tile
        const int kbeg = batched ? 0 : z * kc, kend = kbeg + kc;
        for (int ks = kbeg; ks < kend && ok; ++ks, ++it) {
          const uint32_t s = it % kStages;
          ok = mbar_wait(&B->empty[s], ((it / kStages) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
          if (!ok) break;
          uint8_t *st = smem + s * L::kStageBytes;
          mbar_arrive_expect_tx(&B->full[s], L::kStageBytes);
          if (batched) {
            tma_load_3d(st, &p.tm_a, &B->full[s], ks * kBK, mb * kBM, z);
            if (p.b_mn) {
              // BN / 64 boxes of [64 K rows][64 N columns], kBMnBox bytes apart
              for (int j = 0; j < BN / 64; ++j)
                tma_load_3d(st + kABytes + j * kBMnBox, &p.tm_b, &B->full[s], nb * BN + 64 * j, ks * kBK, z);
            } else {
              tma_load_3d(st + kABytes, &p.tm_b, &B->full[s], ks * kBK, nb * BN, z);
            }
          } else {
            tma_load_2d(st, &p.tm_a, &B->full[s], ks * kBK, mb * kBM);
            tma_load_2d(st + kABytes, &p.tm_b, &B->full[s], ks * kBK, nb * BN);
          }
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
      constexpr uint32_t idesc_k = idesc_f16(1, 1, 0, 0, kBM, BN), idesc_mn = idesc_f16(1, 1, 0, 1, kBM, BN);
      const bool b_mn = batched && p.b_mn;
      const uint32_t idesc = b_mn ? idesc_mn : idesc_k;
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++lt) {
        const uint32_t ab = lt & 1;
        ok = mbar_wait(&B->acc_empty[ab], ((lt >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
        tc_fence_after();
        const int kbeg = batched ? 0 : (tile / tiles_mn) * kc, kend = kbeg + kc;
        for (int ks = kbeg; ks < kend && ok; ++ks, ++it) {
          const uint32_t s = it % kStages;
          ok = mbar_wait(&B->full[s], (it / kStages) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_addr = s_base + s * L::kStageBytes;
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // MN-major B: K step kk is rows 16 kk.. of every box (2048 bytes
            // in), the boxes (64 N columns each) kBMnBox apart, 8-row groups
            // 1024 bytes apart
            const uint64_t bd = b_mn ? smem_desc(b_addr + kk * 2048, kBMnBox, 1024, LAYOUT_SW128)
                                     : smem_desc(b_addr + kk * 32, 16, 1024, LAYOUT_SW128);
            mma_f16_ss(tmem + ab * L::kAccCols, smem_desc(a_addr + kk * 32, 16, 1024, LAYOUT_SW128), bd, idesc,
                       (ks != kbeg || kk) ? 1u : 0u);
          }
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
      const int z = tile / tiles_mn, t = tile % tiles_mn;
      const int mb = t % tiles_m, nb = t / tiles_m;
      const uint32_t ab = lt & 1;
      bool bad = !mbar_wait(&B->acc_full[ab], (lt >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
      if (__any_sync(0xffffffffu, bad)) break;
      tc_fence_after();
      const int row = mb * kBM + 32 * sub + lane;
      const bool row_ok = row < p.M;
      const uint32_t tbase = tmem + ab * L::kAccCols + lane_base;
      epilogue_tile<BN, EPI>(p, tbase, row, row_ok, nb, (batched || nsplit > 1) ? z * p.c_bstride : 0);
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


// ---------------------------------------------------------------------------
// CTA-pair form: a cluster of two CTAs computes a 256 x BN tile with one
// M = 256 tcgen05.mma per K step (cta_group::2, issued by rank 0).  Each CTA
// loads its own 128 rows of A and its own BN / 2 rows of B, so a pair moves
// (256 + BN) x 64 elements per K step instead of 2 x (128 + BN) for two
// independent CTAs: half the B traffic per SM.
//   full[s]      (leader)  one arrival with expect_tx of both CTAs' bytes;
//                          both CTAs' copies complete on it
//   empty[s]     (each)    leader's commit, multicast to both CTAs
//   acc_full[b]  (each)    leader's commit, multicast to both CTAs
//   acc_empty[b] (leader)  one arrival per epilogue warp of both CTAs
namespace gemmk {
constexpr int kPairStages = 6;
template <int BN>
struct PairLayout {
  static constexpr uint32_t kBBytes = (BN / 2) * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t OFF_BAR = kPairStages * kStageBytes;
  static constexpr uint32_t kSmem = OFF_BAR + 256 + 1024;
};
struct PairBars {
  uint64_t full[kPairStages], empty[kPairStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
}  // namespace gemmk

template <int BN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_pair_bf16_tn_kernel(const __grid_constant__ GemmParams p) {
  using L = PairLayout<BN>;
  static_assert(sizeof(PairBars) <= 256, "barrier block");
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  PairBars *B = reinterpret_cast<PairBars *>(smem + L::OFF_BAR);
  const uint32_t s_base = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int *abort = &B->abort;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_m = (p.M + 2 * kBM - 1) / (2 * kBM);
  const int tiles_n = (p.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int ksteps = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPairStages; ++i) {
      mbar_init(&B->full[i], 1);
      mbar_init(&B->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->acc_full[i], 1);
      mbar_init(&B->acc_empty[i], 8);
    }
    mbar_init(&B->drain, 1);
    B->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&B->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem = B->tmem_base;
  // as a programmatic dependent: every global access comes after the wait
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_a);
      tma_prefetch_desc(&p.tm_b);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        const int mb = tile % tiles_m, nb = tile / tiles_m;
        for (int ks = 0; ks < ksteps && ok; ++ks, ++it) {
          const uint32_t s = it % kPairStages;
          ok = mbar_wait(&B->empty[s], ((it / kPairStages) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
          if (!ok) break;
          if (leader) mbar_arrive_expect_tx(&B->full[s], 2 * L::kStageBytes);
          const uint32_t full_l = mapa_shared(smem_u32(&B->full[s]), 0);
          uint8_t *st = smem + s * L::kStageBytes;
          tma_load_2d_pair(st, &p.tm_a, full_l, ks * kBK,
                           zigzag_tile(2 * mb + static_cast<int>(rank), p.zz_world, p.zz_c128) * kBM);
          tma_load_2d_pair(st + kABytes, &p.tm_b, full_l, ks * kBK, nb * BN + static_cast<int>(rank) * (BN / 2));
        }
      }
      if (!ok && leader) {
        for (uint32_t s = 0; s < kPairStages && s < it; ++s) {
          const uint32_t last = s + kPairStages * ((it - 1 - s) / kPairStages);
          drain_wait(&B->full[s], (last / kPairStages) & 1, p.err);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_f16(1, 1, 0, 0, 2 * kBM, BN);
      const uint64_t desc0 = smem_desc(s_base, 16, 1024, LAYOUT_SW128);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs, ++lt) {
        const uint32_t ab = lt & 1;
        ok = mbar_wait(&B->acc_empty[ab], ((lt >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
        tc_fence_after();
        for (int ks = 0; ks < ksteps && ok; ++ks, ++it) {
          const uint32_t s = it % kPairStages;
          ok = mbar_wait(&B->full[s], (it / kPairStages) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint64_t a = desc0 + ((s * L::kStageBytes) >> 4);
          const uint64_t b = a + (kABytes >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_f16_ss_pair(tmem + ab * 256, a + 2 * kk, b + 2 * kk, idesc, (ks | kk) ? 1u : 0u);
          mma_commit_pair(&B->empty[s], 0x3);
        }
        if (ok) mma_commit_pair(&B->acc_full[ab], 0x3);
      }
      mma_commit_pair(&B->drain, 0x1);
      drain_wait(&B->drain, 0, p.err);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int sub = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(32 * sub) << 16;
    uint32_t lt = 0;
    for (int tile = pair; tile < tiles; tile += npairs, ++lt) {
      const int mb = tile % tiles_m, nb = tile / tiles_m;
      const uint32_t ab = lt & 1;
      bool bad = !mbar_wait(&B->acc_full[ab], (lt >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
      if (__any_sync(0xffffffffu, bad)) break;
      tc_fence_after();
      const int row = (2 * mb + static_cast<int>(rank)) * kBM + 32 * sub + lane;
      epilogue_tile<BN, EPI>(p, tmem + ab * 256 + lane_base, row, row < p.M, nb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&B->acc_empty[ab]), 0));
    }
  }

  tc_fence_before();
  cluster_sync_all();  // the leader's MMAs into both CTAs' tensor memory have completed
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

template <int BN, int EPI>
static cudaError_t launch_gemm_t(const GemmParams &p, int sms, cudaStream_t stream, const char *name, bool dep) {
  using L = Layout<BN>;
  cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tn_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kSmem);
  if (e != cudaSuccess) return e;
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN) * (p.batch > 1 ? p.batch : 1) *
                    (p.ksplit > 1 ? p.ksplit : 1);
  const int grid = tiles < sms ? tiles : sms;
  ProfScope ps(name, stream);
  if (dep) return launch_dependent(gemm_bf16_tn_kernel<BN, EPI>, dim3(grid), dim3(192), L::kSmem, stream, p);
  gemm_bf16_tn_kernel<BN, EPI><<<grid, 192, L::kSmem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm(const GemmParams &p, int bn, int epi, int sms, cudaStream_t stream, const char *name,
                        bool dep) {
  if (!name) name = epi == EPI_QROPE ? "gemm_qrope" : "gemm_bf16";
  if (p.ksplit > 1 && (p.batch > 1 || epi != EPI_F32 || ((p.K + kBK - 1) / kBK) % p.ksplit != 0))
    return cudaErrorInvalidValue;
  if (p.b_mn && p.batch <= 1) return cudaErrorInvalidValue;
  if (epi == EPI_QROPE) {
    if (p.N % 192 != 0 || p.batch > 1) return cudaErrorInvalidValue;
    if (bn == 256) return launch_gemm_t<256, EPI_QROPE>(p, sms, stream, name, dep);
    if (bn == 192) return launch_gemm_t<192, EPI_QROPE>(p, sms, stream, name, dep);
    return cudaErrorInvalidValue;
  }
  if (bn == 256) {
    if (epi == EPI_F32) return launch_gemm_t<256, EPI_F32>(p, sms, stream, name, dep);
    if (epi == EPI_BF16) return launch_gemm_t<256, EPI_BF16>(p, sms, stream, name, dep);
  } else if (bn == 192) {
    if (epi == EPI_F32) return launch_gemm_t<192, EPI_F32>(p, sms, stream, name, dep);
    if (epi == EPI_BF16) return launch_gemm_t<192, EPI_BF16>(p, sms, stream, name, dep);
  } else if (bn == 128) {
    if (epi == EPI_F32) return launch_gemm_t<128, EPI_F32>(p, sms, stream, name, dep);
    if (epi == EPI_BF16) return launch_gemm_t<128, EPI_BF16>(p, sms, stream, name, dep);
  } else if (bn == 64) {
    if (epi == EPI_F32) return launch_gemm_t<64, EPI_F32>(p, sms, stream, name, dep);
  }
  return cudaErrorInvalidValue;
}

template <int BN, int EPI>
static cudaError_t launch_gemm_pair_t(const GemmParams &p, int sms, cudaStream_t stream, const char *name, bool dep) {
  using L = PairLayout<BN>;
  static_assert(L::kSmem <= 232448, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(gemm_pair_bf16_tn_kernel<BN, EPI>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem);
  if (e != cudaSuccess) return e;
  const int tiles = ((p.M + 2 * kBM - 1) / (2 * kBM)) * ((p.N + BN - 1) / BN);
  int pairs = sms / 2;
  if (pairs > tiles) pairs = tiles;
  if (pairs < 1) pairs = 1;
  ProfScope ps(name, stream);
  if (dep) return launch_dependent(gemm_pair_bf16_tn_kernel<BN, EPI>, dim3(2 * pairs), dim3(192), L::kSmem, stream, p);
  gemm_pair_bf16_tn_kernel<BN, EPI><<<2 * pairs, 192, L::kSmem, stream>>>(p);
  return cudaGetLastError();
}

// B's tensor map box must be {64, bn / 2} rows for the pair form.
cudaError_t launch_gemm_pair(const GemmParams &p, int bn, int epi, int sms, cudaStream_t stream, const char *name,
                             bool dep) {
  if (bn != 256 || p.batch > 1 || p.ksplit > 1) return cudaErrorInvalidValue;
  if (!name) name = epi == EPI_QROPE ? "gemm_qrope" : "gemm_bf16";
  if (epi == EPI_QROPE) {
    if (p.N % 192 != 0) return cudaErrorInvalidValue;
    return launch_gemm_pair_t<256, EPI_QROPE>(p, sms, stream, name, dep);
  }
  if (epi == EPI_F32) return launch_gemm_pair_t<256, EPI_F32>(p, sms, stream, name, dep);
  if (epi == EPI_BF16) return launch_gemm_pair_t<256, EPI_BF16>(p, sms, stream, name, dep);
  return cudaErrorInvalidValue;
}

// Inverse frequencies theta^(-2i/dim), i < dim/2, computed on the host (the
// reference's own expression, src/mla_compressed_state.c:12-13).
struct RopeFreqs {
  double inv[128];
};

// cos/sin of pos * inv_freq[i], one table row per position: row j < split is
// position pos_a + j, row j >= split position pos_b + j - split (double angle,
// float result, as src/mla_compressed_state.c:14-16).
__global__ void rope_table_kernel(float2 *cs, int rows, int half, const __grid_constant__ RopeFreqs fr, int split,
                                  int pos_a, int pos_b) {
  const long long n = static_cast<long long>(rows) * half;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(i / half), k = static_cast<int>(i % half);
    const int pos = j < split ? pos_a + j : pos_b + (j - split);
    const double ang = static_cast<double>(pos) * fr.inv[k];
    double sn, cn;
    sincos(ang, &sn, &cn);
    cs[i] = make_float2(static_cast<float>(cn), static_cast<float>(sn));
  }
}

cudaError_t launch_rope_table_rows(float2 *cs, int rows, int dim, float theta, int split, int pos_a, int pos_b,
                                   cudaStream_t stream) {
  if (dim <= 0 || dim > 256 || (dim & 1) || rows <= 0 || pos_a < 0 || pos_b < 0) return cudaErrorInvalidValue;
  const int half = dim / 2;
  RopeFreqs fr;
  for (int k = 0; k < half; ++k)
    fr.inv[k] = std::pow(static_cast<double>(theta), -(static_cast<double>(2 * k) / static_cast<double>(dim)));
  const long long n = static_cast<long long>(rows) * half;
  const int grid = static_cast<int>((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
  ProfScope ps("rope_table", stream);
  rope_table_kernel<<<grid, 256, 0, stream>>>(cs, rows, half, fr, split, pos_a, pos_b);
  return cudaGetLastError();
}

cudaError_t launch_rope_table(float2 *cs, int rows, int dim, float theta, cudaStream_t stream) {
  return launch_rope_table_rows(cs, rows, dim, theta, rows, 0, 0, stream);
}

}  // namespace kvl
