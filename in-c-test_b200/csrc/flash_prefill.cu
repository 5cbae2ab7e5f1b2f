// flash_prefill.cu -- causal MLA prefill attention on sm_100a (the attention
// of src/mla_prefill_streaming.c:141-193 in the non-absorbed form):
//     s_tj = (q_nope_t . k_nope_j + q_rope_t . k_rope_j) * scale,   j <= t
//     o_t  = sum_j softmax_j(s_t) v_j
// per head, with q_rope/k_rope already rotated, k_rope shared by the heads.
//
// Work item = (head, 128-query tile); items are dealt to persistent CTAs in
// snake order of decreasing cost (a query tile i attends i + 1 key tiles).
// Per key tile: S[128 q x 128 k] = Q . K^T on tcgen05 (12 MMAs, M=N=128),
// softmax by four warps with one thread per query row (no cross-thread
// reductions; lazy rescale of the running max, threshold 2^8), P (bf16) to
// shared memory, O[128 q x 128 dv] += P . V (8 MMAs, V MN-major).  S is
// double-buffered in tensor memory so the scores of tile j + 1 are computed
// while the softmax of tile j runs.
//
// Shared memory: Q 48 KB (3 SW128 boxes), K ring 2 x 48 KB (k_nope 2 boxes +
// k_rope 1 box), V 32 KB (2 boxes), P 32 KB (2 boxes).
// Roles (256 threads): warp 0 TMA for Q and K, warp 2 TMA for V, warp 1 TMEM
// owner + MMA issuer, warps 4-7 softmax and epilogue (TMEM subpartitions 0-3;
// thread = query row).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "flash_prefill.cuh"
#include "prof.cuh"
#include "sm100.cuh"

namespace kvl {
namespace fpre {

constexpr int kT = 128;                  // queries / keys per tile
constexpr uint32_t kBox = kT * 128;      // 128 rows x 64 bf16 = 16 KB
constexpr int kKStages = 2;
constexpr uint32_t OFF_Q = 0;                         // 3 boxes
constexpr uint32_t OFF_K = OFF_Q + 3 * kBox;          // kKStages x 3 boxes
constexpr uint32_t OFF_V = OFF_K + kKStages * 3 * kBox;  // 2 boxes
constexpr uint32_t OFF_P = OFF_V + 2 * kBox;          // 2 boxes
constexpr uint32_t OFF_BAR = OFF_P + 2 * kBox;

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full, v_empty;
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full, p_empty;
  uint64_t o_full, o_empty, drain;
  uint32_t tmem_base;
  int abort;
};

constexpr uint32_t kSmem = OFF_BAR + sizeof(Bars) + 1024;
static_assert(kSmem <= 232448, "shared memory budget");
constexpr uint32_t kTmemCols = 512;  // S: 2 x 128 columns; O: 128 columns at 256
constexpr uint32_t kColO = 256;

// Item k of the CTA: snake order over the items sorted by decreasing cost.
__device__ __forceinline__ bool item_of(int k, int grid, int cta, int n_items, int nq, int &head, int &qt) {
  // one item per CTA per lap, the lap direction alternating
  const int pos = (k & 1) ? (k + 1) * grid - 1 - cta : k * grid + cta;
  if (pos >= n_items) return false;
  qt = nq - 1 - pos / 16;  // 16 heads per cost level
  head = pos % 16;
  return true;
}

}  // namespace fpre

using namespace fpre;

__global__ void __launch_bounds__(256, 1) flash_prefill_kernel(const __grid_constant__ FlashParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars *B = reinterpret_cast<Bars *>(smem + OFF_BAR);
  const uint32_t s_base = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int *abort = &B->abort;
  const int nq = (p.S + kT - 1) / kT;
  const int n_items = nq * 16;

  if (threadIdx.x == 0) {
    mbar_init(&B->q_full, 1);
    mbar_init(&B->q_empty, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&B->k_full[i], 1);
      mbar_init(&B->k_empty[i], 1);
    }
    mbar_init(&B->v_full, 1);
    mbar_init(&B->v_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->s_full[i], 1);
      mbar_init(&B->s_empty[i], 4);
    }
    mbar_init(&B->p_full, 4);
    mbar_init(&B->p_empty, 1);
    mbar_init(&B->o_full, 1);
    mbar_init(&B->o_empty, 4);
    mbar_init(&B->drain, 1);
    B->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&B->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B->tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_kv);
      tma_prefetch_desc(&p.tm_kr);
      uint32_t kt = 0;  // key tiles issued by this CTA
      bool ok = true;
      int head, qt;
      for (int k = 0; ok && item_of(k, gridDim.x, blockIdx.x, n_items, nq, head, qt); ++k) {
        ok = mbar_wait(&B->q_empty, (k & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
        mbar_arrive_expect_tx(&B->q_full, 3 * kBox);
        for (int b = 0; b < 3; ++b) tma_load_3d(smem + OFF_Q + b * kBox, &p.tm_q, &B->q_full, 64 * b, head, qt * kT);
        for (int j = 0; j <= qt && ok; ++j, ++kt) {
          const uint32_t s = kt % kKStages;
          ok = mbar_wait(&B->k_empty[s], ((kt / kKStages) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
          if (!ok) break;
          uint8_t *kd = smem + OFF_K + s * 3 * kBox;
          mbar_arrive_expect_tx(&B->k_full[s], 3 * kBox);
          tma_load_3d(kd, &p.tm_kv, &B->k_full[s], 0, head, j * kT);
          tma_load_3d(kd + kBox, &p.tm_kv, &B->k_full[s], 64, head, j * kT);
          tma_load_2d(kd + 2 * kBox, &p.tm_kr, &B->k_full[s], p.kr_col, j * kT);
        }
      }
      if (!ok) {
        for (uint32_t s = 0; s < kKStages && s < kt; ++s) {
          const uint32_t last = s + kKStages * ((kt - 1 - s) / kKStages);
          drain_wait(&B->k_full[s], (last / kKStages) & 1, p.err);
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- V producer
    // (its own warp: the single V buffer must not hold back the K prefetch)
    if (lane == 0) {
      uint32_t kt = 0;
      bool ok = true;
      int head, qt;
      for (int k = 0; ok && item_of(k, gridDim.x, blockIdx.x, n_items, nq, head, qt); ++k) {
        for (int j = 0; j <= qt && ok; ++j, ++kt) {
          ok = mbar_wait(&B->v_empty, (kt & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
          if (!ok) break;
          mbar_arrive_expect_tx(&B->v_full, 2 * kBox);
          tma_load_3d(smem + OFF_V, &p.tm_kv, &B->v_full, 128, head, j * kT);
          tma_load_3d(smem + OFF_V + kBox, &p.tm_kv, &B->v_full, 192, head, j * kT);
        }
      }
      if (!ok && kt > 0) drain_wait(&B->v_full, (kt - 1) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(1, 1, 0, 0, kT, kT);   // A = Q (K-major), B = K (K-major)
      constexpr uint32_t idesc_pv = idesc_f16(1, 1, 0, 1, kT, 128);  // A = P (K-major), B = V (MN-major)
      uint32_t kt = 0;
      bool ok = true;
      int head, qt;
      auto issue_pv = [&](uint32_t jt, bool first, int item) -> bool {
        if (!mbar_wait(&B->p_full, jt & 1, abort, p.err, ERR_TIMEOUT_FULL)) return false;
        if (!mbar_wait(&B->v_full, jt & 1, abort, p.err, ERR_TIMEOUT_FULL)) return false;
        if (first && item > 0 && !mbar_wait(&B->o_empty, (item - 1) & 1, abort, p.err, ERR_TIMEOUT_FULL))
          return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk) {
          const uint64_t a = smem_desc(s_base + OFF_P + (kk >> 2) * kBox + (kk & 3) * 32, 16, 1024, LAYOUT_SW128);
          const uint64_t b = smem_desc(s_base + OFF_V + kk * 2048, kBox, 1024, LAYOUT_SW128);
          mma_f16_ss(tmem + kColO, a, b, idesc_pv, (first && kk == 0) ? 0u : 1u);
        }
        mma_commit(&B->p_empty);
        mma_commit(&B->v_empty);
        return true;
      };
      for (int k = 0; ok && item_of(k, gridDim.x, blockIdx.x, n_items, nq, head, qt); ++k) {
        ok = mbar_wait(&B->q_full, k & 1, abort, p.err, ERR_TIMEOUT_FULL);
        for (int j = 0; j <= qt && ok; ++j, ++kt) {
          const uint32_t sb = kt & 1, s = kt % kKStages;
          ok = mbar_wait(&B->s_empty[sb], ((kt >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY) &&
               mbar_wait(&B->k_full[s], (kt / kKStages) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint32_t kaddr = s_base + OFF_K + s * 3 * kBox;
#pragma unroll
          for (int b = 0; b < 3; ++b)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16_ss(tmem + sb * 128, smem_desc(s_base + OFF_Q + b * kBox + kk * 32, 16, 1024, LAYOUT_SW128),
                         smem_desc(kaddr + b * kBox + kk * 32, 16, 1024, LAYOUT_SW128), idesc_qk,
                         (b | kk) ? 1u : 0u);
          mma_commit(&B->s_full[sb]);
          mma_commit(&B->k_empty[s]);
          if (j == qt) mma_commit(&B->q_empty);
          if (j > 0) ok = issue_pv(kt - 1, j == 1, k);
        }
        if (!ok) break;
        ok = issue_pv(kt - 1, qt == 0, k);
        if (ok) mma_commit(&B->o_full);
      }
      mma_commit(&B->drain);
      drain_wait(&B->drain, 0, p.err);
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int w = warp - 4;
    const int tt = 32 * w + lane;  // query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * w) << 16;
    uint32_t kt = 0;
    int head, qt;
    bool bad = false;
    for (int k = 0; !bad && item_of(k, gridDim.x, blockIdx.x, n_items, nq, head, qt); ++k) {
      const int qrow = qt * kT + tt;
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j <= qt; ++j, ++kt) {
        const uint32_t sb = kt & 1;
        bad = !mbar_wait(&B->s_full[sb], (kt >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (__any_sync(0xffffffffu, bad)) { bad = true; break; }
        tc_fence_after();
        float s[kT];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tmem + sb * 128 + 32 * c + lane_base, s + 32 * c);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->s_empty[sb]);
        // causal mask on the diagonal tile, key bound on the last
        const int kbase = j * kT;
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < kT; ++c) {
          const int key = kbase + c;
          const bool ok_key = key <= qrow && key < p.S;
          s[c] = ok_key ? s[c] * p.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
        const bool need = mx > m_ref + 8.0f;
        if (__any_sync(0xffffffffu, need)) {
          const float mn = fmaxf(m_ref, mx);
          const float alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - mn);
          if (j > 0) {
            // rescale this row of O once P.V(j-1) has landed
            bad = !mbar_wait(&B->p_empty, (kt - 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
            if (__any_sync(0xffffffffu, bad)) { bad = true; break; }
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              float o[32];
              tmem_ld32(tmem + kColO + 32 * c + lane_base, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= alpha;
              tmem_st32(tmem + kColO + 32 * c + lane_base, o);
            }
            tmem_wait_st();
          }
          l *= alpha;
          m_ref = mn;
        }
        float rowsum = 0.f;
#pragma unroll
        for (int c = 0; c < kT; ++c) {
          s[c] = exp2f(s[c] - m_ref);
          rowsum += s[c];
        }
        l += rowsum;
        // P is single-buffered: wait for P.V(j-1) before overwriting it
        bad = !mbar_wait(&B->p_empty, (kt & 1) ^ 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (__any_sync(0xffffffffu, bad)) { bad = true; break; }
#pragma unroll
        for (int c8 = 0; c8 < kT / 8; ++c8) {
          uint4 o;
          o.x = pack_bf16(s[8 * c8], s[8 * c8 + 1]);
          o.y = pack_bf16(s[8 * c8 + 2], s[8 * c8 + 3]);
          o.z = pack_bf16(s[8 * c8 + 4], s[8 * c8 + 5]);
          o.w = pack_bf16(s[8 * c8 + 6], s[8 * c8 + 7]);
          *reinterpret_cast<uint4 *>(smem + OFF_P + (c8 >> 3) * kBox + sw128_offset(tt, (c8 & 7) * 8)) = o;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->p_full);
      }
      if (bad) break;
      // ---- epilogue: o = O / l as bf16 into out[row][head][0:128]
      bad = !mbar_wait(&B->o_full, k & 1, abort, p.err, ERR_TIMEOUT_MMA);
      if (__any_sync(0xffffffffu, bad)) break;
      tc_fence_after();
      const float inv = 1.0f / l;
      __nv_bfloat16 *dst = p.out + (static_cast<size_t>(qrow) * 16 + head) * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(tmem + kColO + 32 * c + lane_base, o);
        tmem_wait_ld();
        if (qrow < p.S) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = pack_bf16(o[i] * inv, o[i + 1] * inv);
            v.y = pack_bf16(o[i + 2] * inv, o[i + 3] * inv);
            v.z = pack_bf16(o[i + 4] * inv, o[i + 5] * inv);
            v.w = pack_bf16(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4 *>(dst + 32 * c + i) = v;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->o_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

cudaError_t launch_flash_prefill(const FlashParams &p, int sms, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  const int items = ((p.S + kT - 1) / kT) * 16;
  const int grid = items < sms ? items : sms;
  ProfScope ps("flash_prefill", stream);
  flash_prefill_kernel<<<grid, 256, kSmem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace kvl
