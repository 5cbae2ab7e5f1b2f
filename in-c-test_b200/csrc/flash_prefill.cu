// flash_prefill.cu -- causal MLA prefill attention on sm_100a (the attention
// of src/mla_prefill_streaming.c:141-193 in the non-absorbed form):
//     s_tj = (q_nope_t . k_nope_j + q_rope_t . k_rope_j) * scale,   j <= t
//     o_t  = sum_j softmax_j(s_t) v_j
// per head, with q_rope/k_rope already rotated, k_rope shared by the heads.
//
// Work item = (head, block of 256 queries) = two 128-query tiles Q0, Q1 that
// share every key/value tile the CTA loads.  Items go to persistent CTAs in
// snake order of decreasing cost.  Per key tile j:
//     S0 = Q0 K_j^T, S1 = Q1 K_j^T      (12 tcgen05 MMAs each, M = N = 128)
//     O0 += P0 V_j,  O1 += P1 V_j       (8 MMAs each; P read from tensor memory)
// Two softmax warpgroups (one per query tile, thread = query row) ping-pong:
// while group 0 turns S0 into P0 the tensor core runs P1 V and Q1 K^T, and
// the other way round.  P is written back as bf16 over the first 64 columns
// of its own S, so tensor memory holds S0 | S1 | O0 | O1 (4 x 128 columns).
// The running max is rescaled lazily (only when it grows by more than 2^8).
// The causal mask and the sequence bound are applied on the last key tile of
// each query tile only; all earlier tiles are entirely visible.
//
// Shared memory: Q0, Q1 (3 SW128 boxes of 128 rows x 64 each), and a ring of
// 8 boxes through which the key tiles (k_nope lo | k_nope hi | k_rope) and
// value tiles (v lo | v hi) stream in consumption order.  The two value
// boxes of one tile sit in consecutive ring slots; when the pair wraps past
// the end of the ring the low half goes to the lower slot, so one MN-major
// descriptor (LBO = the distance between the halves) always covers V.
// Roles (384 threads): warps 0-3 softmax of Q0, warps 4-7 softmax of Q1
// (TMEM lanes 32 * (warp % 4)), warp 8 TMA producer, warp 9 TMEM owner and
// MMA issuer, warps 10-11 idle.  Every wait is bounded and reports through p.err.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "flash_prefill.cuh"
#include "prof.cuh"
#include "sm100.cuh"

namespace kvl {
namespace fpre {

constexpr int kT = 128;                   // queries / keys per tile
constexpr uint32_t kBox = kT * 128;       // 128 rows x 64 bf16 = 16 KB
constexpr uint32_t kSlots = 8;            // ring of boxes
constexpr uint32_t OFF_Q = 0;             // Q0: 3 boxes, Q1: 3 boxes
constexpr uint32_t OFF_RING = 6 * kBox;
constexpr uint32_t OFF_BAR = OFF_RING + kSlots * kBox;
constexpr int kThreads = 384;
// Register split (setmaxnreg): the two softmax warpgroups grow to kRegsSoftmax,
// the producer / MMA warpgroup shrinks to kRegsOther.  The sum must not exceed
// what the block was launched with (threads x registers per thread), which the
// host checks before every launch.
constexpr int kRegsSoftmax = 184;
constexpr int kRegsOther = 136;
constexpr int kRegsNeeded = 256 * kRegsSoftmax + 128 * kRegsOther;

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t full[kSlots], empty[kSlots];
  uint64_t s_full[2], p_full[2], o_full[2], o_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

constexpr uint32_t kSmem = OFF_BAR + sizeof(Bars) + 1024;
static_assert(kSmem <= 232448, "shared memory budget");
constexpr uint32_t kTmemCols = 512;  // S0 @0, S1 @128, O0 @256, O1 @384

// Item k of the CTA: snake order over the items sorted by decreasing cost
// (a 256-query block b attends 2b + 2 key tiles).
__device__ __forceinline__ bool item_of(int k, int grid, int cta, int n_items, int nb, int &head, int &blk) {
  const int pos = (k & 1) ? (k + 1) * grid - 1 - cta : k * grid + cta;
  if (pos >= n_items) return false;
  blk = nb - 1 - pos / 16;
  head = pos % 16;
  return true;
}

// Position of the ring box with sequence number n.
__device__ __forceinline__ uint32_t slot_of(uint32_t n) { return n % kSlots; }
__device__ __forceinline__ uint32_t use_of(uint32_t n) { return n / kSlots; }

__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// (a0, a1) * (b, b) + (c, c) on the paired fp32 path.
__device__ __forceinline__ void ffma2(float &d0, float &d1, float a0, float a1, float b, float c) {
  uint64_t a, bb, cc, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(bb) : "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(cc) : "f"(c));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(bb), "l"(cc));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ void fadd2(float &a0, float &a1, float b0, float b1) {
  uint64_t a, b, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(d));
}

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t *v) {
  tmem_st32(taddr, reinterpret_cast<const float *>(v));
}

}  // namespace fpre

using namespace fpre;

__global__ void __launch_bounds__(kThreads, 1) flash_prefill_kernel(const __grid_constant__ FlashParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars *B = reinterpret_cast<Bars *>(smem + OFF_BAR);
  const uint32_t s_base = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int *abort = &B->abort;
  const int nkv = (p.S + kT - 1) / kT;           // key tiles
  const int nb = (p.S + 2 * kT - 1) / (2 * kT);  // 256-query blocks
  const int n_items = nb * 16;

  if (threadIdx.x == 0) {
    mbar_init(&B->q_full, 1);
    mbar_init(&B->q_empty, 1);
    for (uint32_t i = 0; i < kSlots; ++i) {
      mbar_init(&B->full[i], 1);
      mbar_init(&B->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->s_full[i], 1);
      mbar_init(&B->p_full[i], 4);
      mbar_init(&B->o_full[i], 1);
      mbar_init(&B->o_empty[i], 4);
    }
    mbar_init(&B->drain, 1);
    B->abort = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&B->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B->tmem_base;

  if (warp >= 8) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsOther));
  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_kv);
      tma_prefetch_desc(&p.tm_kr);
      uint32_t seq = 0;  // ring boxes issued
      uint32_t q_issued = 0;
      int k = 0;
      bool ok = true;
      int head, blk;
      auto take = [&](uint32_t &s) -> bool {
        s = slot_of(seq);
        const bool r = mbar_wait(&B->empty[s], (use_of(seq) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (r) ++seq;
        return r;
      };
      for (; ok && item_of(k, gridDim.x, blockIdx.x, n_items, nb, head, blk); ++k) {
        ok = mbar_wait(&B->q_empty, (k & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
        ++q_issued;
        mbar_arrive_expect_tx(&B->q_full, 6 * kBox);
        for (int t = 0; t < 2; ++t)
          for (int b = 0; b < 3; ++b)
            tma_load_3d(smem + OFF_Q + (3 * t + b) * kBox, &p.tm_q, &B->q_full, 64 * b, head, (2 * blk + t) * kT);
        const int n1 = min(2 * blk + 2, nkv);
        for (int j = 0; j < n1 && ok; ++j) {
          uint32_t s;
          // key tile: k_nope lo, k_nope hi, k_rope
          for (int b = 0; b < 3 && ok; ++b) {
            ok = take(s);
            if (!ok) break;
            mbar_arrive_expect_tx(&B->full[s], kBox);
            if (b < 2)
              tma_load_3d(smem + OFF_RING + s * kBox, &p.tm_kv, &B->full[s], 64 * b, head, j * kT);
            else
              tma_load_2d(smem + OFF_RING + s * kBox, &p.tm_kr, &B->full[s], p.kr_col, j * kT);
          }
          if (!ok) break;
          // value tile: the low half always in the lower of its two slots
          const uint32_t lo = min(slot_of(seq), slot_of(seq + 1));
          for (int h = 0; h < 2 && ok; ++h) {
            ok = take(s);
            if (!ok) break;
            mbar_arrive_expect_tx(&B->full[s], kBox);
            tma_load_3d(smem + OFF_RING + s * kBox, &p.tm_kv, &B->full[s], s == lo ? 128 : 192, head, j * kT);
          }
        }
      }
      if (!ok) {
        // let every copy already issued land before the CTA exits
        for (uint32_t s = 0; s < kSlots && s < seq; ++s) {
          const uint32_t last = s + kSlots * ((seq - 1 - s) / kSlots);
          drain_wait(&B->full[s], use_of(last) & 1, p.err);
        }
        if (q_issued > 0) drain_wait(&B->q_full, (q_issued - 1) & 1, p.err);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(1, 1, 0, 0, kT, kT);   // A = Q, B = K (both K-major)
      constexpr uint32_t idesc_pv = idesc_f16(1, 1, 0, 1, kT, 128);  // A = P (tensor memory), B = V (MN-major)
      // K-major SW128 descriptor of ring slot 0; slot s, box offsets and the
      // 16-element K steps are added to its address field (smem < 256 KB, so
      // the 14-bit field never carries into the next one)
      const uint64_t ring_desc = smem_desc(s_base + OFF_RING, 16, 1024, LAYOUT_SW128);
      const uint64_t ring_desc_v = ring_desc & ~(0x3FFFull << 16);  // LBO field set per value tile
      uint32_t seq = 0;                 // ring boxes consumed
      uint32_t pc[2] = {0, 0};          // P tiles consumed per query tile
      bool ok = true;
      int head, blk;
      for (int k = 0; ok && item_of(k, gridDim.x, blockIdx.x, n_items, nb, head, blk); ++k) {
        const int n0 = min(2 * blk + 1, nkv), n1 = min(2 * blk + 2, nkv);
        ok = mbar_wait(&B->q_full, k & 1, abort, p.err, ERR_TIMEOUT_FULL);
        uint32_t vseq = 0;    // sequence number of the previous tile's first value box
        bool vready = false;  // its full barriers already waited
        for (int j = 0; j <= n1 && ok; ++j) {
          const uint32_t kseq = seq;  // this tile's key boxes: kseq .. kseq + 2
          bool kready = false;
          auto wait_k = [&]() -> bool {
            if (kready) return true;
            for (uint32_t b = 0; b < 3; ++b)
              if (!mbar_wait(&B->full[slot_of(kseq + b)], use_of(kseq + b) & 1, abort, p.err, ERR_TIMEOUT_FULL))
                return false;
            kready = true;
            tc_fence_after();
            return true;
          };
          auto wait_v = [&]() -> bool {
            if (vready) return true;
            for (uint32_t b = 0; b < 2; ++b)
              if (!mbar_wait(&B->full[slot_of(vseq + b)], use_of(vseq + b) & 1, abort, p.err, ERR_TIMEOUT_FULL))
                return false;
            vready = true;
            tc_fence_after();
            return true;
          };
          auto issue_pv = [&](int t) -> bool {
            // O_t (+)= P_t V_{j-1}
            if (!mbar_wait(&B->p_full[t], pc[t] & 1, abort, p.err, ERR_TIMEOUT_MMA)) return false;
            ++pc[t];
            if (j == 1 && k > 0 && !mbar_wait(&B->o_empty[t], (k - 1) & 1, abort, p.err, ERR_TIMEOUT_MMA))
              return false;
            if (!wait_v()) return false;
            tc_fence_after();
            // V: the low half sits in the lower of the two slots (see the producer)
            const uint32_t sa = slot_of(vseq);
            const uint64_t vd = ring_desc_v + (sa == kSlots - 1 ? 0u : sa * (kBox >> 4)) +
                                (static_cast<uint64_t>(sa == kSlots - 1 ? (kSlots - 1) * (kBox >> 4) : (kBox >> 4)) << 16);
            const uint32_t a_tm = tmem + 128 * t;
            const uint32_t d_tm = tmem + 256 + 128 * t;
            mma_f16_ts(d_tm, a_tm, vd, idesc_pv, j == 1 ? 0u : 1u);
#pragma unroll
            for (int kk = 1; kk < kT / 16; ++kk) mma_f16_ts(d_tm, a_tm + 8 * kk, vd + 128 * kk, idesc_pv, 1u);
            return true;
          };
          auto issue_qk = [&](int t) {
            const uint64_t qd = ring_desc - (static_cast<uint64_t>(OFF_RING - OFF_Q - 3 * t * kBox) >> 4);
            const uint32_t d_tm = tmem + 128 * t;
#pragma unroll
            for (int b = 0; b < 3; ++b) {
              const uint64_t kd = ring_desc + slot_of(kseq + b) * (kBox >> 4);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_f16_ss(d_tm, qd + b * (kBox >> 4) + 2 * kk, kd + 2 * kk, idesc_qk, (b | kk) ? 1u : 0u);
            }
            mma_commit(&B->s_full[t]);
          };
          // A: P0 V_{j-1}
          if (j >= 1 && j <= n0) {
            ok = issue_pv(0);
            if (!ok) break;
            if (j == n0) mma_commit(&B->o_full[0]);
          }
          // B: S0 = Q0 K_j^T
          if (j < n0) {
            ok = wait_k();
            if (!ok) break;
            issue_qk(0);
          }
          // C: P1 V_{j-1}, then V_{j-1} is free
          if (j >= 1) {
            ok = issue_pv(1);
            if (!ok) break;
            mma_commit(&B->empty[slot_of(vseq)]);
            mma_commit(&B->empty[slot_of(vseq + 1)]);
            if (j == n1) mma_commit(&B->o_full[1]);
          }
          // D: S1 = Q1 K_j^T, then K_j is free
          if (j < n1) {
            ok = wait_k();
            if (!ok) break;
            issue_qk(1);
            for (uint32_t b = 0; b < 3; ++b) mma_commit(&B->empty[slot_of(kseq + b)]);
            if (j == n1 - 1) mma_commit(&B->q_empty);
            vseq = kseq + 3;
            vready = false;
            seq = kseq + 5;
          }
        }
      }
      mma_commit(&B->drain);
      drain_wait(&B->drain, 0, p.err);
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- softmax + epilogue
    // (warps 0-7 only: warps 10-11 of the shrunk warpgroup must not come here)
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int t = warp >> 2;            // query tile of this warpgroup
    const int sub = warp & 3;           // TMEM lane quarter
    const int r = 32 * sub + lane;      // query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * sub) << 16;
    const uint32_t s_col = tmem + lane_base + 128 * t;
    const uint32_t o_col = tmem + lane_base + 256 + 128 * t;
    const float sl = p.scale_log2;
    uint32_t sc = 0;  // S tiles consumed
    int head, blk;
    bool bad = false;
    for (int k = 0; !bad && item_of(k, gridDim.x, blockIdx.x, n_items, nb, head, blk); ++k) {
      const int n_t = min(2 * blk + 1 + t, nkv);
      const int qrow = (2 * blk + t) * kT + r;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n_t; ++j, ++sc) {
        bad = !mbar_wait(&B->s_full[t], sc & 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (__any_sync(0xffffffffu, bad)) { bad = true; break; }
        tc_fence_after();
        float s[kT];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_col + 32 * c, s + 32 * c);
        tmem_wait_ld();
        if (j == n_t - 1) {
          // diagonal tile and sequence end: key kb + c is visible iff c <= lim
          const int lim = min(qrow, p.S - 1) - j * kT;
#pragma unroll
          for (int c = 0; c < kT; ++c) s[c] = c <= lim ? s[c] : -INFINITY;
        }
        float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]), mx2 = fmaxf(s[4], s[5]), mx3 = fmaxf(s[6], s[7]);
#pragma unroll
        for (int c = 8; c < kT; c += 8) {
          mx0 = max3(mx0, s[c], s[c + 1]);
          mx1 = max3(mx1, s[c + 2], s[c + 3]);
          mx2 = max3(mx2, s[c + 4], s[c + 5]);
          mx3 = max3(mx3, s[c + 6], s[c + 7]);
        }
        const float mx = fmaxf(max3(mx0, mx1, mx2), mx3);
        const bool need = mx * sl > m * sl + 8.0f || m == -INFINITY;
        if (__any_sync(0xffffffffu, need)) {
          const float mn = fmaxf(m, mx);
          const float alpha = (m == -INFINITY) ? 0.f : ex2((m - mn) * sl);
          if (j > 0) {
            // every earlier P V of this tile has completed (s_full covers them)
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              float o[32];
              tmem_ld32(o_col + 32 * c, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= alpha;
              tmem_st32(o_col + 32 * c, o);
            }
          }
          l *= alpha;
          m = mn;
        }
        const float neg = -m * sl;
        float sum0 = 0.f, sum1 = 0.f, sum2 = 0.f, sum3 = 0.f;
        uint32_t pk[kT / 2];
#pragma unroll
        for (int c = 0; c < kT; c += 4) {
          float a0, a1, a2, a3;
          ffma2(a0, a1, s[c], s[c + 1], sl, neg);
          ffma2(a2, a3, s[c + 2], s[c + 3], sl, neg);
          a0 = ex2(a0);
          a1 = ex2(a1);
          a2 = ex2(a2);
          a3 = ex2(a3);
          fadd2(sum0, sum1, a0, a1);
          fadd2(sum2, sum3, a2, a3);
          pk[c / 2] = pack_bf16(a0, a1);
          pk[c / 2 + 1] = pack_bf16(a2, a3);
        }
        l += (sum0 + sum1) + (sum2 + sum3);
        // P over the first 64 columns of S
        tmem_st32u(s_col, pk);
        tmem_st32u(s_col + 32, pk + 32);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->p_full[t]);
      }
      if (bad) break;
      // ---- epilogue: o = O / l as bf16 into out[row][head][0:128]
      bad = !mbar_wait(&B->o_full[t], k & 1, abort, p.err, ERR_TIMEOUT_MMA);
      if (__any_sync(0xffffffffu, bad)) break;
      tc_fence_after();
      const float inv = 1.0f / l;
      __nv_bfloat16 *dst = p.out + (static_cast<size_t>(qrow) * 16 + head) * 128;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float o[32];
        tmem_ld32(o_col + 32 * c, o);
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
      if (lane == 0) mbar_arrive(&B->o_empty[t]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

cudaError_t launch_flash_prefill(const FlashParams &p, int sms, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  static int regs = 0;  // registers per thread the kernel is launched with
  if (regs == 0) {
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, flash_prefill_kernel);
    if (e != cudaSuccess) return e;
    regs = fa.numRegs;
  }
  if (regs * kThreads < kRegsNeeded) return cudaErrorInvalidConfiguration;  // the split would never be granted
  const int items = ((p.S + 2 * kT - 1) / (2 * kT)) * 16;
  const int grid = items < sms ? items : sms;
  ProfScope ps("flash_prefill", stream);
  flash_prefill_kernel<<<grid, kThreads, kSmem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace kvl
