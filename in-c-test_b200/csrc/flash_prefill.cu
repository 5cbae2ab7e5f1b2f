// flash_prefill.cu -- causal MLA prefill attention on sm_100a (the attention
// of src/mla_prefill_streaming.c:141-193 in the non-absorbed form):
//     s_tj = (q_nope_t . k_nope_j + q_rope_t . k_rope_j) * scale,   j <= t
//     o_t  = sum_j softmax_j(s_t) v_j
// per head, with q_rope/k_rope already rotated, k_rope shared by the heads.
//
// Work item = (head, 128-query tile); items go to persistent CTAs in snake
// order of decreasing cost (query tile i attends key tiles 0..i).  Per key
// tile j the tensor core computes S_j = Q K_j^T (12 tcgen05 MMAs, M = N = 128)
// into one of three S buffers in tensor memory and O += P_j V_j (8 MMAs, P
// read from tensor memory).  With three S buffers the scores of tiles j + 1
// and j + 2 are ready while the softmax of tile j runs, so the softmax and
// the MMAs overlap fully: S_{j+3} is issued right after P_j V_j, which has
// consumed the P_j stored over the first 64 columns of that buffer.
//
// Softmax: two warpgroups share each 128 x 128 score tile, one per half of
// the keys (thread = query row), and exchange their row maxima through shared
// memory once per tile.  The running max is rescaled lazily (only when it
// grows by more than 2^8 in the exp2 domain); each group rescales its half of
// the O row and keeps its own partial row sum, the two sums being added in
// the epilogue.  The causal mask and the sequence bound are applied on the
// last key tile of a query tile only; all earlier tiles are entirely visible.
//
// Tensor memory: S0 | S1 | S2 | O (4 x 128 columns).  Shared memory: Q (3 SW128
// boxes of 128 rows x 64), K ring 2 x (k_nope lo, k_nope hi, k_rope), V ring
// 2 x (v lo, v hi), the max / sum exchange and the barriers.
// Roles (384 threads): warps 0-3 softmax of keys 0-63, warps 4-7 keys 64-127
// (TMEM lanes 32 * (warp % 4)), warp 8 Q and K copies, warp 9 TMEM owner and
// MMA issuer, warp 10 V copies, warp 11 idle.  Every wait is bounded and
// reports through p.err.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "flash_prefill.cuh"
#include "gemm.cuh"
#include "pdl.cuh"
#include "prof.cuh"
#include "sm100.cuh"

namespace kvl {
namespace fpre {

constexpr int kT = 128;                    // queries / keys per tile
constexpr uint32_t kBox = kT * 128;        // 128 rows x 64 bf16 = 16 KB
constexpr int kKSt = 2, kVSt = 2;          // ring stages
constexpr int kSBuf = 3;                   // S buffers in tensor memory
constexpr uint32_t OFF_Q = 0;                              // 3 boxes
constexpr uint32_t OFF_K = 3 * kBox;                       // kKSt x 3 boxes
constexpr uint32_t OFF_V = OFF_K + kKSt * 3 * kBox;        // kVSt x 2 boxes
constexpr uint32_t OFF_X = OFF_V + kVSt * 2 * kBox;        // float xm[2][2][128], xl[2][128]
constexpr uint32_t OFF_BAR = OFF_X + 6 * 128 * 4;
constexpr int kThreads = 384;
constexpr uint32_t kColO = 384;

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kKSt];
  uint64_t v_full[kVSt];
  uint64_t s_full[kSBuf], p_full[kSBuf], pv_done[kSBuf];
  uint64_t o_full, o_empty, drain;
  uint32_t tmem_base;
  int abort;
};

constexpr uint32_t kSmem = OFF_BAR + sizeof(Bars) + 1024;
static_assert(kSmem <= 232448, "shared memory budget");
constexpr uint32_t kTmemCols = 512;

// A work unit: key tiles [k0, k1) of query tile qt and one head; pos is its
// index in the unit order (the slot of its partial result when cut).
struct Unit {
  int head, qt, k0, k1, pos;
  bool cut;
};

// Query tile groups in the unit order: the tiles of [q_tile0, nq) from the
// last down, then those of the optional lower range [lo_t0, lo_t1) from its
// last down (n_hi tiles above it) -- decreasing key counts within each range.
__host__ __device__ __forceinline__ int group_tile(const FlashParams &p, int nq, int n_hi, int t) {
  return t < n_hi ? nq - 1 - t : p.lo_t1 - 1 - (t - n_hi);
}

// Pieces of an item with n key tiles.
__host__ __device__ __forceinline__ int pieces_of(int n, int kpiece) {
  return kpiece > 0 ? (n + kpiece - 1) / kpiece : 1;
}

__host__ __device__ __forceinline__ int unit_count(const FlashParams &p, int nq, int n_hi, int kpiece) {
  const int groups = n_hi + p.lo_t1 - p.lo_t0;
  if (kpiece <= 0) return groups * 16;
  int n = 0;
  for (int t = 0; t < groups; ++t) n += 16 * pieces_of(group_tile(p, nq, n_hi, t) + 1, kpiece);
  return n;
}

// Unit pos: within a query tile group the units are piece-major (piece, head).
__device__ __forceinline__ void unit_at(const FlashParams &p, int nq, int n_hi, int pos, Unit &u) {
  u.pos = pos;
  if (p.kpiece <= 0) {
    u.qt = group_tile(p, nq, n_hi, pos / 16);
    u.head = pos % 16;
    u.k0 = 0;
    u.k1 = u.qt + 1;
    u.cut = false;
    return;
  }
  int base = 0;
  for (int t = 0;; ++t) {
    const int qt = group_tile(p, nq, n_hi, t), np = pieces_of(qt + 1, p.kpiece);
    if (pos < base + 16 * np) {
      const int in = pos - base, piece = in / 16;
      u.qt = qt;
      u.head = in % 16;
      u.k0 = piece * p.kpiece;
      u.k1 = np > 1 ? min(qt + 1, u.k0 + p.kpiece) : qt + 1;
      if (np == 1) u.k0 = 0;
      u.cut = np > 1;
      return;
    }
    base += 16 * np;
  }
}

// Unit k of the CTA: snake order over the units (sorted by decreasing cost
// within each range).
__device__ __forceinline__ bool item_of(const FlashParams &p, int k, int nq, int n_hi, int n_units, Unit &u) {
  const int grid = gridDim.x, cta = blockIdx.x;
  const int pos = (k & 1) ? (k + 1) * grid - 1 - cta : k * grid + cta;
  if (pos >= n_units) return false;
  unit_at(p, nq, n_hi, pos, u);
  return true;
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

// Row tile of tm_q and out that holds query tile qt.
__device__ __forceinline__ int q_slot(const FlashParams &p, int qt) {
  if (!p.q_compact) return qt;
  return qt >= p.q_tile0 ? p.lo_t1 - p.lo_t0 + qt - p.q_tile0 : qt - p.lo_t0;
}

}  // namespace fpre

using namespace fpre;

__global__ void __launch_bounds__(kThreads, 1) flash_prefill_kernel(const __grid_constant__ FlashParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars *B = reinterpret_cast<Bars *>(smem + OFF_BAR);
  float *xm = reinterpret_cast<float *>(smem + OFF_X);   // [tile parity][group][row]
  float *xl = xm + 4 * 128;                               // [group][row]
  const uint32_t s_base = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int *abort = &B->abort;
  const int nq = (p.S + kT - 1) / kT;
  const int n_hi = nq - p.q_tile0;
  const int n_units = unit_count(p, nq, n_hi, p.kpiece);  // query tiles [q_tile0, nq) ++ [lo_t0, lo_t1)

  if (threadIdx.x == 0) {
    mbar_init(&B->q_full, 1);
    for (int i = 0; i < kKSt; ++i) mbar_init(&B->k_full[i], 1);
    for (int i = 0; i < kVSt; ++i) mbar_init(&B->v_full[i], 1);
    for (int i = 0; i < kSBuf; ++i) {
      mbar_init(&B->s_full[i], 1);
      mbar_init(&B->p_full[i], 8);
      mbar_init(&B->pv_done[i], 1);
    }
    mbar_init(&B->o_full, 1);
    mbar_init(&B->o_empty, 8);
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
  // as a programmatic dependent: every global access comes after the wait
  pdl_wait();
  pdl_trigger();

  if (warp == 8) {
    // ---------------------------------------------------------------- Q and K copies
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_kv);
      tma_prefetch_desc(&p.tm_kr);
      // A stage is free once the MMAs that read it have completed: Q after
      // the last S of the previous item, the K of tile g after S_g (s_full of
      // tile g).  The parity is unambiguous: S_{g+3} needs a K this warp loads
      // later, and S_{g-3} completed before S_{g-2}, which was waited for.
      uint32_t kc = 0, qc = 0;  // kc: key tiles issued = global S tile index
      bool ok = true;
      Unit u;
      for (int k = 0; ok && item_of(p, k, nq, n_hi, n_units, u); ++k) {
        if (kc > 0) {
          const uint32_t gl = kc - 1;  // last S of the previous item
          ok = mbar_wait(&B->s_full[gl % kSBuf], (gl / kSBuf) & 1, abort, p.err, ERR_TIMEOUT_EMPTY);
          if (!ok) break;
        }
        ++qc;
        mbar_arrive_expect_tx(&B->q_full, 3 * kBox);
        for (int b = 0; b < 3; ++b)
          tma_load_3d(smem + OFF_Q + b * kBox, &p.tm_q, &B->q_full, 64 * b, u.head, q_slot(p, u.qt) * kT);
        for (int j = u.k0; j < u.k1 && ok; ++j, ++kc) {
          const uint32_t s = kc % kKSt;
          if (kc >= static_cast<uint32_t>(kKSt)) {
            const uint32_t gp = kc - kKSt;  // the tile that last used this stage
            ok = mbar_wait(&B->s_full[gp % kSBuf], (gp / kSBuf) & 1, abort, p.err, ERR_TIMEOUT_EMPTY);
            if (!ok) break;
          }
          uint8_t *kd = smem + OFF_K + s * 3 * kBox;
          mbar_arrive_expect_tx(&B->k_full[s], 3 * kBox);
          tma_load_3d(kd, &p.tm_kv, &B->k_full[s], 0, u.head, j * kT);
          tma_load_3d(kd + kBox, &p.tm_kv, &B->k_full[s], 64, u.head, j * kT);
          tma_load_2d(kd + 2 * kBox, &p.tm_kr, &B->k_full[s], p.kr_col, zigzag_tile(j, p.zz_world, p.zz_c128) * kT);
        }
      }
      if (!ok) {
        for (uint32_t s = 0; s < static_cast<uint32_t>(kKSt) && s < kc; ++s) {
          const uint32_t last = s + kKSt * ((kc - 1 - s) / kKSt);
          drain_wait(&B->k_full[s], (last / kKSt) & 1, p.err);
        }
        if (qc > 0) drain_wait(&B->q_full, (qc - 1) & 1, p.err);
      }
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------------- V copies
    if (lane == 0) {
      uint32_t vc = 0;
      bool ok = true;
      Unit u;
      for (int k = 0; ok && item_of(p, k, nq, n_hi, n_units, u); ++k) {
        for (int j = u.k0; j < u.k1 && ok; ++j, ++vc) {
          // the V of tile g is free once P_g V_g has completed (pv_done of tile g)
          const uint32_t s = vc % kVSt;
          if (vc >= static_cast<uint32_t>(kVSt)) {
            const uint32_t gp = vc - kVSt;
            ok = mbar_wait(&B->pv_done[gp % kSBuf], (gp / kSBuf) & 1, abort, p.err, ERR_TIMEOUT_EMPTY);
            if (!ok) break;
          }
          uint8_t *vd = smem + OFF_V + s * 2 * kBox;
          mbar_arrive_expect_tx(&B->v_full[s], 2 * kBox);
          tma_load_3d(vd, &p.tm_kv, &B->v_full[s], 128, u.head, j * kT);
          tma_load_3d(vd + kBox, &p.tm_kv, &B->v_full[s], 192, u.head, j * kT);
        }
      }
      if (!ok) {
        for (uint32_t s = 0; s < static_cast<uint32_t>(kVSt) && s < vc; ++s) {
          const uint32_t last = s + kVSt * ((vc - 1 - s) / kVSt);
          drain_wait(&B->v_full[s], (last / kVSt) & 1, p.err);
        }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(1, 1, 0, 0, kT, kT);   // A = Q, B = K (both K-major)
      constexpr uint32_t idesc_pv = idesc_f16(1, 1, 0, 1, kT, 128);  // A = P (tensor memory), B = V (MN-major)
      // descriptors: the address field of a base descriptor advanced by offsets
      // (shared memory < 256 KB, so the 14-bit field never carries over)
      const uint64_t q_desc = smem_desc(s_base + OFF_Q, 16, 1024, LAYOUT_SW128);
      const uint64_t k_desc = smem_desc(s_base + OFF_K, 16, 1024, LAYOUT_SW128);
      const uint64_t v_desc = smem_desc(s_base + OFF_V, kBox, 1024, LAYOUT_SW128);
      uint32_t tc = 0, kc = 0, vc = 0;  // S tiles, K stages, V stages consumed
      bool ok = true;
      Unit u;
      for (int k = 0; ok && item_of(p, k, nq, n_hi, n_units, u); ++k) {
        const int n = u.k1 - u.k0;
        ok = mbar_wait(&B->q_full, k & 1, abort, p.err, ERR_TIMEOUT_FULL);
        auto issue_s = [&](int j) -> bool {
          // S_j = Q K_j^T into buffer (tc + j) % 3
          const uint32_t b = (tc + j) % kSBuf, s = kc % kKSt;
          if (!mbar_wait(&B->k_full[s], (kc / kKSt) & 1, abort, p.err, ERR_TIMEOUT_FULL)) return false;
          tc_fence_after();
          const uint64_t kd = k_desc + s * (3 * kBox >> 4);
#pragma unroll
          for (int bx = 0; bx < 3; ++bx)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16_ss(tmem + 128 * b, q_desc + bx * (kBox >> 4) + 2 * kk, kd + bx * (kBox >> 4) + 2 * kk,
                         idesc_qk, (bx | kk) ? 1u : 0u);
          mma_commit(&B->s_full[b]);  // also frees the K stage (and Q after the item's last S)
          ++kc;
          return true;
        };
        for (int j = 0; j < n && j < kSBuf && ok; ++j) ok = issue_s(j);
        for (int j = 0; j < n && ok; ++j) {
          const uint32_t g = tc + j, b = g % kSBuf, s = vc % kVSt;
          ok = mbar_wait(&B->p_full[b], (g / kSBuf) & 1, abort, p.err, ERR_TIMEOUT_MMA);
          if (ok && j == 0 && k > 0) ok = mbar_wait(&B->o_empty, (k - 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
          if (ok) ok = mbar_wait(&B->v_full[s], (vc / kVSt) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          // O (+)= P_j V_j
          const uint64_t vd = v_desc + s * (2 * kBox >> 4);
#pragma unroll
          for (int kk = 0; kk < kT / 16; ++kk)
            mma_f16_ts(tmem + kColO, tmem + 128 * b + 8 * kk, vd + 128 * kk, idesc_pv, (j | kk) ? 1u : 0u);
          mma_commit(&B->pv_done[b]);  // also frees the V stage
          ++vc;
          if (j == n - 1) mma_commit(&B->o_full);
          if (j + kSBuf < n) ok = issue_s(j + kSBuf);
        }
        tc += n;
      }
      mma_commit(&B->drain);
      drain_wait(&B->drain, 0, p.err);
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- softmax + epilogue
    const int w = warp >> 2;            // key half of this warpgroup
    const int sub = warp & 3;           // TMEM lane quarter
    const int r = 32 * sub + lane;      // query row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(32 * sub) << 16;
    const uint32_t o_col = tmem + lane_base + kColO + 64 * w;
    const float sl = p.scale_log2;
    uint32_t g = 0;  // S tiles consumed (same sequence as the MMA issuer's)
    Unit u;
    bool bad = false;
    for (int k = 0; !bad && item_of(p, k, nq, n_hi, n_units, u); ++k) {
      const int n = u.k1 - u.k0;
      const int qrow = u.qt * kT + r;
      float m = -INFINITY, l = 0.f;
      for (int jj = 0; jj < n; ++jj, ++g) {
        const int j = u.k0 + jj;  // key tile
        const uint32_t b = g % kSBuf;
        const uint32_t s_col = tmem + lane_base + 128 * b;
        bad = !mbar_wait(&B->s_full[b], (g / kSBuf) & 1, abort, p.err, ERR_TIMEOUT_MMA);
        float s[64];
        if (!bad) {
          tc_fence_after();
          tmem_ld32(s_col + 64 * w, s);
          tmem_ld32(s_col + 64 * w + 32, s + 32);
          tmem_wait_ld();
        }
        if (j == u.qt) {
          // diagonal tile and sequence end: key j*128 + 64w + c is visible iff c <= lim
          const int lim = min(qrow, p.S - 1) - j * kT - 64 * w;
#pragma unroll
          for (int c = 0; c < 64; ++c) s[c] = c <= lim ? s[c] : -INFINITY;
        }
        float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]), mx2 = fmaxf(s[4], s[5]), mx3 = fmaxf(s[6], s[7]);
#pragma unroll
        for (int c = 8; c < 64; c += 8) {
          mx0 = max3(mx0, s[c], s[c + 1]);
          mx1 = max3(mx1, s[c + 2], s[c + 3]);
          mx2 = max3(mx2, s[c + 4], s[c + 5]);
          mx3 = max3(mx3, s[c + 6], s[c + 7]);
        }
        xm[((g & 1) * 2 + w) * 128 + r] = fmaxf(max3(mx0, mx1, mx2), mx3);
        // both halves of the row meet here (the S loads of both are complete,
        // so P may now overwrite the first 64 columns)
        if (named_bar_or(1, 256, bad)) { bad = true; break; }
        const float mx = fmaxf(xm[(g & 1) * 256 + r], xm[(g & 1) * 256 + 128 + r]);
        const bool need = mx * sl > m * sl + 8.0f || m == -INFINITY;
        if (__any_sync(0xffffffffu, need)) {
          const float mn = fmaxf(m, mx);
          const float alpha = (m == -INFINITY) ? 0.f : ex2((m - mn) * sl);
          if (jj > 0) {
            // this group's half of the O row, once P_{j-1} V_{j-1} (and so every
            // earlier P V) has landed.  Per-buffer barriers keep the parity
            // unambiguous: s_full of tile g implies P V of tile g - 3 is done,
            // and P V of tile g + 2 cannot start before this group's P.
            const uint32_t gp = g - 1;
            bad = !mbar_wait(&B->pv_done[gp % kSBuf], (gp / kSBuf) & 1, abort, p.err, ERR_TIMEOUT_MMA);
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
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
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
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
        // P (bf16 pairs) over columns [32w, 32w + 32) of this S buffer
        tmem_st32(s_col + 32 * w, reinterpret_cast<const float *>(pk));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->p_full[b]);
      }
      if (bad) break;
      // ---- epilogue: o = O / (l_0 + l_1) as bf16 into out[row][head][0:128]
      bad = !mbar_wait(&B->o_full, k & 1, abort, p.err, ERR_TIMEOUT_MMA);
      xl[w * 128 + r] = l;
      if (named_bar_or(2, 256, bad)) break;
      tc_fence_after();
      const float lsum = xl[r] + xl[128 + r];
      const float inv = 1.0f / lsum;
      if (u.cut) {
        // a piece of a cut item: O / l in fp32 and log2 of l at the exp2 scale
        // of the scores, for the combine kernel
        float *dst = p.part_o + (static_cast<size_t>(u.pos) * kT + r) * 128 + 64 * w;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float o[32];
          tmem_ld32(o_col + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4 *>(dst + 32 * c + i) =
                make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
        }
        if (w == 0) p.part_lse[static_cast<size_t>(u.pos) * kT + r] = m * sl + log2f(lsum);
      } else {
        __nv_bfloat16 *dst = p.out + (static_cast<size_t>(q_slot(p, u.qt) * kT + r) * 16 + u.head) * 128 + 64 * w;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
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
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->o_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// The cut items' pieces combined: block b takes rows 8 (b % 16) .. + 7 of the
// (b / 16)-th cut item in unit order, 32 threads per row, four dimensions per
// thread; o = sum_p w_p O_p / sum_p w_p with w_p = 2^(lse_p - max lse) (every
// piece of a row has at least one visible key, so each lse is finite).
__global__ void __launch_bounds__(256) flash_combine_kernel(const __grid_constant__ FlashParams p) {
  const int nq = (p.S + kT - 1) / kT, n_hi = nq - p.q_tile0, groups = n_hi + p.lo_t1 - p.lo_t0;
  int base = 0, item = blockIdx.x / 16, qt = -1, np = 0, head = 0;
  for (int t = 0; t < groups; ++t) {
    const int q = group_tile(p, nq, n_hi, t), n = pieces_of(q + 1, p.kpiece);
    if (n > 1) {
      if (item < 16) {
        qt = q;
        np = n;
        head = item;
        break;
      }
      item -= 16;
    }
    base += 16 * n;
  }
  const int r = 8 * (blockIdx.x % 16) + (threadIdx.x >> 5), d = 4 * (threadIdx.x & 31);
  if (qt < 0 || qt * kT + r >= p.S) return;
  float lmax = -INFINITY;
  for (int i = 0; i < np; ++i) lmax = fmaxf(lmax, p.part_lse[static_cast<size_t>(base + 16 * i + head) * kT + r]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  for (int i = 0; i < np; ++i) {
    const size_t u = static_cast<size_t>(base + 16 * i + head);
    const float wt = exp2f(p.part_lse[u * kT + r] - lmax);
    const float4 o = *reinterpret_cast<const float4 *>(p.part_o + (u * kT + r) * 128 + d);
    acc.x += wt * o.x;
    acc.y += wt * o.y;
    acc.z += wt * o.z;
    acc.w += wt * o.w;
    wsum += wt;
  }
  const float inv = 1.0f / wsum;
  uint2 v;
  v.x = pack_bf16(acc.x * inv, acc.y * inv);
  v.y = pack_bf16(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2 *>(p.out + (static_cast<size_t>(q_slot(p, qt) * kT + r) * 16 + head) * 128 + d) = v;
}

// Largest CTA load (key tiles, plus about 1.3 tiles of pipeline drain and
// refill per unit) when the units of a launch cut at kpiece are dealt out in
// snake order over `grid` CTAs.
static double snake_max_load(const FlashParams &p, int nq, int n_hi, int kpiece, int units, int grid) {
  std::vector<double> cost(units);
  const int groups = n_hi + p.lo_t1 - p.lo_t0;
  for (int t = 0, pos = 0; t < groups; ++t) {
    const int n = group_tile(p, nq, n_hi, t) + 1, np = pieces_of(n, kpiece);
    for (int i = 0; i < np; ++i) {
      const int len = np > 1 ? std::min(n, (i + 1) * kpiece) - i * kpiece : n;
      for (int h = 0; h < 16; ++h) cost[pos++] = len + 1.3;
    }
  }
  std::vector<double> load(grid, 0.0);
  for (int pos = 0; pos < units; ++pos) {
    const int k = pos / grid, i = pos % grid;
    load[(k & 1) ? grid - 1 - i : i] += cost[pos];
  }
  return *std::max_element(load.begin(), load.end());
}

cudaError_t launch_flash_prefill(const FlashParams &p_in, int sms, cudaStream_t stream, bool dep) {
  cudaError_t e = cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
  if (e != cudaSuccess) return e;
  FlashParams p = p_in;
  const int nq = (p.S + kT - 1) / kT, n_hi = nq - p.q_tile0;
  if (nq - p.q_tile0 + p.lo_t1 - p.lo_t0 <= 0 || p.q_tile0 < 0 || p.lo_t0 < 0 || p.lo_t1 < p.lo_t0 ||
      p.lo_t1 > p.q_tile0)
    return cudaErrorInvalidValue;
  if (p.kpiece < 0) {
    // cut only when the items leave SMs idle, at the piece length whose snake
    // deal has the smallest largest load (within the partial-result slots)
    const int items = unit_count(p, nq, n_hi, 0);
    p.kpiece = 0;
    if (items < sms && p.part_o && p.part_lse) {
      double best = snake_max_load(p, nq, n_hi, 0, items, items);
      for (int kp = 2; kp <= nq; ++kp) {
        const int units = unit_count(p, nq, n_hi, kp);
        if (units > kFlashMaxUnits) continue;
        const double ld = snake_max_load(p, nq, n_hi, kp, units, std::min(units, sms));
        // a cut costs the combine launch: ask for two key tiles of gain
        if (ld + 2.0 < best) {
          best = ld;
          p.kpiece = kp;
        }
      }
    }
  }
  const int units = unit_count(p, nq, n_hi, p.kpiece);
  if (p.kpiece > 0 && (units > kFlashMaxUnits || !p.part_o || !p.part_lse)) return cudaErrorInvalidValue;
  const int grid = units < sms ? units : sms;
  {
    ProfScope ps("flash_prefill", stream);
    if (dep) {
      e = launch_dependent(flash_prefill_kernel, dim3(grid), dim3(kThreads), kSmem, stream, p);
    } else {
      flash_prefill_kernel<<<grid, kThreads, kSmem, stream>>>(p);
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) return e;
  }
  if (p.kpiece > 0) {
    int cut = 0;
    for (int t = 0; t < n_hi + p.lo_t1 - p.lo_t0; ++t) cut += pieces_of(group_tile(p, nq, n_hi, t) + 1, p.kpiece) > 1;
    if (cut > 0) {
      ProfScope ps("flash_combine", stream);
      flash_combine_kernel<<<16 * 16 * cut, 256, 0, stream>>>(p);
      e = cudaGetLastError();
    }
  }
  return e;
}

}  // namespace kvl

