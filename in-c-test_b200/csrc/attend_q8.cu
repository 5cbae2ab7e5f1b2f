// attend_q8.cu -- absorbed MLA decode attention over the row-wise Q8 latent
// state (int8 latent [rows][512], fp32 scale [rows], bf16 rope [rows][64]: the
// reference's layout, include/kvl/mla_compressed_q8_state.h).
//
// Reference semantics: src/mla_compressed_q8_state.c:216-238, with the
// dequantised row latent_j = (float)q_j * scale_j (:57-61).  The stored int8
// values are exact in fp16, so the kernel feeds them to the tensor core
// unscaled and applies the row scale outside the MMA:
//     s_j  = scale_j * (q_lat . q_j) + (q_rope . rope_j)
//     O    = sum_j (p_j * scale_j) q_j           (P' = p * scale in fp16)
// which equals sum_j p_j * dequant(q_j) up to the rounding of P'.
//
// Tiles of 128 KV rows (see attend_bf16.cu for the MMA cost model).  Shared
// memory: int8 staging ring 2 x 16 KB (128 rows x 128 dims), fp16 ring 4 x
// 32 KB (one tile; a slot is released when its P.V MMAs end), rope ring 2 x
// 16 KB.
//
// Roles (384 threads, one CTA per SM):
//   warp 0      TMA producer (int8 staging + rope)
//   warp 1      TMEM owner and tcgen05 issuer
//   warps 4-7   query load per segment (q_lat -> fp16, q_rope -> bf16 SW128
//               tiles), softmax and epilogue (TMEM subpartitions 0-3; thread = KV row)
//   warps 8-11  converters: int8 staging -> fp16 SW128 ring
#include "attend_common.cuh"
#include "prof.cuh"
#include "sm100.cuh"

namespace kvl {
namespace q8dec {

constexpr int kStgSlots = 2;
constexpr int kCvtSlots = 4;
constexpr int kRopeSlots = 2;
constexpr uint32_t kBox = kTileTok * 128;      // 128 rows x 128 B = 16 KB
constexpr uint32_t kStgBytes = kBox;           // int8: 128 rows x 128 dims
constexpr uint32_t kCvtBytes = 2 * kBox;       // fp16: 128 rows x 128 dims (two 64-dim boxes)
constexpr uint32_t kRopeBytes = kBox;          // bf16: 128 rows x 64 dims
constexpr uint32_t kQBytes = 9 * 2048;
constexpr uint32_t kPChunkSbo = (kTileTok / 8) * 128;
constexpr uint32_t kPBytes = 2 * kPChunkSbo;
constexpr uint32_t OFF_CVT = 0;
constexpr uint32_t OFF_STG = OFF_CVT + kCvtSlots * kCvtBytes;
constexpr uint32_t OFF_ROPE = OFF_STG + kStgSlots * kStgBytes;
constexpr uint32_t OFF_Q = OFF_ROPE + kRopeSlots * kRopeBytes;
constexpr uint32_t OFF_P = OFF_Q + kQBytes;
constexpr uint32_t OFF_BAR = OFF_P + 2 * kPBytes;

struct Bars {
  uint64_t stg_full[kStgSlots], stg_empty[kStgSlots];
  uint64_t cvt_full[kCvtSlots], cvt_empty[kCvtSlots];
  uint64_t rope_full[kRopeSlots], rope_empty[kRopeSlots];
  uint64_t q_full;
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full, o_empty, drain;
  uint32_t tmem_base;
  int abort;
  float red[4][kHeads];
};

constexpr uint32_t kSmemBytes = OFF_BAR + sizeof(Bars) + 1024;
static_assert(OFF_STG % 1024 == 0 && OFF_ROPE % 1024 == 0 && OFF_Q % 1024 == 0 && OFF_P % 1024 == 0, "align");
static_assert(kSmemBytes <= 232448, "shared memory budget");

// TMEM columns: latent scores 2 buffers x 16 @0, rope scores 2 x 16 @32, O 4 x 16 @64.
constexpr uint32_t kColRope = 32;
constexpr uint32_t kColO = 64;
constexpr uint32_t kTmemCols = 128;
constexpr uint32_t kThreads = 384;

// Four signed bytes -> four fp16 values, exactly: bias each byte by 128 so it
// becomes the low mantissa byte of 1024 + u (fp16 0x64uu), then subtract 1152.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t &lo, uint32_t &hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a, b;
  asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x5342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152.0
  __half2 ha = __hsub2(*reinterpret_cast<__half2 *>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<__half2 *>(&b), bias);
  lo = *reinterpret_cast<uint32_t *>(&ha);
  hi = *reinterpret_cast<uint32_t *>(&hb);
}

}  // namespace q8dec

using namespace q8dec;

__global__ void __launch_bounds__(kThreads, 1)
    mla_attend_q8_kernel(const __grid_constant__ AttendParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars *B = reinterpret_cast<Bars *>(smem + OFF_BAR);
  const uint32_t s_base = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int seg_lo = p.cta_seg[blockIdx.x];
  const int seg_hi = p.cta_seg[blockIdx.x + 1];
  volatile int *abort = &B->abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStgSlots; ++i) { mbar_init(&B->stg_full[i], 1); mbar_init(&B->stg_empty[i], 4); }
    for (int i = 0; i < kCvtSlots; ++i) { mbar_init(&B->cvt_full[i], 4); mbar_init(&B->cvt_empty[i], 1); }
    for (int i = 0; i < kRopeSlots; ++i) { mbar_init(&B->rope_full[i], 1); mbar_init(&B->rope_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->s_full[i], 1);
      mbar_init(&B->s_empty[i], 4);
      mbar_init(&B->p_full[i], 4);
      mbar_init(&B->p_empty[i], 1);
    }
    mbar_init(&B->q_full, 4);
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
  // Let a programmatically dependent merge grid get scheduled early (it waits
  // for this grid's completion before reading anything).
  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_lat8);
      tma_prefetch_desc(&p.tm_rope);
      uint32_t g = 0, n_stg = 0, n_rope = 0;
      bool ok = true;
      for (int si = seg_lo; si < seg_hi && ok; ++si) {
        const AttendSegment sg = p.segs[si];
        const long long row0 = p.seq_row0[sg.seq] + sg.tok_begin;
        const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
        for (int t = 0; t < nt && ok; ++t, ++g) {
          const int32_t y = static_cast<int32_t>(row0 + static_cast<long long>(kTileTok) * t);
          for (int c = 0; c < 4 && ok; ++c) {
            const uint32_t li = 4 * g + c, ls = li % kStgSlots;
            ok = mbar_wait(&B->stg_empty[ls], ((li / kStgSlots) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
            if (!ok) break;
            mbar_arrive_expect_tx(&B->stg_full[ls], kStgBytes);
            tma_load_2d(smem + OFF_STG + ls * kStgBytes, &p.tm_lat8, &B->stg_full[ls], 128 * c, y);
            n_stg = li + 1;
            if (c == 0) {
              const uint32_t rs = g % kRopeSlots;
              ok = mbar_wait(&B->rope_empty[rs], ((g / kRopeSlots) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
              if (!ok) break;
              mbar_arrive_expect_tx(&B->rope_full[rs], kRopeBytes);
              tma_load_2d(smem + OFF_ROPE + rs * kRopeBytes, &p.tm_rope, &B->rope_full[rs], 0, y);
              n_rope = g + 1;
            }
          }
        }
      }
      if (!ok) {
        for (uint32_t s = 0; s < kStgSlots && s < n_stg; ++s) {
          const uint32_t last = s + kStgSlots * ((n_stg - 1 - s) / kStgSlots);
          drain_wait(&B->stg_full[s], (last / kStgSlots) & 1, p.err);
        }
        for (uint32_t s = 0; s < kRopeSlots && s < n_rope; ++s) {
          const uint32_t last = s + kRopeSlots * ((n_rope - 1 - s) / kRopeSlots);
          drain_wait(&B->rope_full[s], (last / kRopeSlots) & 1, p.err);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_lat = idesc_f16(0, 0, 0, 0, 128, kHeads);   // fp16 x fp16
      constexpr uint32_t idesc_rope = idesc_f16(1, 1, 0, 0, 128, kHeads);  // bf16 x bf16
      constexpr uint32_t idesc_pv = idesc_f16(0, 0, 1, 0, 128, kHeads);    // fp16, A MN-major
      uint32_t g = 0;
      int seg_i = 0;
      bool ok = true;
      for (int si = seg_lo; si < seg_hi && ok; ++si, ++seg_i) {
        const AttendSegment sg = p.segs[si];
        const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
        ok = mbar_wait(&B->q_full, seg_i & 1, abort, p.err, ERR_TIMEOUT_FULL);
        const uint32_t q_addr = s_base + OFF_Q;
        for (int t = 0; t < nt && ok; ++t, ++g) {
          const uint32_t sb = g & 1, rs = g % kRopeSlots;
          ok = mbar_wait(&B->s_empty[sb], ((g >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY) &&
               mbar_wait(&B->rope_full[rs], (g / kRopeSlots) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint32_t rope_box = s_base + OFF_ROPE + rs * kRopeBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss(tmem + kColRope + sb * 16, smem_desc(rope_box + kk * 32, 16, 1024, LAYOUT_SW128),
                       smem_desc(q_addr + 8 * 2048 + kk * 32, 16, 1024, LAYOUT_SW128), idesc_rope, kk ? 1u : 0u);
          for (int c = 0; c < 4 && ok; ++c) {
            const uint32_t li = 4 * g + c;
            ok = mbar_wait(&B->cvt_full[li % kCvtSlots], (li / kCvtSlots) & 1, abort, p.err, ERR_TIMEOUT_FULL);
            if (!ok) break;
            tc_fence_after();
            const uint32_t slot = s_base + OFF_CVT + (li % kCvtSlots) * kCvtBytes;
#pragma unroll
            for (int half = 0; half < 2; ++half)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_f16_ss(tmem + sb * 16, smem_desc(slot + half * kBox + kk * 32, 16, 1024, LAYOUT_SW128),
                           smem_desc(q_addr + (2 * c + half) * 2048 + kk * 32, 16, 1024, LAYOUT_SW128), idesc_lat,
                           (c | half | kk) ? 1u : 0u);
          }
          if (!ok) break;
          mma_commit(&B->s_full[sb]);
          mma_commit(&B->rope_empty[rs]);
          const bool first = (t == 0);
          ok = mbar_wait(&B->p_full[sb], (g >> 1) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (ok && first && seg_i > 0) ok = mbar_wait(&B->o_empty, (seg_i - 1) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint32_t p_addr = s_base + OFF_P + sb * kPBytes;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t li = 4 * g + c;
            const uint32_t slot = s_base + OFF_CVT + (li % kCvtSlots) * kCvtBytes;
#pragma unroll
            for (int kk = 0; kk < kTileTok / 16; ++kk)
              mma_f16_ss(tmem + kColO + 16 * c, smem_desc(slot + kk * 2048, kBox, 1024, LAYOUT_SW128),
                         smem_desc(p_addr + kk * 256, 128, kPChunkSbo, LAYOUT_INTERLEAVE), idesc_pv,
                         (first && kk == 0) ? 0u : 1u);
            mma_commit(&B->cvt_empty[li % kCvtSlots]);
          }
          mma_commit(&B->p_empty[sb]);
        }
        if (ok) mma_commit(&B->o_full);
      }
      mma_commit(&B->drain);
      drain_wait(&B->drain, 0, p.err);
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ converters
    const int ct = threadIdx.x - 256;  // 0..127
    uint32_t g = 0;
    bool ok = true;
    for (int si = seg_lo; si < seg_hi && ok; ++si) {
      const AttendSegment sg = p.segs[si];
      const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
      for (int t = 0; t < nt && ok; ++t, ++g) {
        for (int c = 0; c < 4; ++c) {
          const uint32_t li = 4 * g + c, ss = li % kStgSlots, cs = li % kCvtSlots;
          int w_ok = 1;
          if (lane == 0) {
            w_ok = mbar_wait(&B->stg_full[ss], (li / kStgSlots) & 1, abort, p.err, ERR_TIMEOUT_FULL) &&
                   mbar_wait(&B->cvt_empty[cs], ((li / kCvtSlots) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
          }
          w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
          if (!w_ok) { ok = false; break; }
          const uint8_t *src = smem + OFF_STG + ss * kStgBytes;
          uint8_t *dst = smem + OFF_CVT + cs * kCvtBytes;
#pragma unroll 4
          for (int i = 0; i < 8; ++i) {
            const int idx = ct + 128 * i;  // 1024 chunks of 16 int8 (128 rows x 8)
            const int row = idx >> 3, k = idx & 7;
            const uint4 v = *reinterpret_cast<const uint4 *>(src + row * 128 + ((k ^ (row & 7)) << 4));
            uint4 o0, o1;
            i8x4_to_f16x4(v.x, o0.x, o0.y);
            i8x4_to_f16x4(v.y, o0.z, o0.w);
            i8x4_to_f16x4(v.z, o1.x, o1.y);
            i8x4_to_f16x4(v.w, o1.z, o1.w);
            // dims 16k..16k+15 of this 128-dim chunk -> fp16 box (k >> 2), 16B chunks 2(k&3), 2(k&3)+1
            uint8_t *box = dst + (k >> 2) * kBox;
            const int fc = 2 * (k & 3);
            *reinterpret_cast<uint4 *>(box + sw128_offset(row, fc * 8)) = o0;
            *reinterpret_cast<uint4 *>(box + sw128_offset(row, fc * 8 + 8)) = o1;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&B->stg_empty[ss]);
            mbar_arrive(&B->cvt_full[cs]);
          }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue
    const int w = warp - 4;
    const int tt = 32 * w + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * w) << 16;
    uint32_t g = 0;
    int seg_i = 0;
    for (int si = seg_lo; si < seg_hi; ++si, ++seg_i) {
      const AttendSegment sg = p.segs[si];
      const long long srow0 = p.seq_row0[sg.seq];
      const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
      // The query tile is free here: every score MMA of the previous segment
      // has completed (its scores were read above).
      load_query_tile(smem + OFF_Q, p.q + static_cast<size_t>(sg.seq) * kHeads * kRow, tt, true);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->q_full);
      float m_ref[kHeads], l_part[kHeads];
#pragma unroll
      for (int h = 0; h < kHeads; ++h) { m_ref[h] = -INFINITY; l_part[h] = 0.f; }
      bool bad = false;
      for (int t = 0; t < nt; ++t, ++g) {
        const int tok = sg.tok_begin + kTileTok * t + tt;
        const bool valid = tok < sg.tok_end;
        const float rs = valid ? p.latent_scale[srow0 + tok] : 0.f;
        const uint32_t sb = g & 1;
        bad = !mbar_wait(&B->s_full[sb], (g >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (named_bar_or(1, 128, bad)) { bad = true; break; }
        tc_fence_after();
        float vl[kHeads], vr[kHeads];
        tmem_ld16(tmem + sb * 16 + lane_base, vl);
        tmem_ld16(tmem + kColRope + sb * 16 + lane_base, vr);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->s_empty[sb]);
        float s[kHeads];
        bool need = false;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          s[h] = valid ? fmaf(rs, vl[h], vr[h]) * p.scale_log2 : -INFINITY;
          need |= s[h] > m_ref[h] + 8.0f;
        }
        if (named_bar_or(1, 128, need)) {
          float mx[kHeads];
#pragma unroll
          for (int h = 0; h < kHeads; ++h) mx[h] = s[h];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int h = 0; h < kHeads; ++h) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
          if (lane == 0)
#pragma unroll
            for (int h = 0; h < kHeads; ++h) B->red[w][h] = mx[h];
          named_bar_sync(1, 128);
          float alpha[kHeads];
#pragma unroll
          for (int h = 0; h < kHeads; ++h) {
            const float tm = fmaxf(fmaxf(B->red[0][h], B->red[1][h]), fmaxf(B->red[2][h], B->red[3][h]));
            const float mn = fmaxf(m_ref[h], tm);
            alpha[h] = (m_ref[h] == -INFINITY) ? 0.f : exp2f(m_ref[h] - mn);
            m_ref[h] = mn;
          }
          named_bar_sync(1, 128);
          if (t > 0) {
            bad = !mbar_wait(&B->p_empty[(g - 1) & 1], ((g - 1) >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
            if (named_bar_or(1, 128, bad)) { bad = true; break; }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float o[kHeads];
              tmem_ld16(tmem + kColO + 16 * c + lane_base, o);
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < kHeads; ++h) o[h] *= alpha[h];
              tmem_st16(tmem + kColO + 16 * c + lane_base, o);
            }
            tmem_wait_st();
          }
#pragma unroll
          for (int h = 0; h < kHeads; ++h) l_part[h] *= alpha[h];
        }
        float pr[kHeads];
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          pr[h] = exp2f(s[h] - m_ref[h]);
          l_part[h] += pr[h];
        }
        bad = !mbar_wait(&B->p_empty[sb], ((g >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (named_bar_or(1, 128, bad)) { bad = true; break; }
        {
          // Rows past the segment end carry rs = 0, so P' = 0; the converted
          // int8 rows are always finite, so 0 * row is 0 in the P.V MMA.
          uint8_t *pd = smem + OFF_P + sb * kPBytes + (tt >> 3) * 128 + (tt & 7) * 2;
#pragma unroll
          for (int h = 0; h < kHeads; ++h)
            *reinterpret_cast<__half *>(pd + (h >> 3) * kPChunkSbo + (h & 7) * 16) = __float2half_rn(pr[h] * rs);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->p_full[sb]);
      }
      if (bad) break;
      bad = !mbar_wait(&B->o_full, seg_i & 1, abort, p.err, ERR_TIMEOUT_MMA);
      if (named_bar_or(1, 128, bad)) break;
      tc_fence_after();
      float lt[kHeads];
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        float l = l_part[h];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        lt[h] = l;
      }
      if (lane == 0)
#pragma unroll
        for (int h = 0; h < kHeads; ++h) B->red[w][h] = lt[h];
      named_bar_sync(1, 128);
#pragma unroll
      for (int h = 0; h < kHeads; ++h) lt[h] = (B->red[0][h] + B->red[1][h]) + (B->red[2][h] + B->red[3][h]);
      named_bar_sync(1, 128);
      float *dst = (sg.slot < 0) ? p.out + static_cast<size_t>(sg.seq) * kHeads * kLatent
                                 : p.part_o + static_cast<size_t>(sg.slot) * kHeads * kLatent;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float o[kHeads];
        tmem_ld16(tmem + kColO + 16 * c + lane_base, o);
        tmem_wait_ld();
        const int d = 128 * c + 32 * w + lane;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) dst[h * kLatent + d] = o[h] / lt[h];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->o_empty);
      if (w == 0 && lane < kHeads) {
        float m = 0.f, l = 1.f;
#pragma unroll
        for (int h = 0; h < kHeads; ++h)
          if (h == lane) { m = m_ref[h]; l = lt[h]; }
        const float lse = (m + log2f(l)) * 0.69314718055994531f;
        float *ldst = (sg.slot < 0) ? p.lse : p.part_lse;
        const int row = (sg.slot < 0) ? sg.seq : sg.slot;
        if (ldst) ldst[row * kHeads + lane] = lse;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

cudaError_t launch_attend_q8(const AttendParams &p, int grid, cudaStream_t stream) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(mla_attend_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  ProfScope ps("mla_attend_q8", stream);
  mla_attend_q8_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace kvl
