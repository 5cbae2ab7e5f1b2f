// attend_bf16.cu -- absorbed MLA decode attention over a bf16 latent state on
// sm_100a: TMA streams 128-row KV tiles into shared memory, tcgen05 computes
// the scores S^T[128 rows x 16 heads] and the mix O^T[512 x 16 heads] into
// tensor memory, and four softmax warps run an online softmax between them.
//
// Reference semantics: src/mla_compressed_state.c:132-148 (attend core of
// kvl_mla_decode_compressed_bf16).  Format choices of this build: the cached
// rows are bf16 (the reference keeps fp32 rows), the absorbed query is rounded
// to bf16 for the tensor core, the probabilities are rounded to bf16 for the
// P.V MMA, and accumulation is fp32 instead of double.
//
// Cost model (measured on B200): a kind::f16 tcgen05.mma with N=16 takes ~48
// cycles whether M is 64 or 128, so rows go on M=128 and a 128-row tile costs
// 36 score MMAs + 32 P.V MMAs.  Shared memory holds one tile plus one chunk:
//   latent ring  5 slots x 32 KB (128 rows x 128 dims = two SW128 boxes), a
//                tile uses 4; a slot is released as soon as its P.V MMAs end
//   rope ring    2 slots x 16 KB (128 rows x 64 dims), released after scores
// and the MMA issuer runs scores(t), then P.V(t) once the softmax has written
// P(t), so the next tile's chunks stream in behind the P.V of this one.
//
// Roles (256 threads, one CTA per SM):
//   warp 0      TMA producer
//   warp 1      TMEM owner and tcgen05 issuer
//   warp 2      query loader: one bulk copy per segment of the bf16 query tile
//               that qprep_bf16_kernel writes before the attend
//   warps 4-7   softmax and epilogue (TMEM subpartitions 0-3; thread = KV row)
#include "attend_common.cuh"
#include "pdl.cuh"
#include "prof.cuh"
#include "sm100.cuh"

namespace kvl {
namespace bf16dec {

constexpr int kLatSlots = 5;
constexpr int kRopeSlots = 2;
constexpr uint32_t kBox = kTileTok * 128;       // 128 rows x 64 dims bf16 = 16 KB
constexpr uint32_t kLatSlotBytes = 2 * kBox;    // 128 dims
constexpr uint32_t kRopeSlotBytes = kBox;       // 64 dims
constexpr uint32_t kQBytes = 9 * 2048;          // 16 heads x 576: nine SW128 boxes of 16 rows
constexpr uint32_t kPChunkSbo = (kTileTok / 8) * 128;  // stride between the two 8-head groups
constexpr uint32_t kPBytes = 2 * kPChunkSbo;    // P^T: 16 heads x 128 rows, 8x16B core matrices
constexpr uint32_t OFF_LAT = 0;
constexpr uint32_t OFF_ROPE = OFF_LAT + kLatSlots * kLatSlotBytes;
constexpr uint32_t OFF_Q = OFF_ROPE + kRopeSlots * kRopeSlotBytes;
constexpr uint32_t OFF_P = OFF_Q + kQBytes;
constexpr uint32_t OFF_BAR = OFF_P + 2 * kPBytes;

struct Bars {
  uint64_t lat_full[kLatSlots], lat_empty[kLatSlots];
  uint64_t rope_full[kRopeSlots], rope_empty[kRopeSlots];
  uint64_t q0_full, q_full, q_empty;
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full[2], o_empty[2], drain;
  uint32_t tmem_base;
  int abort;
  float red[4][kHeads];
};

constexpr uint32_t kSmemBytes = OFF_BAR + sizeof(Bars) + 1024;  // + alignment slack
static_assert(OFF_ROPE % 1024 == 0 && OFF_Q % 1024 == 0 && OFF_P % 1024 == 0 && OFF_BAR % 8 == 0, "align");
static_assert(kSmemBytes <= 232448, "shared memory budget");

// S: 2 buffers x 16 columns @0; O: kOBufs buffers (by segment index) x 4
// chunks x 16 columns @32.  Two O buffers let a segment's first P.V skip the
// wait for the previous segment's epilogue, but the 256-column allocation they
// need measured 2 us slower on the single-sequence long decode (60.4 against
// 58.4 us at L = 131072) for 1 % on batched decode, so one buffer it is.
constexpr uint32_t kOBufs = 1;  // O accumulators (by segment index mod kOBufs)
constexpr uint32_t kTmemCols = kOBufs == 2 ? 256 : 128;
constexpr uint32_t kColO = 32;
constexpr uint32_t kOCols = 64;
constexpr int kLoaderWarp = 2;  // bulk-loads each segment's query image
constexpr uint32_t kThreads = 256;

}  // namespace bf16dec

using namespace bf16dec;

// At most 192 registers: a merge block (256 threads x 64 registers) must fit
// beside a resident attend CTA (256 x 192) in the 65,536 registers of an SM,
// so that the merge grid, launched as the attend's programmatic dependent,
// waits on the SMs and starts the moment the attend grid completes.  With 208
// registers it did not fit, and config 5 (attend + merge) went from 58.4 to
// 60.4 us, a 64 x 32768 batch from 478 to 484 us.  (A reciprocal per head in
// the epilogue instead of a division per element took config 5 to 56.3 us
// under this cap but the batch to 486 us, so the epilogue divides.)
// kFirstAlone (launches of few tiles per CTA, p.first_tile_alone): the copies
// beyond a CTA's first tile wait for that tile to land.  A separate
// instantiation, so that long batches run exactly the code without it.
template <bool kFirstAlone>
__global__ void __maxnreg__(192)
    mla_attend_bf16_kernel(const __grid_constant__ AttendParams p) {
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
    for (int i = 0; i < kLatSlots; ++i) { mbar_init(&B->lat_full[i], 1); mbar_init(&B->lat_empty[i], 1); }
    for (int i = 0; i < kRopeSlots; ++i) { mbar_init(&B->rope_full[i], 1); mbar_init(&B->rope_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->s_full[i], 1);
      mbar_init(&B->s_empty[i], 4);
      mbar_init(&B->p_full[i], 4);
      mbar_init(&B->p_empty[i], 1);
    }
    mbar_init(&B->q0_full, 4);  // the softmax warps write the first segment's query
    mbar_init(&B->q_full, 1);   // the loader's expect-tx arrival (later segments)
    mbar_init(&B->q_empty, 1);  // the issuer's commit after the segment's last scores
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->o_full[i], 1);
      mbar_init(&B->o_empty[i], 4);
    }
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
      tma_prefetch_desc(&p.tm_kv);
      uint32_t g = 0, n_lat = 0, n_rope = 0;
      bool ok = true;
      for (int si = seg_lo; si < seg_hi && ok; ++si) {
        const AttendSegment sg = p.segs[si];
        const long long row0 = sg.row0 + sg.tok_begin;
        const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
        for (int t = 0; t < nt && ok; ++t, ++g) {
          const int32_t y = static_cast<int32_t>(row0 + static_cast<long long>(kTileTok) * t);
          for (int c = 0; c < 4 && ok; ++c) {
            const uint32_t li = 4 * g + c, ls = li % kLatSlots;
            // With few tiles per CTA, the copies beyond the first tile wait for
            // it to land, so the whole grid's first tiles are not queued behind
            // the prefetch of second ones (config 5: 58.4 -> 56.3 us; with ~57
            // tiles per CTA it cost 1 %, so the plan turns it off there).
            if (kFirstAlone && li == 4 && !(ok = mbar_wait(&B->lat_full[3], 0, abort, p.err, ERR_TIMEOUT_FULL)))
              break;
            ok = mbar_wait(&B->lat_empty[ls], ((li / kLatSlots) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
            if (!ok) break;
            uint8_t *dst = smem + OFF_LAT + ls * kLatSlotBytes;
            mbar_arrive_expect_tx(&B->lat_full[ls], kLatSlotBytes);
            tma_load_2d(dst, &p.tm_kv, &B->lat_full[ls], 128 * c, y);
            tma_load_2d(dst + kBox, &p.tm_kv, &B->lat_full[ls], 128 * c + 64, y);
            n_lat = li + 1;
            if (c == 0) {
              // the rope box rides with the first chunk so scores can start early
              const uint32_t rs = g % kRopeSlots;
              ok = mbar_wait(&B->rope_empty[rs], ((g / kRopeSlots) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
              if (!ok) break;
              mbar_arrive_expect_tx(&B->rope_full[rs], kRopeSlotBytes);
              tma_load_2d(smem + OFF_ROPE + rs * kRopeSlotBytes, &p.tm_kv, &B->rope_full[rs], kLatent, y);
              n_rope = g + 1;
            }
          }
        }
      }
      if (!ok) {
        // Drain: the most recent load issued into each slot must land before
        // the CTA exits (earlier ones completed before the slot was reissued).
        for (uint32_t s = 0; s < kLatSlots && s < n_lat; ++s) {
          const uint32_t last = s + kLatSlots * ((n_lat - 1 - s) / kLatSlots);
          drain_wait(&B->lat_full[s], (last / kLatSlots) & 1, p.err);
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
      constexpr uint32_t idesc_qk = idesc_f16(1, 1, 0, 0, 128, kHeads);  // A = KV rows (K-major)
      constexpr uint32_t idesc_pv = idesc_f16(1, 1, 1, 0, 128, kHeads);  // A = latent^T (MN-major)
      uint32_t g = 0;
      int seg_i = 0;
      bool ok = true;
      AttendSegment nx = p.segs[seg_lo];  // descriptors are read one segment ahead
      for (int si = seg_lo; si < seg_hi && ok; ++si, ++seg_i) {
        const AttendSegment sg = nx;
        if (si + 1 < seg_hi) nx = p.segs[si + 1];
        const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
        const uint32_t ob = seg_i % kOBufs;  // this segment's O buffer
        ok = seg_i == 0 ? mbar_wait(&B->q0_full, 0, abort, p.err, ERR_TIMEOUT_FULL)
                        : mbar_wait(&B->q_full, (seg_i - 1) & 1, abort, p.err, ERR_TIMEOUT_FULL);
        const uint32_t q_addr = s_base + OFF_Q;
        for (int t = 0; t < nt && ok; ++t, ++g) {
          // ---- scores S^T(g) = KV(g) . Q^T
          const uint32_t sb = g & 1, rs = g % kRopeSlots;
          ok = mbar_wait(&B->s_empty[sb], ((g >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY) &&
               mbar_wait(&B->rope_full[rs], (g / kRopeSlots) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint32_t rope_box = s_base + OFF_ROPE + rs * kRopeSlotBytes;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss(tmem + sb * 16, smem_desc(rope_box + kk * 32, 16, 1024, LAYOUT_SW128),
                       smem_desc(q_addr + 8 * 2048 + kk * 32, 16, 1024, LAYOUT_SW128), idesc_qk, kk ? 1u : 0u);
          for (int c = 0; c < 4 && ok; ++c) {
            const uint32_t li = 4 * g + c;
            ok = mbar_wait(&B->lat_full[li % kLatSlots], (li / kLatSlots) & 1, abort, p.err, ERR_TIMEOUT_FULL);
            if (!ok) break;
            tc_fence_after();
            const uint32_t slot = s_base + OFF_LAT + (li % kLatSlots) * kLatSlotBytes;
#pragma unroll
            for (int half = 0; half < 2; ++half)
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_f16_ss(tmem + sb * 16, smem_desc(slot + half * kBox + kk * 32, 16, 1024, LAYOUT_SW128),
                           smem_desc(q_addr + (2 * c + half) * 2048 + kk * 32, 16, 1024, LAYOUT_SW128), idesc_qk,
                           1u);
          }
          if (!ok) break;
          mma_commit(&B->s_full[sb]);
          mma_commit(&B->rope_empty[rs]);
          // the query tile is free once the segment's last scores are done
          if (t + 1 == nt) mma_commit(&B->q_empty);
          // ---- O^T += latent(g)^T . P^T(g), slot by slot
          const bool first = (t == 0);
          ok = mbar_wait(&B->p_full[sb], (g >> 1) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          // O buffer ob was last read by the epilogue of segment seg_i - kOBufs
          if (ok && first && seg_i >= static_cast<int>(kOBufs))
            ok = mbar_wait(&B->o_empty[ob], (seg_i / kOBufs - 1) & 1, abort, p.err, ERR_TIMEOUT_FULL);
          if (!ok) break;
          tc_fence_after();
          const uint32_t p_addr = s_base + OFF_P + sb * kPBytes;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t li = 4 * g + c;
            const uint32_t slot = s_base + OFF_LAT + (li % kLatSlots) * kLatSlotBytes;
#pragma unroll
            for (int kk = 0; kk < kTileTok / 16; ++kk)
              mma_f16_ss(tmem + kColO + kOCols * ob + 16 * c, smem_desc(slot + kk * 2048, kBox, 1024, LAYOUT_SW128),
                         smem_desc(p_addr + kk * 256, 128, kPChunkSbo, LAYOUT_INTERLEAVE), idesc_pv,
                         (first && kk == 0) ? 0u : 1u);
            mma_commit(&B->lat_empty[li % kLatSlots]);
          }
          mma_commit(&B->p_empty[sb]);
        }
        if (ok) mma_commit(&B->o_full[ob]);
      }
      // All issued tensor-core work must finish before TMEM is released.
      mma_commit(&B->drain);
      drain_wait(&B->drain, 0, p.err);
    }
  } else if (warp == kLoaderWarp) {
    // ------------------------------------------------------------ query loader
    // From the CTA's second segment on: one bulk copy of the segment's query
    // image (prepared by qprep_bf16_kernel, this grid's programmatic
    // predecessor, launched when some CTA has more than one segment) once the
    // previous segment's last score MMAs are done.  The first segment's query
    // is converted by the softmax warps themselves, so no CTA waits for the
    // prep kernel at its start.
    if (lane == 0) {
      uint32_t issued = 0;
      bool ok = true;
      for (int si = seg_lo + 1, seg_i = 1; si < seg_hi; ++si, ++seg_i) {
        const int seq = p.segs[si].seq;
        ok = mbar_wait(&B->q_empty, (seg_i - 1) & 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
        if (seg_i == 1) asm volatile("griddepcontrol.wait;" ::: "memory");
        mbar_arrive_expect_tx(&B->q_full, kQImgBf16Bytes);
        bulk_load(smem + OFF_Q, p.qimg + static_cast<size_t>(seq) * kQImgStride, kQImgBf16Bytes, &B->q_full);
        ++issued;
      }
      // the last copy must land before the CTA exits
      if (!ok && issued > 0) drain_wait(&B->q_full, (issued - 1) & 1, p.err);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue
    const int w = warp - 4;
    const int tt = 32 * w + lane;  // KV row of the tile owned by this thread
    const uint32_t lane_base = static_cast<uint32_t>(32 * w) << 16;
    uint32_t g = 0;
    int seg_i = 0;
    AttendSegment nx = p.segs[seg_lo];  // descriptors are read one segment ahead
    for (int si = seg_lo; si < seg_hi; ++si, ++seg_i) {
      const AttendSegment sg = nx;
      if (si + 1 < seg_hi) nx = p.segs[si + 1];
      const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
      const uint32_t ob = seg_i % kOBufs;  // this segment's O buffer
      const uint32_t col_o = tmem + kColO + kOCols * ob;
      if (seg_i == 0) {
        if (p.q_after_wait) pdl_wait();
        load_query_tile(smem + OFF_Q, p.q + static_cast<size_t>(sg.seq) * kHeads * kRow, tt);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->q0_full);
      }
      float m_ref[kHeads], l_part[kHeads];
#pragma unroll
      for (int h = 0; h < kHeads; ++h) { m_ref[h] = -INFINITY; l_part[h] = 0.f; }
      bool bad = false;
      for (int t = 0; t < nt; ++t, ++g) {
        const uint32_t sb = g & 1;
        bad = !mbar_wait(&B->s_full[sb], (g >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
        // the P buffer of this tile is free by now (P.V of tile g - 2 ended
        // before the scores of tile g - 1 started); its wait rides on the
        // same barrier as the scores' wait and the rescale vote
        bad |= !mbar_wait(&B->p_empty[sb], ((g >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_MMA);
        tc_fence_after();
        float v[kHeads];
        tmem_ld16(tmem + sb * 16 + lane_base, v);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->s_empty[sb]);
        const int tok = sg.tok_begin + kTileTok * t + tt;
        const bool valid = tok < sg.tok_end;
        float s[kHeads];
        bool need = false;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          s[h] = valid ? v[h] * p.scale_log2 : -INFINITY;
          need |= s[h] > m_ref[h] + 8.0f;
        }
        if (named_bar_or(1, 128, need || bad)) {
          if (named_bar_or(1, 128, bad)) { bad = true; break; }
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
            // O holds tiles [0, t) of this segment: rescale after P.V(t-1) lands.
            bad = !mbar_wait(&B->p_empty[(g - 1) & 1], ((g - 1) >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
            if (named_bar_or(1, 128, bad)) { bad = true; break; }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float o[kHeads];
              tmem_ld16(col_o + 16 * c + lane_base, o);
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < kHeads; ++h) o[h] *= alpha[h];
              tmem_st16(col_o + 16 * c + lane_base, o);
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
        if (!valid) {
          // Rows past the segment end get p = 0, but 0 * (NaN/Inf garbage) is
          // NaN in the P.V MMA: clear their latent rows (the score MMAs of this
          // tile have completed, so the slots may be modified).
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint8_t *row = smem + OFF_LAT + ((4 * g + c) % kLatSlots) * kLatSlotBytes + tt * 128;
#pragma unroll
            for (int half = 0; half < 2; ++half)
#pragma unroll
              for (int k = 0; k < 8; ++k)
                *reinterpret_cast<uint4 *>(row + half * kBox + k * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        {
          uint8_t *pd = smem + OFF_P + sb * kPBytes + (tt >> 3) * 128 + (tt & 7) * 2;
#pragma unroll
          for (int h = 0; h < kHeads; ++h)
            *reinterpret_cast<__nv_bfloat16 *>(pd + (h >> 3) * kPChunkSbo + (h & 7) * 16) =
                __float2bfloat16_rn(pr[h]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->p_full[sb]);
      }
      if (bad) break;
      // ---- epilogue: O / l, lse
      bad = !mbar_wait(&B->o_full[ob], (seg_i / kOBufs) & 1, abort, p.err, ERR_TIMEOUT_MMA);
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
        tmem_ld16(col_o + 16 * c + lane_base, o);
        tmem_wait_ld();
        const int d = 128 * c + 32 * w + lane;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) dst[h * kLatent + d] = o[h] / lt[h];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->o_empty[ob]);
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

// The query images of a launch: block b converts sequence b's absorbed query
// ([16][576] fp32) into the bf16 SW128 tile the score MMAs read (128 threads).
// The attend grid is its programmatic dependent and may start as soon as this
// grid is past its own wait; only the attend's loader waits for this grid.
__global__ void __launch_bounds__(128) qprep_bf16_kernel(const float *q, uint8_t *img) {
  // launched as a programmatic dependent of the query's producer: the attend
  // (this grid's dependent) is released only after that producer is done, so
  // the query rows it reads before its own wait are complete
  pdl_wait();
  pdl_trigger();
  load_query_tile(img + static_cast<size_t>(blockIdx.x) * kQImgStride,
                  q + static_cast<size_t>(blockIdx.x) * kHeads * kRow, threadIdx.x);
}

template <bool kFirstAlone>
static cudaError_t attend_bf16_grid(const AttendParams &p, int grid, bool qprep, cudaStream_t stream) {
  static std::atomic<unsigned long long> opted{0};
  const void *fn = reinterpret_cast<const void *>(mla_attend_bf16_kernel<kFirstAlone>);
  cudaError_t e = smem_opt_in(fn, kSmemBytes, opted);
  if (e != cudaSuccess) return e;
  // A programmatic dependent of the prep kernel (its loader waits for the
  // images; the prep releases it after its own wait, so every input the kernel
  // reads directly is complete by then), or of the query's producer when
  // q_after_wait is set; otherwise an ordinary launch.
  if (qprep || p.q_after_wait) return launch_pdl(fn, grid, kThreads, kSmemBytes, stream, p);
  mla_attend_bf16_kernel<kFirstAlone><<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

static cudaError_t attend_bf16_launches(const AttendParams &p, int grid, int batch, bool qprep, cudaStream_t stream,
                                        bool profiled) {
  cudaError_t e = cudaSuccess;
  if (qprep) {
    ProfScope ps(profiled ? "qprep_bf16" : nullptr, stream);
    e = launch_dependent(qprep_bf16_kernel, dim3(batch), dim3(128), 0, stream, p.q, const_cast<uint8_t *>(p.qimg));
    if (e != cudaSuccess) return e;
  }
  ProfScope ps(profiled ? "mla_attend_bf16" : nullptr, stream);
  return p.first_tile_alone ? attend_bf16_grid<true>(p, grid, qprep, stream)
                            : attend_bf16_grid<false>(p, grid, qprep, stream);
}

// Host launcher: the query prep for `batch` sequences (only when some CTA of
// the plan has more than one segment: `qprep`), then the attend grid.
cudaError_t launch_attend_bf16(const AttendParams &p, int grid, int batch, bool qprep, cudaStream_t stream) {
  return attend_bf16_launches(p, grid, batch, qprep, stream, true);
}

// Same launches without the optional per-kernel timing, whose CUDA events are
// created on demand: used by the entry point that must not allocate.
cudaError_t launch_attend_bf16_unprofiled(const AttendParams &p, int grid, int batch, bool qprep,
                                         cudaStream_t stream) {
  return attend_bf16_launches(p, grid, batch, qprep, stream, false);
}

}  // namespace kvl
