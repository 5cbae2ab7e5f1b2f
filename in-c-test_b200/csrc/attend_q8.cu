// attend_q8.cu -- absorbed MLA decode attention over the row-wise Q8 latent
// state (int8 latent [rows][512], fp32 scale [rows], bf16 rope [rows][64]: the
// reference's layout, include/kvl/mla_compressed_q8_state.h).
//
// Reference semantics: src/mla_compressed_q8_state.c:216-238, with the
// dequantised row latent_j = (float)q_j * scale_j (:57-61).  Both contractions
// run on the int8 tensor-core path (tcgen05 kind::i8, int32 accumulation)
// straight from the int8 rows TMA brings in -- no conversion pass:
//
//   scores  q_lat is split per head into two int8 parts, q ~ sq * (hi + lo/256)
//           (sq = max|q_lat| / 127, so about 16 bits of precision); both parts
//           go into one N = 32 MMA against the int8 rows (exact int32 sums), and
//             s_j = scale_j * sq * (S_hi + S_lo / 256) + q_rope . rope_j
//           with the rope term on the bf16 tensor core (fp32 accumulation).
//   mix     P'_j = p_j * scale_j is split per head and tile the same way,
//           P' ~ sp * (hi + lo/256) (sp = max_j |P'_j| / 127), and the P.V MMA
//           reads the same int8 rows as an MN-major operand: per tile
//             O += sp * (O_hi + O_lo / 256)
//           folded into fp32 register accumulators by the softmax threads.
// The int32 sums are exact; the roundings are the two 16-bit splits, q_rope
// to bf16 for the rope term, and fp32 arithmetic (the reference accumulates in
// double).
//
// Tiles of 128 KV rows.  Shared memory is one ring of 12 boxes of 16 KB
// (128 rows x 128 B): a tile is five boxes -- the bf16 rope and four 128-dim
// int8 chunks -- so the producer runs about two tiles ahead.  The rope box is
// released when the tile's score MMAs end, a chunk when its P.V MMAs end.
// Within a segment the issuer runs the scores of tile g+1 before the P.V of
// tile g, so the tensor pipe works while the softmax of tile g runs.
//
// Roles (608 threads, one CTA per SM):
//   warp 0       TMA producer
//   warp 1       TMEM owner and tcgen05 issuer
//   warps 2-17   four warpgroups of four heads each: softmax, P' split, fold
//                of the per-tile P.V sums, epilogue (thread = KV row of the
//                tile for the scores, = latent dim of each 128-dim chunk for
//                the mix).  Four heads per thread keep the per-tile softmax
//                short enough to hide under the tile's HBM time (eight heads
//                per thread took ~3k cycles per tile, close to the period).
//   warp 18      query loader: one bulk copy per segment of the query image
//                (int8 parts, bf16 q_rope and the per-head scale) that
//                qprep_q8_kernel writes before the attend, so a segment
//                boundary costs one copy latency instead of the softmax warps
//                splitting the next query after their epilogue
#include "attend_common.cuh"
#include "pdl.cuh"
#include "prof.cuh"
#include "sm100.cuh"

namespace kvl {
namespace q8dec {

constexpr int kSlots = 12;
constexpr int kBoxesPerTile = 5;               // rope + four int8 chunks
constexpr uint32_t kBox = kTileTok * 128;      // 128 rows x 128 B = 16 KB
constexpr uint32_t kQiBytes = 4 * 32 * 128;    // q parts [32][512] int8: four SW128 boxes of 32 rows
constexpr uint32_t kQrBytes = kHeads * 128;    // q_rope [16][64] bf16: one SW128 box
constexpr uint32_t kPBytes = 128 * 32;         // P' parts [128 KV rows][32] int8, MN-major, 32-byte swizzle
constexpr uint32_t OFF_RING = 0;
constexpr uint32_t OFF_QI = OFF_RING + kSlots * kBox;
constexpr uint32_t OFF_QR = OFF_QI + kQiBytes;
constexpr uint32_t OFF_QS = OFF_QR + kQrBytes;  // sq [16] fp32, loaded with the query image
constexpr uint32_t OFF_P = OFF_QS + 1024;
static_assert(OFF_QS - OFF_QI + kHeads * 4 == kQImgQ8Bytes, "the query image is qi | qr | sq");
constexpr uint32_t OFF_BAR = OFF_P + 2 * kPBytes;

struct Bars {
  uint64_t full[kSlots], empty[kSlots];
  uint64_t q0_full, q_full, q_empty;
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full[2], p_empty[2];
  uint64_t o_full[2], o_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float red[4][4][4];          // per warpgroup: running-max / sum exchange
  float pmax[2][4][4][4];      // per tile parity and warpgroup: max |P'| of each warp
};

constexpr uint32_t kSmemBytes = OFF_BAR + sizeof(Bars) + 1024;
static_assert(OFF_QI % 1024 == 0 && OFF_QR % 1024 == 0 && OFF_P % 1024 == 0 && OFF_BAR % 8 == 0, "align");
static_assert(kSmemBytes <= 232448, "shared memory budget");

// TMEM columns: int32 scores 2 x 32 (heads hi | lo) @0, fp32 rope scores
// 2 x 16 @64, int32 P.V sums 2 buffers x 4 chunks x 32 @128.
constexpr uint32_t kColS = 0;
constexpr uint32_t kColR = 64;
constexpr uint32_t kColO = 128;
constexpr uint32_t kTmemCols = 512;
// Softmax warpgroups: four groups of four heads.  A group is four
// consecutive warps 2 + 4 wg .. 5 + 4 wg, which cover the four TMEM
// subpartitions (warp w reads lanes 32 (w % 4) ..) in rotated order.
constexpr int kWGs = 4;
constexpr int kHPW = kHeads / kWGs;
constexpr int kLoaderWarp = 2 + 4 * kWGs;  // bulk-loads each segment's query image
constexpr uint32_t kThreads = 32 * (kLoaderWarp + 1);
constexpr uint32_t LAYOUT_SW32 = 6;  // tcgen05 shared-memory descriptor: 32-byte swizzle

// Byte offset of (row n, byte k) in an SW128 K-major box of 128-byte rows.
__device__ __forceinline__ uint32_t sw128_byte(uint32_t n, uint32_t k) {
  return (n >> 3) * 1024u + (n & 7u) * 128u + ((((k >> 4) ^ n) & 7u) << 4) + (k & 15u);
}

// v ~ s * (hi + lo / 256) with hi, lo int8; x = v / s in [-127, 127].
__device__ __forceinline__ void split16(float x, int &hi, int &lo) {
  const float h = rintf(x);
  float l = rintf((x - h) * 256.0f);
  l = fminf(fmaxf(l, -127.0f), 127.0f);
  hi = static_cast<int>(h);
  lo = static_cast<int>(l);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

// One unit of the absorbed query of a sequence ([16][576] fp32) as score
// operands: q_lat split into int8 hi (rows 0-15) and lo (rows 16-31) parts,
// K-major over four SW128 boxes of 128 dims, and q_rope as one bf16 SW128 box.
// Unit u (0..255) is head u / 16, latent dims 32 * (u % 16) .. +31 and rope
// dims 4 * (u % 16) .. +3; the sixteen units of a head are sixteen
// consecutive lanes (one half-warp).
// The loads of unit u, issued before any use so that a caller can signal
// that they are in flight (query_unit_split below finishes the unit).
struct QueryUnitLoads {
  float4 v[8], r0;
};
__device__ __forceinline__ void query_unit_load(const float *q, int u, QueryUnitLoads &ld) {
  const int h = u >> 4, j = u & 15;
  const float *src = q + h * kRow + 32 * j;
#pragma unroll
  for (int i = 0; i < 8; ++i) ld.v[i] = *reinterpret_cast<const float4 *>(src + 4 * i);
  ld.r0 = *reinterpret_cast<const float4 *>(q + h * kRow + kLatent + 4 * j);
}

__device__ __forceinline__ void query_unit_split(uint8_t *qi, uint8_t *qr, float *qscale, int u,
                                                 const QueryUnitLoads &ld) {
  const int h = u >> 4, j = u & 15;
  const float4 *v = ld.v;
  const float4 r0 = ld.r0;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float inv = amax > 0.f ? 127.0f / amax : 0.f;
  if (j == 0) qscale[h] = amax / 127.0f;
  // dims 32j + 16i .. +15: box j/4, 16-byte chunk 2 (j % 4) + i of the row
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 a = v[4 * i + e];
      int h0, l0, h1, l1, h2, l2, h3, l3;
      split16(a.x * inv, h0, l0);
      split16(a.y * inv, h1, l1);
      split16(a.z * inv, h2, l2);
      split16(a.w * inv, h3, l3);
      hw[e] = pack4(h0, h1, h2, h3);
      lw[e] = pack4(l0, l1, l2, l3);
    }
    const uint32_t k = 16u * (2u * (j & 3) + i);
    uint8_t *box = qi + (j >> 2) * 4096;
    *reinterpret_cast<uint4 *>(box + sw128_byte(h, k)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4 *>(box + sw128_byte(16 + h, k)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  // rope dims 4j .. 4j + 3: bytes 8j .. 8j + 7 of head h's 128-byte row
  *reinterpret_cast<uint2 *>(qr + (h >> 3) * 1024 + (h & 7) * 128 + (((j >> 1) ^ (h & 7)) << 4) + 8 * (j & 1)) =
      make_uint2(pack2_bf16(r0.x, r0.y), pack2_bf16(r0.z, r0.w));
}

// Both phases at once.
__device__ __forceinline__ void load_query_unit(uint8_t *qi, uint8_t *qr, float *qscale, const float *q, int u) {
  QueryUnitLoads ld;
  query_unit_load(q, u, ld);
  query_unit_split(qi, qr, qscale, u, ld);
}

// 4 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

// 8 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// hi * 256 + lo of two int32 MMA sums (|hi| <= 512 * 127 * 127, so it fits).
__device__ __forceinline__ float join16(uint32_t hi, uint32_t lo) {
  return static_cast<float>(static_cast<int>(hi) * 256 + static_cast<int>(lo));
}

// Warp-wide maximum of 32-bit unsigned values (non-negative floats order like
// their bit patterns).
__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
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
    for (int i = 0; i < kSlots; ++i) { mbar_init(&B->full[i], 1); mbar_init(&B->empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B->s_full[i], 1);
      mbar_init(&B->s_empty[i], 4 * kWGs);  // every softmax warp
      mbar_init(&B->p_full[i], 4 * kWGs);
      mbar_init(&B->p_empty[i], 1);
      mbar_init(&B->o_full[i], 1);
      mbar_init(&B->o_empty[i], 4 * kWGs);
    }
    mbar_init(&B->q0_full, 8);                // warpgroups 0-1 split the first segment's query
    mbar_init(&B->q_full, 1);                 // the loader's expect-tx arrival (later segments)
    mbar_init(&B->q_empty, 1 + 4 * kWGs);     // the issuer's commit after the segment's last
                                              // scores, and every softmax warp once it has read sq
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
      uint32_t ri = 0;  // boxes issued
      bool ok = true;
      for (int si = seg_lo; si < seg_hi && ok; ++si) {
        const AttendSegment sg = p.segs[si];
        const long long row0 = sg.row0 + sg.tok_begin;
        const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
        for (int t = 0; t < nt && ok; ++t) {
          const int32_t y = static_cast<int32_t>(row0 + static_cast<long long>(kTileTok) * t);
          for (int b = 0; b < kBoxesPerTile; ++b, ++ri) {
            const uint32_t s = ri % kSlots;
            ok = mbar_wait(&B->empty[s], ((ri / kSlots) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY);
            if (!ok) break;
            uint8_t *dst = smem + OFF_RING + s * kBox;
            mbar_arrive_expect_tx(&B->full[s], kBox);
            if (b == 0)
              tma_load_2d(dst, &p.tm_rope, &B->full[s], 0, y);
            else
              tma_load_2d(dst, &p.tm_lat8, &B->full[s], 128 * (b - 1), y);
          }
        }
      }
      if (!ok) {
        // The most recent load issued into each slot must land before the CTA
        // exits (earlier ones completed before the slot was reissued).
        for (uint32_t s = 0; s < kSlots && s < ri; ++s) {
          const uint32_t last = s + kSlots * ((ri - 1 - s) / kSlots);
          drain_wait(&B->full[s], (last / kSlots) & 1, p.err);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_rope = idesc_f16(1, 1, 0, 0, 128, kHeads);  // bf16 rows x bf16 q_rope
      constexpr uint32_t idesc_s = idesc_s8(0, 0, 128, 32);                // int8 rows x q parts
      constexpr uint32_t idesc_pv = idesc_s8(1, 1, 128, 32);               // int8 rows^T x P' parts, both MN-major
      const uint32_t ring = s_base + OFF_RING, qi = s_base + OFF_QI, qr = s_base + OFF_QR;
      // scores of tile gg: rope (bf16) and the four int8 chunks
      auto issue_scores = [&](uint32_t gg, bool last_of_segment) -> bool {
        const uint32_t sb = gg & 1, r0 = kBoxesPerTile * gg;
        if (!mbar_wait(&B->s_empty[sb], ((gg >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_EMPTY) ||
            !mbar_wait(&B->full[r0 % kSlots], (r0 / kSlots) & 1, abort, p.err, ERR_TIMEOUT_FULL))
          return false;
        tc_fence_after();
        const uint32_t rope_box = ring + (r0 % kSlots) * kBox;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + kColR + 16 * sb, smem_desc(rope_box + kk * 32, 16, 1024, LAYOUT_SW128),
                     smem_desc(qr + kk * 32, 16, 1024, LAYOUT_SW128), idesc_rope, kk ? 1u : 0u);
        mma_commit(&B->empty[r0 % kSlots]);
        for (int c = 0; c < 4; ++c) {
          const uint32_t ri = r0 + 1 + c;
          if (!mbar_wait(&B->full[ri % kSlots], (ri / kSlots) & 1, abort, p.err, ERR_TIMEOUT_FULL)) return false;
          tc_fence_after();
          const uint32_t box = ring + (ri % kSlots) * kBox;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_s8_ss(tmem + kColS + 32 * sb, smem_desc(box + kk * 32, 16, 1024, LAYOUT_SW128),
                      smem_desc(qi + c * 4096 + kk * 32, 16, 1024, LAYOUT_SW128), idesc_s, (c | kk) ? 1u : 0u);
        }
        mma_commit(&B->s_full[sb]);
        // the query operands are free once the segment's last scores are done
        if (last_of_segment) mma_commit(&B->q_empty);
        return true;
      };
      // P'.V of tile gg into its own int32 buffer (folded by the softmax threads)
      auto issue_pv = [&](uint32_t gg) -> bool {
        const uint32_t pb = gg & 1;
        if (!mbar_wait(&B->p_full[pb], (gg >> 1) & 1, abort, p.err, ERR_TIMEOUT_FULL) ||
            !mbar_wait(&B->o_empty[pb], ((gg >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_FULL))
          return false;
        tc_fence_after();
        const uint32_t pa = s_base + OFF_P + pb * kPBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t ri = kBoxesPerTile * gg + 1 + c;
          const uint32_t box = ring + (ri % kSlots) * kBox;
          // A = the chunk read MN-major: 128 dims (one 128-byte span) x 32 rows
          // per MMA (four 8-row swizzle atoms, 1 KB apart); B = P' MN-major,
          // 32 bytes per KV row, 8-row atoms of 256 bytes
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_s8_ss(tmem + kColO + 128 * pb + 32 * c, smem_desc(box + kk * 4096, kBox, 1024, LAYOUT_SW128),
                      smem_desc(pa + kk * 1024, kPBytes, 256, LAYOUT_SW32), idesc_pv, kk ? 1u : 0u);
          mma_commit(&B->empty[ri % kSlots]);
        }
        mma_commit(&B->p_empty[pb]);
        mma_commit(&B->o_full[pb]);
        return true;
      };
      uint32_t g = 0;
      int seg_i = 0;
      bool ok = true;
      AttendSegment nx = p.segs[seg_lo];  // descriptors are read one segment ahead
      for (int si = seg_lo; si < seg_hi && ok; ++si, ++seg_i) {
        const AttendSegment sg = nx;
        if (si + 1 < seg_hi) nx = p.segs[si + 1];
        const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
        ok = (seg_i == 0 ? mbar_wait(&B->q0_full, 0, abort, p.err, ERR_TIMEOUT_FULL)
                         : mbar_wait(&B->q_full, (seg_i - 1) & 1, abort, p.err, ERR_TIMEOUT_FULL)) &&
             issue_scores(g, nt == 1);
        for (int t = 0; t < nt && ok; ++t, ++g) {
          // the next tile's scores go ahead of this tile's P.V (same segment:
          // the next segment's query lands only after this one's scores end)
          if (t + 1 < nt) ok = issue_scores(g + 1, t + 2 == nt);
          if (ok) ok = issue_pv(g);
        }
      }
      // All issued tensor-core work must finish before TMEM is released.
      mma_commit(&B->drain);
      drain_wait(&B->drain, 0, p.err);
    }
  } else if (warp < kLoaderWarp) {
    // ------------------------------------------------------------ softmax, fold, epilogue
    const int wg = (warp - 2) >> 2;  // warpgroup: heads kHPW wg .. + kHPW - 1
    const int w = warp & 3;          // TMEM subpartition = rows / dims 32 w .. 32 w + 31
    const int tt = 32 * w + lane;
    const int hb = kHPW * wg;
    const uint32_t bid = 1 + wg;     // this warpgroup's named barrier
    const uint32_t lane_base = static_cast<uint32_t>(32 * w) << 16;
    uint32_t g = 0;
    int seg_i = 0;
    // The next segment's descriptor is read at the start of this one, and the
    // row scales of its first tile during this one's last tile, so a segment
    // boundary waits on no dependent global load.
    AttendSegment nx = p.segs[seg_lo];
    float rs_nx = nx.tok_begin + tt < nx.tok_end ? p.latent_scale[nx.row0 + nx.tok_begin + tt] : 0.f;
    for (int si = seg_lo; si < seg_hi; ++si, ++seg_i) {
      const AttendSegment sg = nx;
      if (si + 1 < seg_hi) nx = p.segs[si + 1];
      const long long srow0 = sg.row0;
      const int nt = (sg.tok_end - sg.tok_begin + kTileTok - 1) / kTileTok;
      float rs_next = rs_nx;
      if (seg_i == 0) {
        // the first segment's query is split here (no wait for the prep kernel)
        if (wg < 2) {
          uint8_t *qi = smem + OFF_QI;
          if (p.q_after_wait) pdl_wait();
          load_query_unit(qi, qi + kQiBytes, reinterpret_cast<float *>(smem + OFF_QS),
                          p.q + static_cast<size_t>(sg.seq) * kHeads * kRow, 128 * wg + tt);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&B->q0_full);
        }
        named_bar_sync(1 + kWGs, 128 * kWGs);
      } else {
        // later segments: sq arrives with the query image
        if (named_bar_or(bid, 128, !mbar_wait(&B->q_full, (seg_i - 1) & 1, abort, p.err, ERR_TIMEOUT_FULL))) break;
      }
      float sq[kHPW];  // sq / 256: the scores are read as S_hi * 256 + S_lo
      const float *qs = reinterpret_cast<const float *>(smem + OFF_QS);
#pragma unroll
      for (int i = 0; i < kHPW; ++i) sq[i] = qs[hb + i] * 0.00390625f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&B->q_empty);
      float m_ref[kHPW], l_part[kHPW], sp_prev[kHPW], acc[4][kHPW];
#pragma unroll
      for (int i = 0; i < kHPW; ++i) {
        m_ref[i] = -INFINITY;
        l_part[i] = 0.f;
        sp_prev[i] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[c][i] = 0.f;
      }
      // acc = (acc + sp * (O_hi * 256 + O_lo)) * alpha for tile gg (sp passed
      // as the P' step / 256; alpha applied when resc)
      auto fold = [&](uint32_t gg, const float (&sp)[kHPW], bool resc, const float (&alpha)[kHPW]) -> bool {
        const uint32_t ob = gg & 1;
        const bool bad = !mbar_wait(&B->o_full[ob], (gg >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (named_bar_or(bid, 128, bad)) return false;
        tc_fence_after();
        uint32_t oh[4][kHPW], ol[4][kHPW];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t col = tmem + kColO + 128 * ob + 32 * c + hb + lane_base;
          tmem_ld4(col, oh[c]);
          tmem_ld4(col + 16, ol[c]);
        }
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < kHPW; ++i) acc[c][i] = fmaf(sp[i], join16(oh[c][i], ol[c][i]), acc[c][i]);
          if (resc)
#pragma unroll
            for (int i = 0; i < kHPW; ++i) acc[c][i] *= alpha[i];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->o_empty[ob]);
        return true;
      };
      bool bad = false;
      for (int t = 0; t < nt; ++t, ++g) {
        const int tok = sg.tok_begin + kTileTok * t + tt;
        const bool valid = tok < sg.tok_end;
        const float rs = rs_next;
        if (t + 1 < nt)
          rs_next = tok + kTileTok < sg.tok_end ? p.latent_scale[srow0 + tok + kTileTok] : 0.f;
        else if (si + 1 < seg_hi)
          rs_nx = nx.tok_begin + tt < nx.tok_end ? p.latent_scale[nx.row0 + nx.tok_begin + tt] : 0.f;
        const uint32_t sb = g & 1;
        bad = !mbar_wait(&B->s_full[sb], (g >> 1) & 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (named_bar_or(bid, 128, bad)) { bad = true; break; }
        tc_fence_after();
        uint32_t sh[kHPW], sl[kHPW], srp[kHPW];
        tmem_ld4(tmem + kColS + 32 * sb + hb + lane_base, sh);
        tmem_ld4(tmem + kColS + 32 * sb + 16 + hb + lane_base, sl);
        tmem_ld4(tmem + kColR + 16 * sb + hb + lane_base, srp);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->s_empty[sb]);
        float s[kHPW];
        bool need = false;
#pragma unroll
        for (int i = 0; i < kHPW; ++i) {
          s[i] = valid ? fmaf(rs * sq[i], join16(sh[i], sl[i]), __uint_as_float(srp[i])) * p.scale_log2 : -INFINITY;
          need |= s[i] > m_ref[i] + 8.0f;
        }
        // lazy rescale: the running maximum moves only by more than 2^8
        bool resc = false;
        float alpha[kHPW];
#pragma unroll
        for (int i = 0; i < kHPW; ++i) alpha[i] = 1.f;
        if (named_bar_or(bid, 128, need)) {
          float mx[kHPW];
#pragma unroll
          for (int i = 0; i < kHPW; ++i) mx[i] = s[i];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int i = 0; i < kHPW; ++i) mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], off));
          if (lane == 0)
#pragma unroll
            for (int i = 0; i < kHPW; ++i) B->red[wg][w][i] = mx[i];
          named_bar_sync(bid, 128);
#pragma unroll
          for (int i = 0; i < kHPW; ++i) {
            const float tm = fmaxf(fmaxf(B->red[wg][0][i], B->red[wg][1][i]), fmaxf(B->red[wg][2][i], B->red[wg][3][i]));
            const float mn = fmaxf(m_ref[i], tm);
            alpha[i] = (m_ref[i] == -INFINITY) ? 0.f : exp2f(m_ref[i] - mn);
            m_ref[i] = mn;
            l_part[i] *= alpha[i];
          }
          named_bar_sync(bid, 128);
          resc = true;
        }
        // P'_j = p_j * scale_j, split per head against the tile's max |P'|
        float pq[kHPW];
#pragma unroll
        for (int i = 0; i < kHPW; ++i) {
          const float pr = exp2f(s[i] - m_ref[i]);
          l_part[i] += pr;
          pq[i] = pr * rs;
        }
#pragma unroll
        for (int i = 0; i < kHPW; ++i) {
          const uint32_t m = warp_max_u32(__float_as_uint(fabsf(pq[i])));
          if (lane == 0) B->pmax[g & 1][wg][w][i] = __uint_as_float(m);
        }
        named_bar_sync(bid, 128);
        float sp[kHPW];
        uint32_t hw = 0u, lw = 0u;
#pragma unroll
        for (int i = 0; i < kHPW; ++i) {
          const float m = fmaxf(fmaxf(B->pmax[g & 1][wg][0][i], B->pmax[g & 1][wg][1][i]),
                                fmaxf(B->pmax[g & 1][wg][2][i], B->pmax[g & 1][wg][3][i]));
          sp[i] = m * (1.0f / (127.0f * 256.0f));
          int ph, pl;
          split16(m > 0.f ? pq[i] * (127.0f * __frcp_rn(m)) : 0.f, ph, pl);
          hw |= (static_cast<uint32_t>(ph) & 0xFFu) << (8 * i);
          lw |= (static_cast<uint32_t>(pl) & 0xFFu) << (8 * i);
        }
        bad = !mbar_wait(&B->p_empty[sb], ((g >> 1) & 1) ^ 1, abort, p.err, ERR_TIMEOUT_MMA);
        if (named_bar_or(bid, 128, bad)) { bad = true; break; }
        {
          // P' parts as the MN-major B operand: KV row tt holds 32 bytes, hi of
          // heads 0-15 then lo of heads 0-15, with the 32-byte swizzle (the
          // 16-byte halves swap in rows with bit 2 set)
          uint8_t *row = smem + OFF_P + sb * kPBytes + (tt >> 3) * 256 + (tt & 7) * 32;
          const uint32_t swz = ((tt >> 2) & 1) << 4;
          *reinterpret_cast<uint32_t *>(row + (hb ^ swz)) = hw;
          *reinterpret_cast<uint32_t *>(row + ((16 + hb) ^ swz)) = lw;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B->p_full[sb]);
        // fold the previous tile's P'.V (its frame is rescaled with this tile's alpha)
        if (t > 0 && !fold(g - 1, sp_prev, resc, alpha)) { bad = true; break; }
#pragma unroll
        for (int i = 0; i < kHPW; ++i) sp_prev[i] = sp[i];
      }
      if (bad) break;
      // ---- epilogue: last tile's P'.V, then O / l and lse
      {
        float one[kHPW];
#pragma unroll
        for (int i = 0; i < kHPW; ++i) one[i] = 1.f;
        if (!fold(g - 1, sp_prev, false, one)) break;
      }
      float lt[kHPW];
#pragma unroll
      for (int i = 0; i < kHPW; ++i) {
        float l = l_part[i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        lt[i] = l;
      }
      if (lane == 0)
#pragma unroll
        for (int i = 0; i < kHPW; ++i) B->red[wg][w][i] = lt[i];
      named_bar_sync(bid, 128);
#pragma unroll
      for (int i = 0; i < kHPW; ++i) lt[i] = (B->red[wg][0][i] + B->red[wg][1][i]) + (B->red[wg][2][i] + B->red[wg][3][i]);
      named_bar_sync(bid, 128);
      float inv[kHPW];  // one division per head, not per element
#pragma unroll
      for (int i = 0; i < kHPW; ++i) inv[i] = 1.0f / lt[i];
      float *dst = (sg.slot < 0) ? p.out + static_cast<size_t>(sg.seq) * kHeads * kLatent
                                 : p.part_o + static_cast<size_t>(sg.slot) * kHeads * kLatent;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int d = 128 * c + tt;
#pragma unroll
        for (int i = 0; i < kHPW; ++i) dst[(hb + i) * kLatent + d] = acc[c][i] * inv[i];
      }
      if (w == 0 && lane < kHPW) {
        float m = 0.f, l = 1.f;
#pragma unroll
        for (int i = 0; i < kHPW; ++i)
          if (i == lane) { m = m_ref[i]; l = lt[i]; }
        const float lse = (m + log2f(l)) * 0.69314718055994531f;
        float *ldst = (sg.slot < 0) ? p.lse : p.part_lse;
        const int row = (sg.slot < 0) ? sg.seq : sg.slot;
        if (ldst) ldst[row * kHeads + hb + lane] = lse;
      }
    }
  } else {
    // ------------------------------------------------------------ query loader
    // From the CTA's second segment on: one bulk copy of the segment's query
    // image (prepared by qprep_q8_kernel, this grid's programmatic predecessor,
    // launched when some CTA has more than one segment) once the previous
    // segment's query is no longer read.  The first segment's query is split
    // by the softmax warps, so no CTA waits for the prep kernel at its start.
    if (lane == 0) {
      uint32_t issued = 0;
      bool ok = true;
      for (int si = seg_lo + 1, seg_i = 1; si < seg_hi; ++si, ++seg_i) {
        const int seq = p.segs[si].seq;
        ok = mbar_wait(&B->q_empty, (seg_i - 1) & 1, abort, p.err, ERR_TIMEOUT_EMPTY);
        if (!ok) break;
        if (seg_i == 1) asm volatile("griddepcontrol.wait;" ::: "memory");
        mbar_arrive_expect_tx(&B->q_full, kQImgQ8Bytes);
        bulk_load(smem + OFF_QI, p.qimg + static_cast<size_t>(seq) * kQImgStride, kQImgQ8Bytes, &B->q_full);
        ++issued;
      }
      // the last copy must land before the CTA exits
      if (!ok && issued > 0) drain_wait(&B->q_full, (issued - 1) & 1, p.err);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// The query images of a launch: block b writes sequence b's q_lat parts, q_rope
// and sq in the shared-memory layout of the kernel above (256 threads, one unit
// each).  The attend grid is its programmatic dependent and may start as soon
// as this grid is past its own wait; only the attend's loader waits for this
// grid.
__global__ void __launch_bounds__(256) qprep_q8_kernel(const float *q, uint8_t *img) {
  // launched as a programmatic dependent of the query's producer: the attend
  // (this grid's dependent) is released only after that producer is done, so
  // the query rows it reads before its own wait are complete
  pdl_wait();
  pdl_trigger();
  uint8_t *base = img + static_cast<size_t>(blockIdx.x) * kQImgStride;
  load_query_unit(base, base + kQiBytes, reinterpret_cast<float *>(base + kQiBytes + kQrBytes),
                  q + static_cast<size_t>(blockIdx.x) * kHeads * kRow, threadIdx.x);
}

// The query prep for `batch` sequences (only when some CTA of the plan has
// more than one segment: `qprep`), then the attend grid.
cudaError_t launch_attend_q8(const AttendParams &p, int grid, int batch, bool qprep, cudaStream_t stream) {
  static std::atomic<unsigned long long> opted{0};
  cudaError_t e = smem_opt_in(reinterpret_cast<const void *>(mla_attend_q8_kernel), kSmemBytes, opted);
  if (e != cudaSuccess) return e;
  if (qprep) {
    ProfScope ps("qprep_q8", stream);
    e = launch_dependent(qprep_q8_kernel, dim3(batch), dim3(256), 0, stream, p.q, const_cast<uint8_t *>(p.qimg));
    if (e != cudaSuccess) return e;
  }
  ProfScope ps("mla_attend_q8", stream);
  // A programmatic dependent of the prep kernel (its loader waits for the
  // images; the prep releases it after its own wait, so every input the kernel
  // reads directly is complete by then), or of the query's producer when
  // q_after_wait is set; otherwise an ordinary launch.
  if (qprep || p.q_after_wait)
    return launch_pdl(reinterpret_cast<const void *>(mla_attend_q8_kernel), grid, kThreads, kSmemBytes, stream, p);
  mla_attend_q8_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace kvl
