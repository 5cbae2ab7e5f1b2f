// attend_common.cuh -- shared definitions of the absorbed-MLA decode attend
// kernels (bf16 latent state and row-wise Q8 latent state).
//
// The attend core restated here is the inner part of the reference decode
// (src/mla_compressed_state.c:132-148, src/mla_compressed_q8_state.c:216-238):
// for every head h and cached row j
//     s_j   = (q_lat_h . latent_j + q_rope_h . rope_j) * scale
//     mix_h = sum_j softmax(s)_j * latent_j
// with all heads sharing one 576-wide cached row (512 latent + 64 rope).
//
// Work decomposition ("stream-K" over KV tiles): the KV rows of every sequence
// are cut into tiles of 64 rows; the concatenated tile list of the whole batch
// is split into equal contiguous ranges, one per CTA.  A CTA's range is a list
// of segments (one sequence each).  A segment that covers a whole sequence
// writes the normalised output directly; a piece of a split sequence writes a
// partial (o, lse) that the merge kernel combines.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace kvl {

constexpr int kHeads = 16;       // tcgen05 N (heads share one latent row)
constexpr int kLatent = 512;     // kv_lora_rank
constexpr int kRope = 64;        // qk_rope_dim
constexpr int kRow = kLatent + kRope;
constexpr int kTileTok = 64;     // KV rows per tile (tcgen05 M of the score MMA)

struct AttendSegment {
  int seq;        // batch index
  int tok_begin;  // first KV row of the segment (tile aligned within the sequence)
  int tok_end;    // one past the last KV row
  int slot;       // partial slot, or -1 when the segment is the whole sequence
};

struct AttendParams {
  CUtensorMap tm_kv;         // bf16 layout: [rows][576] (latent | rope)
  CUtensorMap tm_rope;       // q8 layout: rope bf16 [rows][64]
  CUtensorMap tm_lat8;       // q8 layout: latent int8 [rows][512]
  const float *latent_scale; // q8 layout: [rows]
  const float *q;            // [B][16][576] fp32 absorbed query (q_lat | q_rope)
  float *out;                // [B][16][512] fp32 normalised mix
  float *lse;                // [B][16] natural-log normaliser (may be null)
  float *part_o;             // [P][16][512]
  float *part_lse;           // [P][16]
  const AttendSegment *segs;
  const int *cta_seg;        // [grid + 1] segment ranges per CTA
  const long long *seq_row0; // [B] first pool row of each sequence
  long long rows;            // rows in the pool
  float scale_log2;          // softmax scale * log2(e)
  uint32_t *err;             // error word (bit-or of kvl::ERR_*)
  float *dbg_s;              // optional: raw scores of the first tiles, [tiles][64][16]
  int dbg_tiles;
};

}  // namespace kvl
