// flash_prefill.cuh -- causal MLA prefill attention (see flash_prefill.cu).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kvl {

struct FlashParams {
  CUtensorMap tm_q;    // q [S][16][192] bf16 (nope 128 | rotated rope 64), 3-D box {64, 1, 128}
  CUtensorMap tm_kv;   // kv [S][16][256] bf16 (k_nope 128 | v 128), 3-D box {64, 1, 128}
  CUtensorMap tm_kr;   // rotated k_rope: columns [kr_col, kr_col + 64) of a [S][ld] bf16 pool, box {64, 128}
  int kr_col;
  int S;               // keys [0, S); queries [128 * q_tile0, S)
  int q_tile0;
  int lo_t0, lo_t1;    // optional second query range: tiles [lo_t0, lo_t1), lo_t1 <= q_tile0
                       // (0, 0: none); each of its tiles attends keys up to its own end
  int q_compact;       // 0: query tile t is rows [128 t, 128 t + 128) of tm_q and out;
                       // 1: tm_q and out hold only the queried tiles, [lo_t0, lo_t1) then [q_tile0, nq)
  float scale_log2;    // softmax scale * log2(e)
  __nv_bfloat16 *out;  // [S][16][128] bf16 (q_compact: [queried rows][16][128])
  uint32_t *err;
  // Key-range pieces, for launches with fewer (head, query tile) items than
  // SMs (the context-parallel prefill): kpiece > 0 cuts every item into pieces
  // of at most kpiece key tiles; a cut item's pieces write their O (normalised
  // by their own sum) and the log2 of that sum to part_o / part_lse at their
  // unit index, and a second kernel combines them.  kpiece < 0: the launcher
  // picks kpiece (or 0) from the items' key counts.  0: no cut.
  int kpiece;
  float *part_o;       // [kFlashMaxUnits][128 rows][128] fp32
  float *part_lse;     // [kFlashMaxUnits][128 rows]
  // zz_world > 0: tm_kr's rows are the context-parallel all-gather (key tile j
  // at zigzag_tile(j, zz_world, zz_c128), gemm.cuh); 0: prompt order.
  int zz_world, zz_c128;
};

// Work units (pieces) a launch may hold when items are cut.
constexpr int kFlashMaxUnits = 296;

// dep: launched as a programmatic dependent of the previous kernel on the
// stream (the kernel orders all its global accesses after griddepcontrol.wait)
cudaError_t launch_flash_prefill(const FlashParams &p, int sms, cudaStream_t stream, bool dep = false);

bool make_tmap_3d(CUtensorMap *m, const void *base, CUtensorMapDataType dt, const uint64_t dims[3],
                  const uint64_t strides_bytes[2], const uint32_t box[3], CUtensorMapSwizzle sw);

}  // namespace kvl
