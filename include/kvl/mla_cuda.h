/*
 * kvl/mla_cuda.h -- B200 entry points of libkvl_mla_cuda beyond the
 * reference's state API.
 *
 * The reference exposes the MLA hot path only through the hidden-state calls
 * of kvl/mla_compressed_state.h, kvl/mla_compressed_q8_state.h and
 * kvl_mla_prefill_bf16.  The calls below expose the same computation on device
 * memory, batched, for callers that keep their states on the GPU (the batched
 * and long-context decode configurations, multi-GPU sharding, benchmarks):
 *
 *   attend core  (src/mla_compressed_state.c:132-148 and
 *                 src/mla_compressed_q8_state.c:216-238): absorbed query
 *                 [B][16][576] fp32 against cached rows -> mix [B][16][512]
 *   merge        combine (o, lse) partials of one sequence split across GPUs
 *   Q8 helpers   the row quantiser (src/mla_compressed_q8_state.c:34-55), the
 *                dequantiser (:57-61) and bf16 RNE (:9-16), bit-exact
 *
 * Pointers named d_* are device pointers; `stream` is a cudaStream_t (NULL =
 * the legacy default stream).  Every call returns 0, or -1 with a message
 * available from kvl_mla_cuda_last_error().  Set KVL_CUDA_VERBOSE=1 to also
 * print failures on stderr.
 */
#ifndef KVL_MLA_CUDA_H
#define KVL_MLA_CUDA_H

#include <stddef.h>
#include <stdint.h>
#include "kvl/ops.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Message of the last failure on this thread ("" when none). */
const char *kvl_mla_cuda_last_error(void);

/* Device-side weight cache keyed by host pointer (enable = 1) or per-call
 * upload (0).  The cache is only correct while the host weight buffers stay
 * allocated and unchanged, which holds in the reference runtime when its trunk
 * cache covers every tensor (KVL_TRUNK_CACHE_MIB >= 1706); that setting, or
 * KVL_CUDA_WEIGHT_CACHE=1, enables it at start-up.  Returns the previous mode. */
int kvl_mla_cuda_weight_cache(int enable);

/* Per-kernel timing.  Enabled (1), every kernel the library launches is
 * bracketed by CUDA events on its launching stream; enabling clears the
 * totals.  Returns the previous mode. */
int kvl_mla_cuda_profile(int enable);
/* Waits for the recorded launches and writes one "kernel,total_ms,launches"
 * line per kernel into buf (NUL-terminated).  Returns the number of kernels,
 * or -1 if cap is too small. */
int kvl_mla_cuda_profile_read(char *buf, size_t cap);

/* Device bytes held by a state created by kvl_mla_compressed_state_init /
 * kvl_mla_compressed_q8_state_init (0 for an unknown state). */
size_t kvl_mla_cuda_state_device_bytes(const void *state);

/* ------------------------------------------------------------------ attend */

/* Work plan of one batch: cached lengths and the first pool row of every
 * sequence (host arrays), split into equal contiguous ranges of 128-row tiles,
 * one per CTA (max_ctas = 0: one per SM).  Owns the partial-output workspace,
 * sized for num_heads x kv_lora_rank outputs per piece.  Created on, and used
 * with, the current CUDA device. */
typedef struct KvlMlaAttendPlan KvlMlaAttendPlan;

int kvl_mla_attend_plan_create(KvlMlaAttendPlan **plan, int batch, const int *seq_len,
                               const int64_t *seq_row0, int num_heads, int kv_lora_rank,
                               int max_ctas);
void kvl_mla_attend_plan_destroy(KvlMlaAttendPlan *plan);
/* ctas: grid size; partials: split-sequence pieces; segments: total pieces. */
int kvl_mla_attend_plan_info(const KvlMlaAttendPlan *plan, int *ctas, int *partials,
                             int *segments);

/* bf16 pool d_kv [rows][kv_lora_rank + rope_dim] (latent | rope).
 * d_q [B][num_heads][kv_lora_rank + rope_dim] fp32 absorbed query,
 * d_out [B][num_heads][kv_lora_rank] fp32, d_lse [B][num_heads] (natural log;
 * may be NULL).  Production shape (16, 512, 64) runs the tcgen05 kernel; other
 * shapes run a CUDA-core kernel.  d_q and d_kv must be 16-byte aligned (the
 * call returns -1 before launching anything otherwise). */
int kvl_mla_attend_bf16(const KvlMlaAttendPlan *plan, float *d_out, float *d_lse,
                        const float *d_q, const uint16_t *d_kv, int64_t rows, int num_heads,
                        int kv_lora_rank, int rope_dim, float softmax_scale, void *stream);

/* Q8 pool (reference layout): d_latent_q8 [rows][R] int8, d_latent_scale
 * [rows] fp32, d_rope_bf16 [rows][DR] bf16, all 16-byte aligned, as d_q.  The
 * production shape runs on the int8 tensor cores: the query and the softmax
 * weights times the row scales enter as two int8 parts each (about 16 bits),
 * against the stored int8 rows with exact int32 sums. */
int kvl_mla_attend_q8(const KvlMlaAttendPlan *plan, float *d_out, float *d_lse,
                      const float *d_q, const int8_t *d_latent_q8, const float *d_latent_scale,
                      const uint16_t *d_rope_bf16, int64_t rows, int num_heads, int kv_lora_rank,
                      int rope_dim, float softmax_scale, void *stream);

/* Single-sequence bf16 attend that allocates nothing.  This call has no
 * counterpart in the reference runtime.  It serves callers that cannot
 * allocate device memory while they decode: a runtime that reserves its whole
 * device-memory budget up front, or a decode loop that must not stall on
 * cudaMalloc (which can synchronise the device and fails once memory is
 * fragmented).  It computes what kvl_mla_attend_bf16 computes for one sequence
 * of seq_len rows starting at pool row seq_row0, split over `splits` KV ranges
 * (0 = one per SM), with its plan and partial outputs in a fixed 4.9 MB device
 * array that the library reserves on every GPU it is loaded on until the
 * process exits.  splits above 148 are rejected; only the (16, 512, 64) shape
 * is accepted.  The first call on a device looks up that array's address.  All
 * calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  The call is synchronous: it returns after `stream`
 * has finished and the result is in d_out, so it cannot be captured into a
 * CUDA graph. */
int kvl_mla_attend_bf16_noalloc(float *d_out, float *d_lse, const float *d_q, const uint16_t *d_kv,
                                int64_t rows, int seq_len, int64_t seq_row0, int num_heads,
                                int kv_lora_rank, int rope_dim, int splits, float softmax_scale,
                                void *stream);

/* Waits for `stream` and returns -1 if a kernel of the plan's last launch
 * reported a device-side error (a bounded wait that ran out); clears it. */
int kvl_mla_attend_check(const KvlMlaAttendPlan *plan, void *stream);

/* Combines `parts` partial results per sequence, stored part-major:
 * d_part_o [parts][batch][num_heads][R], d_part_lse [parts][batch][num_heads]
 * (e.g. gathered from the GPUs of a split-KV decode) into d_out / d_lse. */
int kvl_mla_merge_partials(float *d_out, float *d_lse, const float *d_part_o,
                           const float *d_part_lse, int parts, int batch, int num_heads,
                           int kv_lora_rank, void *stream);

/* Same combine over packed records, one per part: d_parts[p] is
 * [batch][num_heads][R] outputs followed by [batch][num_heads] lse values
 * (record stride batch * num_heads * (R + 1) floats), e.g. what one NCCL
 * all-gather of each GPU's (o, lse) buffer produces. */
int kvl_mla_merge_packed(float *d_out, float *d_lse, const float *d_parts, int parts, int batch,
                         int num_heads, int kv_lora_rank, void *stream);

/* ------------------------------------------------------------------ split-KV across GPUs */

/* The combine of a split-KV decode across the GPUs of one node in one launch
 * (in place of an all-gather plus kvl_mla_merge_packed): each GPU stores its
 * (o, lse) values into every other GPU's exchange buffer over NVLink as tagged
 * 64-bit words (call number and value in one store) and merges the world
 * records once every word it needs carries the call's tag.  One process per GPU:
 *   create (allocates this GPU's buffer; writes its CUDA IPC handle, of
 *   kvl_mla_peer_handle_bytes() bytes, to handle_out) -> the caller gathers the
 *   world handles in rank order (any host collective) -> connect -> per step
 *   kvl_mla_merge_exchange (packed record d_record = [batch][num_heads][R] then
 *   lse [batch][num_heads]) or kvl_mla_attend_bf16_exchange on every rank, in
 *   the same order -> destroy.
 * batch * num_heads <= 256, world <= 8, kv_lora_rank a multiple of 128; d_out
 * and d_record 16-byte aligned.  Waits are bounded (2 s);
 * kvl_mla_peer_group_check reports a peer whose values did not arrive.  After
 * such a timeout the ranks' call counts no longer agree (the rank that timed
 * out went on without the peer's values), so the group cannot be used again:
 * destroy it on every rank and create and connect a new one. */
typedef struct KvlMlaPeerGroup KvlMlaPeerGroup;
size_t kvl_mla_peer_handle_bytes(void);
int kvl_mla_peer_group_create(KvlMlaPeerGroup **group, int rank, int world, int batch, int num_heads,
                              int kv_lora_rank, void *handle_out);
int kvl_mla_peer_group_connect(KvlMlaPeerGroup *group, const void *handles);
int kvl_mla_merge_exchange(KvlMlaPeerGroup *group, float *d_out, float *d_lse, const float *d_record,
                           void *stream);
int kvl_mla_peer_group_check(KvlMlaPeerGroup *group, void *stream);
void kvl_mla_peer_group_destroy(KvlMlaPeerGroup *group);
/* The attend of this rank's KV range (plan of `batch` sequences, 16 heads,
 * R = 512, rope 64) and the cross-GPU combine in two launches: the attend leaves
 * split sequences as partials, and one kernel per (sequence, head, 128-wide
 * slice) combines them locally (as kvl_mla_attend_bf16 would), exchanges the
 * slice with every peer and merges the world slices into d_out [batch][16][512]
 * and d_lse [batch][16] (NULL: not written).  Replaces kvl_mla_attend_bf16 +
 * kvl_mla_merge_exchange; d_out 16-byte aligned; the plan's batch must equal the
 * group's. */
int kvl_mla_attend_bf16_exchange(const KvlMlaAttendPlan *plan, KvlMlaPeerGroup *group, float *d_out,
                                 float *d_lse, const float *d_q, const uint16_t *d_kv, int64_t rows,
                                 float softmax_scale, void *stream);

/* ------------------------------------------------------------------ batched decode step */

/* Device-resident layer weights (bf16, same shapes as KvlMlaBF16). */
typedef struct {
    const uint16_t *q_proj;
    const uint16_t *kv_a_proj;
    const uint16_t *kv_a_norm;
    const uint16_t *kv_b_proj;
    const uint16_t *o_proj;
} KvlMlaDeviceWeights;

/* Per-call scratch of kvl_mla_decode_step_bf16 for `batch` tokens. */
size_t kvl_mla_decode_step_workspace_bytes(const KvlMlaConfig *cfg, int batch);

/* One absorbed decode step for `batch` sequences of a bf16 pool, all on the
 * device: projections, append of each token's row at d_row[b] (RoPE position
 * d_pos[b]), attend over the plan's ranges (which must already include the
 * appended rows), V up-projection and o_proj.  d_x/d_out [batch][H] fp32.
 * Batches of 16 or more with 16-byte aligned weights, d_out and workspace run
 * the projections as tensor-core GEMMs on bf16-rounded activations; smaller
 * batches use per-token matvecs.  A device-side error of any of the step's
 * kernels is reported by kvl_mla_attend_check(plan, stream). */
int kvl_mla_decode_step_bf16(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w,
                             const KvlMlaAttendPlan *plan, float *d_out, const float *d_x,
                             uint16_t *d_kv, int64_t rows, const int64_t *d_row,
                             const int *d_pos, int batch, void *d_workspace, void *stream);

/* The same step over a Q8 pool in the reference layout (d_latent_q8 [rows][R]
 * int8, d_latent_scale [rows] fp32, d_rope_bf16 [rows][DR] bf16; the layout of
 * KvlMlaCompressedQ8State): each token's new row goes through the reference's
 * row quantiser (src/mla_compressed_q8_state.c:34-55, 111-127) and the attend
 * runs the int8 tensor-core kernel of kvl_mla_attend_q8.  Replaces one
 * kvl_mla_decode_compressed_q8_bf16 call (src/mla_compressed_q8_state.c:161-255)
 * per sequence.  Workspace as kvl_mla_decode_step_workspace_bytes. */
int kvl_mla_decode_step_q8(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w,
                           const KvlMlaAttendPlan *plan, float *d_out, const float *d_x,
                           int8_t *d_latent_q8, float *d_latent_scale, uint16_t *d_rope_bf16,
                           int64_t rows, const int64_t *d_row, const int *d_pos, int batch,
                           void *d_workspace, void *stream);

/* ------------------------------------------------------------------ prefill on device */

/* Scratch bytes kvl_mla_prefill_dev needs for seq_len tokens. */
size_t kvl_mla_prefill_workspace_bytes(const KvlMlaConfig *cfg, int seq_len);

/* Causal MLA prefill of one sequence entirely on the device (the computation
 * of kvl_mla_prefill_bf16): d_x [seq_len][H] bf16 token activations ->
 * d_out [seq_len][H] fp32.  Asynchronous on `stream`.  d_workspace must be
 * 256-byte aligned; d_x, d_out and the weights 16-byte aligned. */
int kvl_mla_prefill_dev(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, float *d_out,
                        const uint16_t *d_x, int seq_len, void *d_workspace, size_t workspace_bytes,
                        void *stream);

/* Context-parallel causal prefill of one seq_len-token prompt over `world`
 * GPUs, one process per GPU (the computation of kvl_mla_prefill_dev, split by
 * query rows).  The prompt is cut into 2 * world chunks of c = seq_len /
 * (2 * world) rows (c a multiple of 128); rank r owns chunks r and
 * 2 * world - 1 - r, so every rank has the same causal attention work.  Two
 * calls, with one all-gather of the compressed rows between them:
 *   kvl_mla_prefill_cp_begin: kv_a projection, RMSNorm and RoPE of the rank's
 *     rows (the per-token append of src/mla_prefill_streaming.c:131-138) into
 *     d_send [2c][576] bf16 (early chunk, then late chunk), and q_proj of those
 *     rows into the workspace;
 *   the caller all-gathers every rank's d_send into d_recv [world][2c][576] in
 *     rank order (one all-gather of 2c * 1152 bytes per rank, e.g. NCCL);
 *   kvl_mla_prefill_cp_end: places the gathered rows in prompt order, expands
 *     K/V with kv_b for the keys its chunks see, runs the causal attention of
 *     its queries (both chunks in one launch) and o_proj into d_out.
 * A rank holds only its own rows: d_x [2c][H] bf16 is the rank's tokens (chunk
 * rank, then chunk 2 * world - 1 - rank) and d_out [2c][H] fp32 receives their
 * outputs in the same order.  Both calls take the same workspace of
 * kvl_mla_prefill_workspace_bytes(cfg, seq_len) bytes (256-byte aligned), which
 * must not be reused between them.  Production head shape only. */
int kvl_mla_prefill_cp_begin(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, const uint16_t *d_x,
                             int seq_len, int rank, int world, uint16_t *d_send, void *d_workspace,
                             size_t workspace_bytes, void *stream);
int kvl_mla_prefill_cp_end(const KvlMlaConfig *cfg, const KvlMlaDeviceWeights *w, float *d_out, int seq_len,
                           int rank, int world, const uint16_t *d_recv, void *d_workspace,
                           size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------ Q8 helpers */
int kvl_mla_q8_quantize_rows(int8_t *d_q, float *d_scale, const float *d_x, int rows, int R,
                             void *stream);
int kvl_mla_q8_dequant(float *d_out, const int8_t *d_q, const float *d_scale, int64_t rows, int R,
                       void *stream);
int kvl_mla_bf16_rne(uint16_t *d_out, const float *d_x, int64_t n, void *stream);

#ifdef __cplusplus
}
#endif

#endif
