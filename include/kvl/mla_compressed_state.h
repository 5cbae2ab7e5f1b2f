/*
 * kvl/mla_compressed_state.h -- compressed (latent) MLA decode state, served by
 * libkvl_mla_cuda on a B200.
 *
 * The struct layout and every function signature are those of the reference
 * runtime (include/kvl/mla_compressed_state.h:7-44), so generate.c,
 * generate_vl.c and the lab tools compile and link unchanged.
 *
 * Storage: the authoritative rows live in GPU memory as bf16 [capacity][R+DR]
 * (latent | rope).  `latent` and `rope` are host mirrors of the same rows in
 * fp32, refreshed after every append.  Rows a caller writes into the mirrors
 * directly (and publishes by raising `len`) are uploaded before the next
 * append/attend; lowering `len` truncates.  Rows below the device length that
 * a caller overwrites in the mirror are not re-read.
 */
#ifndef KVL_MLA_COMPRESSED_STATE_H
#define KVL_MLA_COMPRESSED_STATE_H

#include <stddef.h>
#include "kvl/ops.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int capacity;
    int len;
    int kv_lora_rank;
    int qk_rope_dim;
    float *latent;   /* host mirror [capacity][kv_lora_rank] */
    float *rope;     /* host mirror [capacity][qk_rope_dim] */
} KvlMlaCompressedState;

/* Allocates host mirrors and the device rows on the current CUDA device.
 * 0 / -1 (bad config, capacity <= 0, odd rope dim, allocation failure). */
int kvl_mla_compressed_state_init(KvlMlaCompressedState *state,
                                  const KvlMlaConfig *cfg,
                                  int capacity);
/* len = 0 (O(1)). */
void kvl_mla_compressed_state_reset(KvlMlaCompressedState *state);
/* len = new_len for 0 <= new_len <= len (O(1)); -1 otherwise. */
int kvl_mla_compressed_state_truncate(KvlMlaCompressedState *state, int new_len);
/* Releases host and device storage and zeroes the struct (double free is safe). */
void kvl_mla_compressed_state_free(KvlMlaCompressedState *state);
/* Host bytes, as the reference counts them (sizeof + capacity*(R+DR)*4). */
size_t kvl_mla_compressed_state_bytes(const KvlMlaCompressedState *state);

/* Appends rows 0..seq_len-1 from x [seq_len][H]; requires len == 0. */
int kvl_mla_compressed_state_prefill_bf16(const float *x,
                                          int seq_len,
                                          const KvlMlaConfig *cfg,
                                          const KvlMlaBF16 *w,
                                          KvlMlaCompressedState *state);

/* One absorbed decode step: appends row `position` (== len) and attends over
 * rows 0..position.  out [H], x [H] host fp32. */
int kvl_mla_decode_compressed_bf16(float *out,
                                   const float *x,
                                   int position,
                                   const KvlMlaConfig *cfg,
                                   const KvlMlaBF16 *w,
                                   KvlMlaCompressedState *state);

/* `count` serial decode steps from start_position (== len). */
int kvl_mla_decode_compressed_block_bf16(float *out,
                                         const float *x,
                                         int count,
                                         int start_position,
                                         const KvlMlaConfig *cfg,
                                         const KvlMlaBF16 *w,
                                         KvlMlaCompressedState *state);

#ifdef __cplusplus
}
#endif

#endif
