/*
 * kvl/mla_compressed_q8_state.h -- row-wise Q8 latent MLA decode state, served
 * by libkvl_mla_cuda on a B200.
 *
 * Struct layout and signatures are those of the reference runtime
 * (include/kvl/mla_compressed_q8_state.h:8-38).  The device rows use the
 * reference's byte layout exactly (int8 latent, fp32 row scale, bf16 rope;
 * 644 bytes per token at R=512, DR=64), and the host arrays below mirror them
 * byte for byte after every append.
 */
#ifndef KVL_MLA_COMPRESSED_Q8_STATE_H
#define KVL_MLA_COMPRESSED_Q8_STATE_H

#include <stddef.h>
#include <stdint.h>
#include "kvl/ops.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int capacity;
    int len;
    int kv_lora_rank;
    int qk_rope_dim;
    int8_t *latent_q8;      /* host mirror [capacity][kv_lora_rank] */
    float *latent_scale;    /* host mirror [capacity] */
    uint16_t *rope_bf16;    /* host mirror [capacity][qk_rope_dim] */
} KvlMlaCompressedQ8State;

int kvl_mla_compressed_q8_state_init(KvlMlaCompressedQ8State *state,
                                     const KvlMlaConfig *cfg,
                                     int capacity);
void kvl_mla_compressed_q8_state_reset(KvlMlaCompressedQ8State *state);
int kvl_mla_compressed_q8_state_truncate(KvlMlaCompressedQ8State *state,
                                         int new_len);
void kvl_mla_compressed_q8_state_free(KvlMlaCompressedQ8State *state);
size_t kvl_mla_compressed_q8_state_bytes(const KvlMlaCompressedQ8State *state);

int kvl_mla_compressed_q8_state_prefill_bf16(const float *x,
                                             int seq_len,
                                             const KvlMlaConfig *cfg,
                                             const KvlMlaBF16 *w,
                                             KvlMlaCompressedQ8State *state);

int kvl_mla_decode_compressed_q8_bf16(float *out,
                                      const float *x,
                                      int position,
                                      const KvlMlaConfig *cfg,
                                      const KvlMlaBF16 *w,
                                      KvlMlaCompressedQ8State *state);

#ifdef __cplusplus
}
#endif

#endif
