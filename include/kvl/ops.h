/*
 * kvl/ops.h -- the MLA subset of the reference runtime's include/kvl/ops.h.
 *
 * Same include guard, type names, field order and prefill signature as the
 * reference (include/kvl/ops.h:17-34, :63-64), so a translation unit that
 * includes the reference's own ops.h first sees identical definitions and
 * skips this one.  Standalone users of libkvl_mla_cuda include this file.
 */
#ifndef KVL_OPS_H
#define KVL_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Model dimensions of one MLA layer (reference include/kvl/ops.h:17-26). */
typedef struct {
    int hidden_size;   /* H */
    int num_heads;     /* NH */
    int qk_nope_dim;   /* DN */
    int qk_rope_dim;   /* DR, even */
    int v_head_dim;    /* DV */
    int kv_lora_rank;  /* R */
    float rms_eps;
    float rope_theta;
} KvlMlaConfig;

/* Host pointers to the layer's bf16 weights, row-major as uint16_t
 * (reference include/kvl/ops.h:28-34):
 *   q_proj    [NH*(DN+DR)][H]     kv_a_proj [R+DR][H]    kv_a_norm [R]
 *   kv_b_proj [NH*(DN+DV)][R]     o_proj    [H][NH*DV] */
typedef struct {
    const uint16_t *q_proj;
    const uint16_t *kv_a_proj;
    const uint16_t *kv_a_norm;
    const uint16_t *kv_b_proj;
    const uint16_t *o_proj;
} KvlMlaBF16;

/* Causal MLA prefill of seq_len tokens: x [seq_len][H] fp32 host ->
 * out [seq_len][H] fp32 host.  Returns 0, or -1 on invalid arguments or a
 * CUDA failure.  Replaces src/mla_prefill_streaming.c:78-206. */
int kvl_mla_prefill_bf16(float *out, const float *x, int seq_len,
                         const KvlMlaConfig *cfg, const KvlMlaBF16 *w);

#ifdef __cplusplus
}
#endif

#endif
