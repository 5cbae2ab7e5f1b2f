/*
 * kvl_oracle.c -- CPU restatement of the reference MLA hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path in
 * in-c-test_b200/ is compared against.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg may load it.  The product library never
 * links, loads or calls it and has no CPU fallback.
 *
 * Every function restates one piece of the reference runtime
 * (tuantran00541-spec/In-c-test) in plain C, keeping the reference's
 * arithmetic order and precision: double accumulators, float score rounding,
 * float expf, double softmax denominator.  The citation above each function
 * names the reference file:line it follows.
 *
 * Parity is pinned two ways (see tests/test_oracle_cpu.py):
 *   1. against golden vectors under tests/golden/ that were produced by the
 *      reference's own C code (compiled from its sources by oracle/Makefile);
 *   2. against the compiled reference itself (oracle/_ref/libkvl_ref.so) on
 *      seeded inputs, when that library is present.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* include/kvl/ops.h:17-26 -- KvlMlaConfig (same field order). */
typedef struct {
    int hidden_size;
    int num_heads;
    int qk_nope_dim;
    int qk_rope_dim;
    int v_head_dim;
    int kv_lora_rank;
    float rms_eps;
    float rope_theta;
} OrcCfg;

/* src/ops.c:12-17: bf16 is the high half of an IEEE binary32. */
ORC_API float orc_bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* src/mla_compressed_q8_state.c:9-16: round-to-nearest-even to bf16.  Inf and
 * NaN keep their top 16 bits unchanged (a NaN whose payload lives only in the
 * low half therefore becomes Inf); no quieting. */
ORC_API uint16_t orc_f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    if ((u & 0x7f800000u) != 0x7f800000u) {
        uint32_t lsb = (u >> 16) & 1u;
        u += 0x7fffu + lsb;
    }
    return (uint16_t)(u >> 16);
}

/* src/mla_compressed_q8_state.c:9-16 applied elementwise. */
ORC_API void orc_f32_to_bf16_rne_n(uint16_t *dst, const float *src, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_f32_to_bf16_rne(src[i]);
}

/* src/mla_compressed_state.c:8-22 (identical copies: mla_compressed_q8_state.c:18-32,
 * mla_prefill_streaming.c:15-29, ops.c:89-103).  Input pairs are interleaved
 * [e0,o0,e1,o1,...]; output is [rotated evens | rotated odds].  Angle in double,
 * cos/sin rounded to float, rotation in float. */
ORC_API void orc_rope(float *dst, const float *raw, int dim, int position, float theta) {
    const int half = dim / 2;
    for (int i = 0; i < half; ++i) {
        double inv_freq = pow((double)theta, -((double)(2 * i) / (double)dim));
        double ang = (double)position * inv_freq;
        float c = (float)cos(ang);
        float s = (float)sin(ang);
        float e = raw[2 * i];
        float o = raw[2 * i + 1];
        dst[i] = e * c - o * s;
        dst[half + i] = o * c + e * s;
    }
}

/* Table form of the angle arithmetic above: cos/sin of pos * theta^(-2i/dim),
 * as float, for positions [0, n_pos).  Layout [n_pos][dim/2] for each. */
ORC_API void orc_rope_table(float *cos_out, float *sin_out, int dim, int n_pos, float theta) {
    const int half = dim / 2;
    for (int p = 0; p < n_pos; ++p)
        for (int i = 0; i < half; ++i) {
            double inv_freq = pow((double)theta, -((double)(2 * i) / (double)dim));
            double ang = (double)p * inv_freq;
            cos_out[(size_t)p * half + i] = (float)cos(ang);
            sin_out[(size_t)p * half + i] = (float)sin(ang);
        }
}

/* src/ops.c:76-83: y = x * (1/sqrtf((float)(sum x^2 / n) + eps)) * w, sum in double. */
ORC_API void orc_rmsnorm(float *y, const float *x, const uint16_t *w, int n, float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
    float inv = 1.0f / sqrtf((float)(ss / (double)n) + eps);
    for (int i = 0; i < n; ++i) y[i] = x[i] * inv * orc_bf16_to_f32(w[i]);
}

/* src/ops.c:19-24 + 53-66 (scalar build): y[o] = (float)(sum_i (double)w[o,i] * x[i]). */
ORC_API void orc_matvec(float *y, const float *x, const uint16_t *w, int in, int out) {
    for (int o = 0; o < out; ++o) {
        const uint16_t *row = w + (size_t)o * in;
        double acc = 0.0;
        for (int i = 0; i < in; ++i) acc += (double)orc_bf16_to_f32(row[i]) * (double)x[i];
        y[o] = (float)acc;
    }
}

/* src/mla_compressed_q8_state.c:34-55: symmetric per-row int8 quantiser.
 * amax == 0 or non-finite -> all-zero row with scale 1.0.  Otherwise
 * scale = amax/127, inv = 1/scale, q = clamp(roundf(x*inv), -127, 127);
 * roundf rounds half away from zero. */
ORC_API void orc_quantize_row(int8_t *q, float *scale_out, const float *src, int n) {
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) {
        float a = fabsf(src[i]);
        if (a > amax) amax = a;
    }
    if (!(amax > 0.0f) || !isfinite(amax)) {
        memset(q, 0, (size_t)n);
        *scale_out = 1.0f;
        return;
    }
    volatile float scale = amax / 127.0f; /* volatile: keep the two roundings separate */
    volatile float inv = 1.0f / scale;
    for (int i = 0; i < n; ++i) {
        volatile float prod = src[i] * inv;
        float r = roundf(prod);
        if (r > 127.0f) r = 127.0f;
        if (r < -127.0f) r = -127.0f;
        q[i] = (int8_t)r;
    }
    *scale_out = scale;
}

/* src/mla_compressed_q8_state.c:57-61: one float multiply. */
ORC_API float orc_dequant(int8_t q, float scale) {
    volatile float r = (float)q * scale;
    return r;
}

ORC_API void orc_dequant_n(float *dst, const int8_t *q, const float *scale, int rows, int R) {
    for (int t = 0; t < rows; ++t)
        for (int r = 0; r < R; ++r)
            dst[(size_t)t * R + r] = orc_dequant(q[(size_t)t * R + r], scale[t]);
}

/* src/mla_compressed_state.c:132-148: the attend core of the absorbed decode,
 * for every head, over cached rows j = 0..L-1.
 *   s_j   = (float)(sum_r q_lat[r]*latent_j[r] + sum_d q_rope[d]*rope_j[d]) * scale
 *   e_j   = expf(s_j - max_j s_j),  denom = sum_j e_j (double)
 *   mix_r = (float) sum_j ((double)e_j / denom) * latent_j[r]
 * q_lat [NH][R], q_rope [NH][DR], latent [L][R], rope [L][DR], mix [NH][R].
 * lse (optional, [NH]) = max + log(denom): the natural-log normaliser of the
 * same scores, used to check split-KV partials (not part of the reference). */
ORC_API int orc_attend_f32(float *mix, float *lse, const float *q_lat, const float *q_rope,
                           const float *latent, const float *rope, int L, int NH, int R,
                           int DR, float scale) {
    if (L <= 0 || NH <= 0 || R <= 0 || DR < 0) return -1;
    int rc = 0;
#pragma omp parallel for schedule(static)
    for (int h = 0; h < NH; ++h) {
        float *sc = (float *)malloc((size_t)L * sizeof(float));
        if (!sc) { rc = -1; continue; }
        const float *ql = q_lat + (size_t)h * R;
        const float *qr = q_rope + (size_t)h * DR;
        float mx = -INFINITY;
        for (int j = 0; j < L; ++j) {
            const float *lj = latent + (size_t)j * R;
            const float *rj = rope + (size_t)j * DR;
            double dot = 0.0;
            for (int r = 0; r < R; ++r) dot += (double)ql[r] * (double)lj[r];
            for (int d = 0; d < DR; ++d) dot += (double)qr[d] * (double)rj[d];
            sc[j] = (float)dot * scale;
            if (sc[j] > mx) mx = sc[j];
        }
        double denom = 0.0;
        for (int j = 0; j < L; ++j) {
            sc[j] = expf(sc[j] - mx);
            denom += sc[j];
        }
        float *mh = mix + (size_t)h * R;
        for (int r = 0; r < R; ++r) {
            double acc = 0.0;
            for (int j = 0; j < L; ++j)
                acc += ((double)sc[j] / denom) * (double)latent[(size_t)j * R + r];
            mh[r] = (float)acc;
        }
        if (lse) lse[h] = (float)((double)mx + log(denom));
        free(sc);
    }
    return rc;
}

/* src/mla_compressed_q8_state.c:216-238: the same attend core over the Q8
 * state: latent_j[r] = dequant(q8[j][r], scale[j]) (one float multiply, :57-61)
 * and rope_j = bf16 -> f32. */
ORC_API int orc_attend_q8(float *mix, float *lse, const float *q_lat, const float *q_rope,
                          const int8_t *latent_q8, const float *latent_scale,
                          const uint16_t *rope_bf16, int L, int NH, int R, int DR, float scale) {
    if (L <= 0 || NH <= 0 || R <= 0 || DR < 0) return -1;
    float *lat = (float *)malloc((size_t)L * R * sizeof(float));
    float *rp = (float *)malloc((size_t)L * (DR > 0 ? DR : 1) * sizeof(float));
    if (!lat || !rp) { free(lat); free(rp); return -1; }
    orc_dequant_n(lat, latent_q8, latent_scale, L, R);
    for (size_t i = 0; i < (size_t)L * DR; ++i) rp[i] = orc_bf16_to_f32(rope_bf16[i]);
    int rc = orc_attend_f32(mix, lse, q_lat, q_rope, lat, rp, L, NH, R, DR, scale);
    free(lat); free(rp);
    return rc;
}

/* src/mla_compressed_state.c:73-80 (one token): kv_a matvec, RMSNorm of the
 * first R outputs with kv_a_norm, RoPE of the last DR outputs at `position`. */
ORC_API void orc_append_f32(float *latent_row, float *rope_row, const float *x, int position,
                            const OrcCfg *c, const uint16_t *kv_a, const uint16_t *kv_a_norm) {
    const int R = c->kv_lora_rank, DR = c->qk_rope_dim;
    float *ka = (float *)malloc((size_t)(R + DR) * sizeof(float));
    orc_matvec(ka, x, kv_a, c->hidden_size, R + DR);
    orc_rmsnorm(latent_row, ka, kv_a_norm, R, c->rms_eps);
    orc_rope(rope_row, ka + R, DR, position, c->rope_theta);
    free(ka);
}

/* src/mla_compressed_q8_state.c:111-127 (one token): the append above followed by
 * the row quantiser and bf16 RNE of the rotated rope. */
ORC_API void orc_append_q8(int8_t *q_row, float *scale_out, uint16_t *rope_row, const float *x,
                           int position, const OrcCfg *c, const uint16_t *kv_a,
                           const uint16_t *kv_a_norm) {
    const int R = c->kv_lora_rank, DR = c->qk_rope_dim;
    float *lat = (float *)malloc((size_t)R * sizeof(float));
    float *rp = (float *)malloc((size_t)DR * sizeof(float));
    orc_append_f32(lat, rp, x, position, c, kv_a, kv_a_norm);
    orc_quantize_row(q_row, scale_out, lat, R);
    for (int d = 0; d < DR; ++d) rope_row[d] = orc_f32_to_bf16_rne(rp[d]);
    free(lat); free(rp);
}

/* src/mla_compressed_state.c:119-131 for one head: q rope at `position` and the
 * absorption q_lat[r] = (float) sum_d kv_b[h*(DN+DV)+d][r] * q_nope[d] (double). */
ORC_API void orc_absorb(float *q_lat, float *q_rope, const float *q, int position,
                        const OrcCfg *c, const uint16_t *kv_b) {
    const int NH = c->num_heads, DN = c->qk_nope_dim, DR = c->qk_rope_dim;
    const int DV = c->v_head_dim, R = c->kv_lora_rank, QD = DN + DR;
    for (int h = 0; h < NH; ++h) {
        const float *qh = q + (size_t)h * QD;
        orc_rope(q_rope + (size_t)h * DR, qh + DN, DR, position, c->rope_theta);
        for (int r = 0; r < R; ++r) {
            double acc = 0.0;
            for (int d = 0; d < DN; ++d)
                acc += (double)orc_bf16_to_f32(kv_b[(size_t)(h * (DN + DV) + d) * R + r]) *
                       (double)qh[d];
            q_lat[(size_t)h * R + r] = (float)acc;
        }
    }
}

/* src/mla_compressed_state.c:149-155: ho[h][d] = (float) sum_r kv_b[h*(DN+DV)+DN+d][r]*mix[h][r]. */
ORC_API void orc_vup(float *ho, const float *mix, const OrcCfg *c, const uint16_t *kv_b) {
    const int NH = c->num_heads, DN = c->qk_nope_dim, DV = c->v_head_dim, R = c->kv_lora_rank;
    for (int h = 0; h < NH; ++h)
        for (int d = 0; d < DV; ++d) {
            const uint16_t *row = kv_b + (size_t)(h * (DN + DV) + DN + d) * R;
            double acc = 0.0;
            for (int r = 0; r < R; ++r)
                acc += (double)orc_bf16_to_f32(row[r]) * (double)mix[(size_t)h * R + r];
            ho[(size_t)h * DV + d] = (float)acc;
        }
}

/* src/mla_compressed_state.c:86-161: one absorbed decode step over an fp32
 * state (latent [cap][R], rope [cap][DR]) holding `position` rows.  Appends row
 * `position` before attending, so the token attends to itself. */
ORC_API int orc_decode_f32(float *out, const float *x, int position, const OrcCfg *c,
                           const uint16_t *q_proj, const uint16_t *kv_a,
                           const uint16_t *kv_a_norm, const uint16_t *kv_b,
                           const uint16_t *o_proj, float *latent, float *rope) {
    const int H = c->hidden_size, NH = c->num_heads, DN = c->qk_nope_dim;
    const int DR = c->qk_rope_dim, DV = c->v_head_dim, R = c->kv_lora_rank, QD = DN + DR;
    float *q = (float *)malloc((size_t)NH * QD * sizeof(float));
    float *ql = (float *)malloc((size_t)NH * R * sizeof(float));
    float *qr = (float *)malloc((size_t)NH * DR * sizeof(float));
    float *mix = (float *)malloc((size_t)NH * R * sizeof(float));
    float *ho = (float *)malloc((size_t)NH * DV * sizeof(float));
    orc_matvec(q, x, q_proj, H, NH * QD);
    orc_append_f32(latent + (size_t)position * R, rope + (size_t)position * DR, x, position, c,
                   kv_a, kv_a_norm);
    orc_absorb(ql, qr, q, position, c, kv_b);
    int rc = orc_attend_f32(mix, NULL, ql, qr, latent, rope, position + 1, NH, R, DR,
                            1.0f / sqrtf((float)QD));
    orc_vup(ho, mix, c, kv_b);
    orc_matvec(out, ho, o_proj, NH * DV, H);
    free(q); free(ql); free(qr); free(mix); free(ho);
    return rc;
}

/* src/mla_compressed_q8_state.c:161-255: the same step over a Q8 state. */
ORC_API int orc_decode_q8(float *out, const float *x, int position, const OrcCfg *c,
                          const uint16_t *q_proj, const uint16_t *kv_a,
                          const uint16_t *kv_a_norm, const uint16_t *kv_b,
                          const uint16_t *o_proj, int8_t *latent_q8, float *latent_scale,
                          uint16_t *rope_bf16) {
    const int H = c->hidden_size, NH = c->num_heads, DN = c->qk_nope_dim;
    const int DR = c->qk_rope_dim, DV = c->v_head_dim, R = c->kv_lora_rank, QD = DN + DR;
    float *q = (float *)malloc((size_t)NH * QD * sizeof(float));
    float *ql = (float *)malloc((size_t)NH * R * sizeof(float));
    float *qr = (float *)malloc((size_t)NH * DR * sizeof(float));
    float *mix = (float *)malloc((size_t)NH * R * sizeof(float));
    float *ho = (float *)malloc((size_t)NH * DV * sizeof(float));
    orc_matvec(q, x, q_proj, H, NH * QD);
    orc_append_q8(latent_q8 + (size_t)position * R, latent_scale + position,
                  rope_bf16 + (size_t)position * DR, x, position, c, kv_a, kv_a_norm);
    orc_absorb(ql, qr, q, position, c, kv_b);
    int rc = orc_attend_q8(mix, NULL, ql, qr, latent_q8, latent_scale, rope_bf16, position + 1,
                           NH, R, DR, 1.0f / sqrtf((float)QD));
    orc_vup(ho, mix, c, kv_b);
    orc_matvec(out, ho, o_proj, NH * DV, H);
    free(q); free(ql); free(qr); free(mix); free(ho);
    return rc;
}

/* src/mla_prefill_streaming.c:78-206: causal MLA prefill, non-absorbed.
 * Per token: latent = rmsnorm(kv_a x)[:R], k_rope = rope(kv_a x [R:]).
 * Per head: k_nope_j | v_j = kv_b_h latent_j; q_h = q_proj_h x_t with rope on
 * the last DR; s_j = (float)(q_nope.k_nope_j + q_rope.k_rope_j) * scale for j<=t,
 * softmax with float expf / double denom, head_out = sum p_j v_j (double).
 * out_t = o_proj head_out_t.  x [S][H] -> out [S][H]. */
ORC_API int orc_prefill(float *out, const float *x, int S, const OrcCfg *c,
                        const uint16_t *q_proj, const uint16_t *kv_a,
                        const uint16_t *kv_a_norm, const uint16_t *kv_b,
                        const uint16_t *o_proj) {
    const int H = c->hidden_size, NH = c->num_heads, DN = c->qk_nope_dim;
    const int DR = c->qk_rope_dim, DV = c->v_head_dim, R = c->kv_lora_rank;
    const int QD = DN + DR, KHV = DN + DV, HO = NH * DV;
    if (S <= 0) return -1;
    float *lat = (float *)malloc((size_t)S * R * sizeof(float));
    float *krope = (float *)malloc((size_t)S * DR * sizeof(float));
    float *kn = (float *)malloc((size_t)S * DN * sizeof(float));
    float *vv = (float *)malloc((size_t)S * DV * sizeof(float));
    float *heads = (float *)malloc((size_t)S * HO * sizeof(float));
    if (!lat || !krope || !kn || !vv || !heads) {
        free(lat); free(krope); free(kn); free(vv); free(heads);
        return -1;
    }
#pragma omp parallel for schedule(static)
    for (int t = 0; t < S; ++t)
        orc_append_f32(lat + (size_t)t * R, krope + (size_t)t * DR, x + (size_t)t * H, t, c,
                       kv_a, kv_a_norm);
    const float scale = 1.0f / sqrtf((float)QD);
    for (int h = 0; h < NH; ++h) {
        const uint16_t *kvh = kv_b + (size_t)h * KHV * R;
#pragma omp parallel for schedule(static)
        for (int j = 0; j < S; ++j) {
            float tmp[1024];
            float *kv = KHV <= 1024 ? tmp : (float *)malloc((size_t)KHV * sizeof(float));
            orc_matvec(kv, lat + (size_t)j * R, kvh, R, KHV);
            memcpy(kn + (size_t)j * DN, kv, (size_t)DN * sizeof(float));
            memcpy(vv + (size_t)j * DV, kv + DN, (size_t)DV * sizeof(float));
            if (kv != tmp) free(kv);
        }
        const uint16_t *qh_w = q_proj + (size_t)h * QD * H;
#pragma omp parallel for schedule(dynamic, 8)
        for (int t = 0; t < S; ++t) {
            float *qt = (float *)malloc((size_t)QD * sizeof(float));
            float *qr = (float *)malloc((size_t)DR * sizeof(float));
            float *sc = (float *)malloc((size_t)(t + 1) * sizeof(float));
            double *acc = (double *)calloc((size_t)DV, sizeof(double));
            orc_matvec(qt, x + (size_t)t * H, qh_w, H, QD);
            orc_rope(qr, qt + DN, DR, t, c->rope_theta);
            float mx = -INFINITY;
            for (int j = 0; j <= t; ++j) {
                double d1 = 0.0, d2 = 0.0;
                for (int d = 0; d < DN; ++d) d1 += (double)qt[d] * (double)kn[(size_t)j * DN + d];
                for (int d = 0; d < DR; ++d) d2 += (double)qr[d] * (double)krope[(size_t)j * DR + d];
                sc[j] = (float)(d1 + d2) * scale;
                if (sc[j] > mx) mx = sc[j];
            }
            double den = 0.0;
            for (int j = 0; j <= t; ++j) {
                sc[j] = expf(sc[j] - mx);
                den += sc[j];
            }
            for (int j = 0; j <= t; ++j) {
                double p = (double)sc[j] / den;
                for (int d = 0; d < DV; ++d) acc[d] += p * (double)vv[(size_t)j * DV + d];
            }
            float *ho = heads + (size_t)t * HO + (size_t)h * DV;
            for (int d = 0; d < DV; ++d) ho[d] = (float)acc[d];
            free(qt); free(qr); free(sc); free(acc);
        }
    }
#pragma omp parallel for schedule(static)
    for (int t = 0; t < S; ++t)
        orc_matvec(out + (size_t)t * H, heads + (size_t)t * HO, o_proj, HO, H);
    free(lat); free(krope); free(kn); free(vv); free(heads);
    return 0;
}
