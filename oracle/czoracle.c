/*
 * czoracle.c -- CPU oracle for the compress-zip model-plus-coder path.
 *
 * TEST INFRASTRUCTURE ONLY (checker and CPU baseline; never the product).
 * A plain-C restatement of the reference Rust crate carsonpo/compress-zip
 * (the rust/src files).  Rust release builds wrap on integer overflow; C signed
 * overflow is undefined, so every add/multiply that may wrap in the reference
 * is done here in unsigned arithmetic and converted back.
 */
#include "czoracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* primitives (rust/src/primitives.rs)                                      */
/* ------------------------------------------------------------------------ */

/* primitives.rs:9-11 -- symmetric int8 clamp [-127, 127] */
int8_t czo_clamp_i8(int32_t x) {
    if (x < -127) return -127;
    if (x > 127) return 127;
    return (int8_t)x;
}

/* primitives.rs:18-42 -- arithmetic shift right, round half to even */
int32_t czo_sra_rne_s32(int32_t v, uint32_t sh) {
    if (sh == 0) return v;
    uint32_t sign = (uint32_t)(v >> 31);              /* all ones when negative */
    uint32_t av = ((uint32_t)v ^ sign) - sign;         /* |v| without overflow   */
    uint32_t mask = (1u << sh) - 1u;
    uint32_t r = av & mask;
    uint32_t q = av >> sh;
    uint32_t half = 1u << (sh - 1);
    if (r > half) q += 1;
    else if (r == half) q += q & 1u;
    return (int32_t)((q ^ sign) - sign);
}

/* primitives.rs:49-73 -- 64-bit shift right, round half to even, clamp to i32 */
int32_t czo_sra_rne_s64_to_s32(int64_t v, uint32_t sh) {
    if (sh == 0) {
        if (v < INT32_MIN) return INT32_MIN;
        if (v > INT32_MAX) return INT32_MAX;
        return (int32_t)v;
    }
    uint64_t sign = (uint64_t)(v >> 63);
    uint64_t av = ((uint64_t)v ^ sign) - sign;
    uint64_t mask = (1ull << sh) - 1ull;
    uint64_t r = av & mask;
    uint64_t q = av >> sh;
    uint64_t half = 1ull << (sh - 1);
    if (r > half) q += 1;
    else if (r == half) q += q & 1ull;
    int64_t out = (int64_t)((q ^ sign) - sign);
    if (out < INT32_MIN) return INT32_MIN;
    if (out > INT32_MAX) return INT32_MAX;
    return (int32_t)out;
}

/* primitives.rs:80-97 -- unsigned division, ties to even only when 2r == d */
uint32_t czo_udiv_rne_u32(uint32_t n, uint32_t d) {
    if (d == 0) return 0;
    uint32_t q = n / d;
    uint32_t r = n - q * d;
    uint32_t twice_r = r << 1;
    if (twice_r > d) return q + 1;
    if (twice_r == d) return q + (q & 1u);
    return q;
}

/* primitives.rs:163-185 -- i32 / u64 with ties to even; the final
 * `(q as i32) * sign` wraps in a release build */
int32_t czo_div_rne_s32_by_u64(int32_t num, uint64_t den) {
    if (den == 0) return 0;
    uint32_t sign_neg = num < 0;
    uint64_t an = sign_neg ? (uint64_t)(0u - (uint32_t)num) : (uint64_t)(uint32_t)num;
    uint64_t q = an / den;
    uint64_t r = an - q * den;
    uint64_t twice_r = r << 1;
    uint64_t rq;
    if (twice_r > den) rq = q + 1;
    else if (twice_r == den) rq = q + (q & 1ull);
    else rq = q;
    uint32_t q32 = (uint32_t)rq;
    return (int32_t)(sign_neg ? 0u - q32 : q32);
}

/* primitives.rs:192-213 -- restoring integer square root */
uint32_t czo_isqrt32(uint32_t x) {
    uint32_t op = x, res = 0, one = 1u << 30;
    while (one > op) one >>= 2;
    while (one != 0) {
        if (op >= res + one) {
            op -= res + one;
            res = (res >> 1) + one;
        } else {
            res >>= 1;
        }
        one >>= 2;
    }
    return res;
}

/* lut.rs:213-235 and softmax_cdf.rs:55-77 (identical formula) */
uint16_t czo_exp_q16(int32_t neg_x, const uint16_t *lut, uint32_t coef_q24) {
    if (neg_x >= 0) return 65535;
    uint32_t neg = 0u - (uint32_t)neg_x;
    uint32_t t256 = (uint32_t)(((uint64_t)neg * (uint64_t)coef_q24 + (1ull << 23)) >> 24);
    uint32_t ip = t256 >> 8;
    uint32_t frac = t256 & 255u;
    if (ip >= 31) return 1;
    uint32_t base = (1u << 16) >> ip;
    uint32_t out = (base * (uint32_t)lut[frac] + 0x8000u) >> 16;
    if (out < 1) out = 1;
    if (out > 65535) out = 65535;
    return (uint16_t)out;
}

/* attention.rs:14-19 -- ATTN_COEF_Q24 = (LOG2E / 64 * 2^24 + 0.5) as u32 */
uint32_t czo_attn_coef_q24(void) {
    const double log2e = 1.4426950408889634;
    return (uint32_t)((log2e / 64.0) * (double)(1ull << 24) + 0.5);
}

/* softmax_cdf.rs:23-28 -- COEF_Q24 = round(0.1 * LOG2E / 64 * 2^24), at least 1 */
uint32_t czo_default_coef_q24(void) {
    const double log2e = 1.4426950408889634;
    double coef_d = (0.1 * log2e) / 64.0;
    double scaled = coef_d * (double)(1u << 24);
    uint32_t r = (uint32_t)round(scaled);   /* f64::round: half away from zero */
    return r < 1 ? 1 : r;
}

/* softmax_cdf.rs:39-46 -- 2^30 - V - 1024 (saturating), at least V + 1 */
uint32_t czo_default_target_total(int V) {
    uint32_t quarter = 1u << 30, vs = (uint32_t)V;
    uint32_t t = quarter > vs ? quarter - vs : 0;
    t = t > 1024 ? t - 1024 : 0;
    return t > vs + 1 ? t : vs + 1;
}

/* ------------------------------------------------------------------------ */
/* layers                                                                   */
/* ------------------------------------------------------------------------ */

/* rmsnorm.rs:14-30 */
int32_t czo_inv_rms_q15(int32_t mean_sq) {
    uint32_t ms = mean_sq > 0 ? (uint32_t)mean_sq : 1u;
    uint32_t x_scaled = ms << 16;
    uint32_t s = czo_isqrt32(x_scaled);
    uint32_t inv = czo_udiv_rne_u32(8388608u, s);
    if (inv < 1) inv = 1;
    if (inv > 32768) inv = 32768;
    return (int32_t)inv;
}

/* rmsnorm.rs:40-75 (rmsnorm_i8 followed by the clamp of rmsnorm_i8_to_i8) */
void czo_rmsnorm_i8(const int8_t *x, const int8_t *w, int d, int32_t eps, int8_t *out) {
    uint32_t sum_sq = 0;
    for (int i = 0; i < d; i++) sum_sq += (uint32_t)((int32_t)x[i] * (int32_t)x[i]);
    int32_t mean_sq = (int32_t)(sum_sq / (uint32_t)d) + eps;
    if (mean_sq < 1) mean_sq = 1;
    int32_t inv = czo_inv_rms_q15(mean_sq);
    for (int i = 0; i < d; i++) {
        int32_t tmp = ((int32_t)x[i] * (int32_t)w[i]) * inv;
        out[i] = czo_clamp_i8(czo_sra_rne_s32(tmp, 15));
    }
}

/* linear.rs:12-31 -- y[o] = sum_i x[i] * W[o, i] */
void czo_linear_i8_i32(const int8_t *x, const int8_t *W, int in_dim, int out_dim, int32_t *y) {
    for (int o = 0; o < out_dim; o++) {
        const int8_t *wr = W + (size_t)o * in_dim;
        int32_t acc = 0;
        for (int i = 0; i < in_dim; i++) acc += (int32_t)x[i] * (int32_t)wr[i];
        y[o] = acc;
    }
}

/* model.rs:280-300 */
void czo_requant(const int32_t *x, int n, int32_t mult, int8_t shift, int8_t *out) {
    for (int i = 0; i < n; i++) {
        int64_t p = (int64_t)x[i] * (int64_t)mult;
        if (shift <= 0) {
            out[i] = (int8_t)(p < -127 ? -127 : (p > 127 ? 127 : p));
        } else {
            out[i] = czo_clamp_i8(czo_sra_rne_s64_to_s32(p, (uint32_t)shift));
        }
    }
}

/* reglu.rs:20-46 -- gate = first d_ff, value = second d_ff */
void czo_reglu(const int8_t *x, int d_ff, int8_t *out) {
    for (int i = 0; i < d_ff; i++) {
        int32_t g = x[i] > 0 ? x[i] : 0;
        out[i] = czo_clamp_i8(czo_sra_rne_s32(g * (int32_t)x[d_ff + i], 7));
    }
}

/* attention.rs:29-50 -- rotate pairs (i, i+32) with the Q1.15 table row `pos` */
void czo_rope_k(int8_t *x, const int16_t *cos_t, const int16_t *sin_t, int pos) {
    for (int i = 0; i < CZO_HALF_DIM; i++) {
        int32_t xv = x[i], yv = x[i + CZO_HALF_DIM];
        int32_t c = cos_t[pos * CZO_HALF_DIM + i], s = sin_t[pos * CZO_HALF_DIM + i];
        x[i] = czo_clamp_i8(czo_sra_rne_s32(xv * c - yv * s, 15));
        x[i + CZO_HALF_DIM] = czo_clamp_i8(czo_sra_rne_s32(xv * s + yv * c, 15));
    }
}

/* attention.rs:53-83 -- as czo_rope_k plus the NET_SHIFT = 3 - 2 = 1 rounding */
void czo_rope_q(int8_t *x, const int16_t *cos_t, const int16_t *sin_t, int pos) {
    for (int i = 0; i < CZO_HALF_DIM; i++) {
        int32_t xv = x[i], yv = x[i + CZO_HALF_DIM];
        int32_t c = cos_t[pos * CZO_HALF_DIM + i], s = sin_t[pos * CZO_HALF_DIM + i];
        int32_t xr = czo_sra_rne_s32(xv * c - yv * s, 15);
        int32_t yr = czo_sra_rne_s32(xv * s + yv * c, 15);
        x[i] = czo_clamp_i8(czo_sra_rne_s32(xr, 1));
        x[i + CZO_HALF_DIM] = czo_clamp_i8(czo_sra_rne_s32(yr, 1));
    }
}

/* softmax_cdf.rs:85-139 */
void czo_build_cumfreqs(const int32_t *logits, int V, const uint16_t *lut, uint32_t coef_q24,
                        uint32_t target_total, uint32_t *cum) {
    int32_t mx = logits[0];
    int amax = 0;
    for (int i = 1; i < V; i++)
        if (logits[i] > mx) { mx = logits[i]; amax = i; }
    uint64_t sum_exp = 0;
    uint16_t *e = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)V);
    for (int i = 0; i < V; i++) {
        int32_t diff = (int32_t)((uint32_t)logits[i] - (uint32_t)mx);
        e[i] = czo_exp_q16(diff, lut, coef_q24);
        sum_exp += e[i];
    }
    uint64_t remaining = (uint64_t)target_total - (uint64_t)V;
    uint64_t freq_sum = 0;
    for (int i = 0; i < V; i++) {
        uint32_t f = 1u + (uint32_t)(((uint64_t)e[i] * remaining) / sum_exp);
        cum[i] = f;   /* holds freq until the prefix sum below */
        freq_sum += f;
    }
    cum[amax] += (uint32_t)((uint64_t)target_total - freq_sum);
    uint32_t run = 0;
    for (int i = 0; i < V; i++) {
        run += cum[i];
        cum[i] = run;
    }
    free(e);
}

/* ------------------------------------------------------------------------ */
/* attention (attention.rs:162-289)                                          */
/* ------------------------------------------------------------------------ */

/* One query head at position `step` over cached rotated keys kc[0..step] and
 * values vc[0..step] ([t][64] each): the ordered online softmax of
 * attention.rs:199-284, with the optional sink key of attention.rs:211-224. */
static void attn_one_head(const int8_t *q_in, const int8_t *kc, const int8_t *vc, int step,
                          int32_t mult, const int8_t *sink_key, const int16_t *cos_t,
                          const int16_t *sin_t, const uint16_t *lut, int8_t *out) {
    const int D = 64;
    const uint32_t coef = czo_attn_coef_q24();
    int8_t q[64];
    memcpy(q, q_in, 64);
    czo_rope_q(q, cos_t, sin_t, step);
    int32_t mrun = INT32_MIN;
    uint64_t s = 0;
    uint32_t vacc[64];   /* i32 with wrapping adds */
    memset(vacc, 0, sizeof(vacc));
    if (sink_key) {
        int32_t dot = 0;
        for (int i = 0; i < D; i++) dot += (int32_t)q[i] * (int32_t)sink_key[i];
        int32_t du = czo_sra_rne_s32(dot, 2);
        mrun = czo_sra_rne_s64_to_s32((int64_t)du * (int64_t)mult, 15);
        s = czo_exp_q16(0, lut, coef);
    }
    for (int t = 0; t <= step; t++) {
        const int8_t *k = kc + (size_t)t * D;
        int32_t dot = 0;
        for (int i = 0; i < D; i++) dot += (int32_t)q[i] * (int32_t)k[i];
        int32_t du = czo_sra_rne_s32(dot, 2);
        int32_t score = czo_sra_rne_s64_to_s32((int64_t)du * (int64_t)mult, 15);
        if (score > mrun) {
            if (mrun != INT32_MIN) {
                int32_t diff = (int32_t)((uint32_t)mrun - (uint32_t)score);
                uint16_t so = czo_exp_q16(diff, lut, coef);
                s = (s * so + 0x8000ull) >> 16;
                for (int i = 0; i < D; i++) {
                    int64_t p = (int64_t)(int32_t)vacc[i] * (int64_t)so;
                    int64_t adj = p >= 0 ? p + (1ll << 15) : p - (1ll << 15);
                    vacc[i] = (uint32_t)(int32_t)(adj >> 16);
                }
            }
            mrun = score;
        }
        int32_t diff = (int32_t)((uint32_t)score - (uint32_t)mrun);
        uint16_t w = czo_exp_q16(diff, lut, coef);
        s += w;
        const int8_t *v = vc + (size_t)t * D;
        for (int i = 0; i < D; i++) vacc[i] += (uint32_t)((int32_t)w * (int32_t)v[i]);
    }
    uint64_t den = s == 0 ? 1 : s;
    for (int i = 0; i < D; i++) out[i] = czo_clamp_i8(czo_div_rne_s32_by_u64((int32_t)vacc[i], den));
}

/* attention.rs:162-289.  qkv holds [q (n_heads*64) | k (64) | v (64) ...] as the
 * reference's single-KV-head attention reads it (attention.rs:174-194).
 * kc/vc: [max_seq_len][64]. */
static void attention_step(const czo_model *m, const czo_layer *L, const int8_t *qkv,
                           int8_t *kc, int8_t *vc, int step, int8_t *out) {
    const int H = m->n_heads, D = 64, d = H * D;
    int8_t krot[64];
    memcpy(krot, qkv + d, 64);
    czo_rope_k(krot, m->rope_cos, m->rope_sin, step);
    memcpy(kc + (size_t)step * D, krot, 64);
    memcpy(vc + (size_t)step * D, qkv + d + 64, 64);
    for (int h = 0; h < H; h++)
        attn_one_head(qkv + h * D, kc, vc, step, L->score_mult[h], L->sink_key, m->rope_cos,
                      m->rope_sin, m->exp2_lut, out + h * D);
}

void czo_attention_seq(const int8_t *q, const int8_t *k, const int8_t *v, int n, int H,
                       const int32_t *score_mult, const int8_t *sink_key, const int16_t *cos_t,
                       const int16_t *sin_t, const uint16_t *lut, int8_t *out) {
    int8_t *kc = (int8_t *)malloc((size_t)n * 64 + 64);
    int8_t *vc = (int8_t *)malloc((size_t)n * 64 + 64);
    for (int t = 0; t < n; t++) {
        memcpy(kc + (size_t)t * 64, k + (size_t)t * 64, 64);
        czo_rope_k(kc + (size_t)t * 64, cos_t, sin_t, t);
        memcpy(vc + (size_t)t * 64, v + (size_t)t * 64, 64);
        for (int h = 0; h < H; h++)
            attn_one_head(q + ((size_t)t * H + h) * 64, kc, vc, t, score_mult[h], sink_key, cos_t,
                          sin_t, lut, out + ((size_t)t * H + h) * 64);
    }
    free(kc);
    free(vc);
}

/* ------------------------------------------------------------------------ */
/* model (model.rs:315-486)                                                  */
/* ------------------------------------------------------------------------ */

int czo_model_check(const czo_model *m) {
    if (m->n_layers < 1 || m->n_layers > CZO_MAX_LAYERS) return -1;
    /* attention.rs:172 */
    if (!(m->n_heads == 4 || m->n_heads == 6 || m->n_heads == 8)) return -2;
    if (m->head_dim != 64) return -3;
    if (m->d_model != m->n_heads * 64) return -4;
    /* attention.rs:176: the batch count must come out as exactly 1 */
    int qkv_rows = m->d_model + 2 * m->n_kv_heads * 64;
    if (m->n_kv_heads < 1 || qkv_rows / (m->d_model + 128) != 1) return -5;
    if (m->vocab <= (int)CZO_BOS) return -6;   /* BOS 1022 indexes the embedding */
    return 0;
}

size_t czo_kv_bytes(const czo_model *m) {
    return (size_t)m->n_layers * 2 * (size_t)m->max_seq_len * 64;
}

/* model.rs:362-480.  `kv` carries this chunk's KV caches between calls.
 * att_cap ([n_layers][d]) and fin_cap ([d]) capture intermediates when non-NULL. */
static void forward_impl(const czo_model *m, int8_t *kv, uint32_t token, int pos, int32_t *logits,
                         int8_t *att_cap, int8_t *fin_cap) {
    const int d = m->d_model, dff = m->d_ff, kvd = m->n_kv_heads * 64;
    const int qkv_rows = d + 2 * kvd;
    int32_t *x = (int32_t *)malloc(sizeof(int32_t) * d);
    int8_t *x8 = (int8_t *)malloc((size_t)d);
    int8_t *nrm = (int8_t *)malloc((size_t)d);
    int32_t *acc = (int32_t *)malloc(sizeof(int32_t) * (size_t)(qkv_rows > 2 * dff ? qkv_rows : 2 * dff));
    int8_t *qkv = (int8_t *)malloc((size_t)qkv_rows);
    int8_t *att = (int8_t *)malloc((size_t)d);
    int8_t *o8 = (int8_t *)malloc((size_t)d);
    int8_t *gu = (int8_t *)malloc((size_t)(2 * dff));
    int8_t *g = (int8_t *)malloc((size_t)dff);

    const int8_t *emb = m->embed + (size_t)token * d;
    for (int i = 0; i < d; i++) x[i] = emb[i];
    for (int l = 0; l < m->n_layers; l++) {
        const czo_layer *L = &m->layers[l];
        int8_t *kc = kv + (size_t)l * 2 * m->max_seq_len * 64;
        int8_t *vc = kc + (size_t)m->max_seq_len * 64;
        for (int i = 0; i < d; i++) x8[i] = czo_clamp_i8(x[i]);
        czo_rmsnorm_i8(x8, L->attn_norm, d, m->eps_scaled, nrm);
        czo_linear_i8_i32(nrm, L->qkv_w, d, qkv_rows, acc);
        czo_requant(acc, qkv_rows, L->qkv_mult, (int8_t)L->qkv_shift, qkv);
        attention_step(m, L, qkv, kc, vc, pos, att);
        if (att_cap) memcpy(att_cap + (size_t)l * d, att, (size_t)d);
        czo_linear_i8_i32(att, L->out_w, d, d, acc);
        czo_requant(acc, d, L->out_mult, (int8_t)L->out_shift, o8);
        czo_rmsnorm_i8(o8, L->ffn_norm, d, m->eps_scaled, nrm);
        for (int i = 0; i < d; i++) x[i] = (int32_t)((uint32_t)x[i] + (uint32_t)(int32_t)nrm[i]);
        for (int i = 0; i < d; i++) x8[i] = czo_clamp_i8(x[i]);
        czo_rmsnorm_i8(x8, L->post_attn_norm, d, m->eps_scaled, nrm);
        czo_linear_i8_i32(nrm, L->up_w, d, 2 * dff, acc);
        czo_requant(acc, 2 * dff, L->up_mult, (int8_t)L->up_shift, gu);
        czo_reglu(gu, dff, g);
        czo_linear_i8_i32(g, L->down_w, dff, d, acc);
        czo_requant(acc, d, L->down_mult, (int8_t)L->down_shift, o8);
        czo_rmsnorm_i8(o8, L->post_ffn_norm, d, m->eps_scaled, nrm);
        for (int i = 0; i < d; i++) x[i] = (int32_t)((uint32_t)x[i] + (uint32_t)(int32_t)nrm[i]);
    }
    for (int i = 0; i < d; i++) x8[i] = czo_clamp_i8(x[i]);
    czo_rmsnorm_i8(x8, m->final_norm, d, m->eps_scaled, nrm);
    if (fin_cap) memcpy(fin_cap, nrm, (size_t)d);
    czo_linear_i8_i32(nrm, m->head_w, d, m->vocab, logits);
    free(x); free(x8); free(nrm); free(acc); free(qkv); free(att); free(o8); free(gu); free(g);
}

void czo_forward(const czo_model *m, int8_t *kv, uint32_t token, int pos, int32_t *logits) {
    forward_impl(m, kv, token, pos, logits, NULL, NULL);
}

/* ------------------------------------------------------------------------ */
/* arithmetic coder (arith_coder.rs)                                         */
/* ------------------------------------------------------------------------ */
#define STATE_MASK 0xFFFFFFFFull
#define HALF_RANGE (1ull << 31)
#define QUARTER_RANGE (1ull << 30)

void czo_enc_init(czo_encoder *e, uint8_t *buf, size_t cap) {
    e->low = 0; e->high = STATE_MASK; e->underflow = 0;
    e->out = buf; e->len = 0; e->cap = cap; e->cur = 0; e->bit_pos = 7; e->overflow = 0;
}

/* arith_coder.rs:51-62 -- MSB-first packing */
static void enc_emit_bit(czo_encoder *e, int bit) {
    if (bit) e->cur |= (uint8_t)(1u << e->bit_pos);
    e->bit_pos -= 1;
    if (e->bit_pos < 0) {
        if (e->len < e->cap) e->out[e->len] = e->cur; else e->overflow = 1;
        e->len++;
        e->cur = 0;
        e->bit_pos = 7;
    }
}

/* arith_coder.rs:66-73 */
static void enc_emit_plus_underflow(czo_encoder *e, int bit) {
    enc_emit_bit(e, bit);
    for (uint32_t i = 0; i < e->underflow; i++) enc_emit_bit(e, bit ^ 1);
    e->underflow = 0;
}

/* arith_coder.rs:101-119 */
static void enc_renorm(czo_encoder *e) {
    for (;;) {
        if (((e->low ^ e->high) & HALF_RANGE) == 0) {
            enc_emit_plus_underflow(e, (int)((e->low >> 31) & 1));
            e->low = (e->low << 1) & STATE_MASK;
            e->high = ((e->high << 1) & STATE_MASK) | 1;
        } else if ((e->low & ~e->high & QUARTER_RANGE) != 0) {
            e->underflow += 1;
            e->low = ((e->low << 1) ^ HALF_RANGE) & STATE_MASK;
            e->high = (((e->high ^ HALF_RANGE) << 1) | HALF_RANGE | 1) & STATE_MASK;
        } else {
            break;
        }
    }
}

void czo_enc_encode_range(czo_encoder *e, uint32_t lo, uint32_t hi, uint32_t total) {
    uint64_t range = e->high - e->low + 1;
    e->high = e->low + ((uint64_t)hi * range / total) - 1;
    e->low = e->low + ((uint64_t)lo * range / total);
    enc_renorm(e);
}

/* arith_coder.rs:80-98 */
void czo_enc_encode(czo_encoder *e, const uint32_t *cum, int V, int sym) {
    uint32_t hi = cum[sym];
    uint32_t lo = sym > 0 ? cum[sym - 1] : 0;
    czo_enc_encode_range(e, lo, hi, cum[V - 1]);
}

/* arith_coder.rs:122-130 */
void czo_enc_finish(czo_encoder *e) {
    enc_emit_bit(e, 1);
    if (e->bit_pos < 7) {
        if (e->len < e->cap) e->out[e->len] = e->cur; else e->overflow = 1;
        e->len++;
    }
}

/* arith_coder.rs:176-190 -- reads past the end give 0 */
static int dec_read_bit(czo_decoder *d) {
    if (d->byte_pos >= d->len) return 0;
    int bit = (d->in[d->byte_pos] >> d->bit_pos) & 1;
    d->bit_pos -= 1;
    if (d->bit_pos < 0) { d->byte_pos++; d->bit_pos = 7; }
    return bit;
}

void czo_dec_init(czo_decoder *d, const uint8_t *in, size_t len) {
    d->low = 0; d->high = STATE_MASK; d->code = 0;
    d->in = in; d->len = len; d->byte_pos = 0; d->bit_pos = 7;
    for (int i = 0; i < 32; i++) d->code = (d->code << 1) | (uint64_t)dec_read_bit(d);
}

/* arith_coder.rs:195-264 */
int czo_dec_decode(czo_decoder *d, const uint32_t *cum, int V) {
    uint64_t total = cum[V - 1];
    uint64_t range = d->high - d->low + 1;
    uint64_t offset = d->code - d->low;
    uint64_t value = ((offset + 1) * total - 1) / range;
    uint32_t v32 = (uint32_t)value;
    int lo = 0, hi = V;
    while (lo < hi) {   /* arith_coder.rs:225-241 */
        int mid = (lo + hi) / 2;
        if (v32 < cum[mid]) hi = mid; else lo = mid + 1;
    }
    int sym = lo < V - 1 ? lo : V - 1;
    uint64_t sh = cum[sym];
    uint64_t sl = sym > 0 ? cum[sym - 1] : 0;
    d->high = d->low + (sh * range / total) - 1;
    d->low = d->low + (sl * range / total);
    for (;;) {
        if (((d->low ^ d->high) & HALF_RANGE) == 0) {
            d->low = (d->low << 1) & STATE_MASK;
            d->high = ((d->high << 1) & STATE_MASK) | 1;
            d->code = ((d->code << 1) & STATE_MASK) | (uint64_t)dec_read_bit(d);
        } else if ((d->low & ~d->high & QUARTER_RANGE) != 0) {
            d->low = ((d->low << 1) ^ HALF_RANGE) & STATE_MASK;
            d->high = (((d->high ^ HALF_RANGE) << 1) | HALF_RANGE | 1) & STATE_MASK;
            d->code = (d->code & HALF_RANGE) | ((d->code << 1) & (STATE_MASK >> 1)) |
                      (uint64_t)dec_read_bit(d);
        } else {
            break;
        }
    }
    return sym;
}

/* ------------------------------------------------------------------------ */
/* chunk drivers (main.rs:206-238, 377-396), threaded over chunks like rayon */
/* ------------------------------------------------------------------------ */

typedef struct {
    const czo_model *m;
    const uint32_t *tokens;
    const uint64_t *starts;
    uint32_t n_chunks;
    uint8_t *out;
    uint64_t slot_cap;
    uint32_t *out_lens;
    const uint8_t *data;
    const uint32_t *n_tokens;
    const uint64_t *tok_offsets;
    uint32_t *out_tokens;
    volatile int next;
    volatile int status;
    pthread_mutex_t mu;
} job_t;

static int job_take(job_t *j) {
    pthread_mutex_lock(&j->mu);
    int c = j->next;
    if (c < (int)j->n_chunks) j->next = c + 1;
    pthread_mutex_unlock(&j->mu);
    return c < (int)j->n_chunks ? c : -1;
}

static void job_fail(job_t *j) {
    pthread_mutex_lock(&j->mu);
    j->status = -1;
    pthread_mutex_unlock(&j->mu);
}

static void *compress_worker(void *arg) {
    job_t *j = (job_t *)arg;
    const czo_model *m = j->m;
    int8_t *kv = (int8_t *)calloc(czo_kv_bytes(m), 1);
    int32_t *logits = (int32_t *)malloc(sizeof(int32_t) * (size_t)m->vocab);
    uint32_t *cum = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)m->vocab);
    int c;
    while ((c = job_take(j)) >= 0) {
        const uint32_t *tk = j->tokens + j->starts[c];
        int n = (int)(j->starts[c + 1] - j->starts[c]);
        czo_encoder e;
        czo_enc_init(&e, j->out + (size_t)c * j->slot_cap, j->slot_cap);
        int bad = n > m->context_length || n > m->max_seq_len;
        for (int i = 0; i < n && !bad; i++) {
            uint32_t prev = i == 0 ? CZO_BOS : tk[i - 1];
            if (prev >= (uint32_t)m->vocab || tk[i] >= (uint32_t)m->vocab) { bad = 1; break; }
            czo_forward(m, kv, prev, i, logits);
            czo_build_cumfreqs(logits, m->vocab, m->exp2_lut, m->coef_q24, m->target_total, cum);
            czo_enc_encode(&e, cum, m->vocab, (int)tk[i]);
        }
        czo_enc_finish(&e);
        j->out_lens[c] = (uint32_t)e.len;
        if (bad || e.overflow) job_fail(j);
    }
    free(kv); free(logits); free(cum);
    return NULL;
}

static void *decompress_worker(void *arg) {
    job_t *j = (job_t *)arg;
    const czo_model *m = j->m;
    int8_t *kv = (int8_t *)calloc(czo_kv_bytes(m), 1);
    int32_t *logits = (int32_t *)malloc(sizeof(int32_t) * (size_t)m->vocab);
    uint32_t *cum = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)m->vocab);
    int c;
    while ((c = job_take(j)) >= 0) {
        int n = (int)j->n_tokens[c];
        uint32_t *dst = j->out_tokens + j->tok_offsets[c];
        if (n > m->context_length || n > m->max_seq_len) { job_fail(j); continue; }
        czo_decoder d;
        czo_dec_init(&d, j->data + j->starts[c], (size_t)(j->starts[c + 1] - j->starts[c]));
        for (int i = 0; i < n; i++) {
            uint32_t prev = i == 0 ? CZO_BOS : dst[i - 1];
            czo_forward(m, kv, prev, i, logits);
            czo_build_cumfreqs(logits, m->vocab, m->exp2_lut, m->coef_q24, m->target_total, cum);
            dst[i] = (uint32_t)czo_dec_decode(&d, cum, m->vocab);
        }
    }
    free(kv); free(logits); free(cum);
    return NULL;
}

static int run_pool(job_t *j, void *(*fn)(void *), int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > (int)j->n_chunks) nthreads = j->n_chunks > 0 ? (int)j->n_chunks : 1;
    pthread_mutex_init(&j->mu, NULL);
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
    for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, fn, j);
    fn(j);
    for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
    free(th);
    pthread_mutex_destroy(&j->mu);
    return j->status;
}

int czo_compress_chunks(const czo_model *m, const uint32_t *tokens, const uint64_t *chunk_starts,
                        uint32_t n_chunks, uint8_t *out, uint64_t slot_cap, uint32_t *out_lens,
                        int nthreads) {
    if (czo_model_check(m) != 0) return -2;
    job_t j;
    memset(&j, 0, sizeof(j));
    j.m = m; j.tokens = tokens; j.starts = chunk_starts; j.n_chunks = n_chunks;
    j.out = out; j.slot_cap = slot_cap; j.out_lens = out_lens;
    return run_pool(&j, compress_worker, nthreads);
}

int czo_decompress_chunks(const czo_model *m, const uint8_t *data, const uint64_t *data_starts,
                          const uint32_t *n_tokens, uint32_t n_chunks, uint32_t *out_tokens,
                          int nthreads) {
    if (czo_model_check(m) != 0) return -2;
    job_t j;
    memset(&j, 0, sizeof(j));
    uint64_t *offs = (uint64_t *)malloc(sizeof(uint64_t) * ((size_t)n_chunks + 1));
    offs[0] = 0;
    for (uint32_t c = 0; c < n_chunks; c++) offs[c + 1] = offs[c] + n_tokens[c];
    j.m = m; j.data = data; j.starts = data_starts; j.n_tokens = n_tokens; j.n_chunks = n_chunks;
    j.tok_offsets = offs; j.out_tokens = out_tokens;
    int st = run_pool(&j, decompress_worker, nthreads);
    free(offs);
    return st;
}

/* Same computation as the compress driver for one chunk, keeping intermediates. */
void czo_chunk_trace(const czo_model *m, const uint32_t *tokens, int n, int32_t *logits,
                     uint32_t *lohi, int8_t *attn, int8_t *final_in) {
    const int d = m->d_model, V = m->vocab;
    int8_t *kv = (int8_t *)calloc(czo_kv_bytes(m), 1);
    int32_t *lg = (int32_t *)malloc(sizeof(int32_t) * (size_t)V);
    uint32_t *cum = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)V);
    for (int i = 0; i < n; i++) {
        uint32_t prev = i == 0 ? CZO_BOS : tokens[i - 1];
        forward_impl(m, kv, prev, i, lg, attn ? attn + (size_t)i * m->n_layers * d : NULL,
                     final_in ? final_in + (size_t)i * d : NULL);
        if (logits) memcpy(logits + (size_t)i * V, lg, sizeof(int32_t) * (size_t)V);
        czo_build_cumfreqs(lg, V, m->exp2_lut, m->coef_q24, m->target_total, cum);
        if (lohi) {
            uint32_t t = tokens[i];
            lohi[2 * i] = t > 0 ? cum[t - 1] : 0;
            lohi[2 * i + 1] = cum[t];
        }
    }
    free(kv); free(lg); free(cum);
}
