/*
 * czoracle.h -- CPU oracle for the compress-zip model-plus-coder path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * Rust crate (the rust/src files of carsonpo/compress-zip), used by the test suite,
 * by __graft_entry__.smoke() and by bench.py's cpu_baseline / reference arm as
 * the checker and the CPU baseline.  The product (libczg.so) never links,
 * loads or calls it.
 *
 * Every function cites the reference file:line whose semantics it follows
 * (Rust release-build semantics: integer overflow wraps).
 */
#ifndef CZORACLE_H
#define CZORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CZO_MAX_LAYERS 64
#define CZO_HEAD_DIM 64
#define CZO_HALF_DIM 32
#define CZO_BOS 1022u

/* ---- primitives (rust/src/primitives.rs) ---- */
int8_t czo_clamp_i8(int32_t x);                               /* primitives.rs:9-11   */
int32_t czo_sra_rne_s32(int32_t v, uint32_t sh);              /* primitives.rs:18-42  */
int32_t czo_sra_rne_s64_to_s32(int64_t v, uint32_t sh);       /* primitives.rs:49-73  */
uint32_t czo_udiv_rne_u32(uint32_t n, uint32_t d);            /* primitives.rs:80-97  */
int32_t czo_div_rne_s32_by_u64(int32_t num, uint64_t den);    /* primitives.rs:163-185 */
uint32_t czo_isqrt32(uint32_t x);                             /* primitives.rs:192-213 */

/* exp weight in Q16 from a non-positive difference.  The attention exp
 * (lut.rs:213-235) and the CDF exp (softmax_cdf.rs:55-77) are the same
 * formula with different coefficients. */
uint16_t czo_exp_q16(int32_t neg_x, const uint16_t *lut, uint32_t coef_q24);

int32_t czo_inv_rms_q15(int32_t mean_sq);                     /* rmsnorm.rs:14-30 */
void czo_rmsnorm_i8(const int8_t *x, const int8_t *w, int d, int32_t eps, int8_t *out); /* rmsnorm.rs:40-75 */
void czo_linear_i8_i32(const int8_t *x, const int8_t *W, int in_dim, int out_dim, int32_t *y); /* linear.rs:12-31 */
void czo_requant(const int32_t *x, int n, int32_t mult, int8_t shift, int8_t *out); /* model.rs:280-300 */
void czo_reglu(const int8_t *x, int d_ff, int8_t *out);       /* reglu.rs:20-46 */
void czo_rope_k(int8_t *x, const int16_t *cos_t, const int16_t *sin_t, int pos); /* attention.rs:29-50 */
void czo_rope_q(int8_t *x, const int16_t *cos_t, const int16_t *sin_t, int pos); /* attention.rs:53-83 */
uint32_t czo_attn_coef_q24(void);                             /* attention.rs:17-19 */

/* Attention of one chunk's positions 0..n-1, H query heads sharing one K/V
 * head (attention.rs:162-289 run for pos = 0..n-1).  q: [n][H][64] and k: [n][64]
 * before RoPE, v: [n][64]; out: [n][H][64].  sink_key may be NULL. */
void czo_attention_seq(const int8_t *q, const int8_t *k, const int8_t *v, int n, int H,
                       const int32_t *score_mult, const int8_t *sink_key, const int16_t *cos_t,
                       const int16_t *sin_t, const uint16_t *lut, int8_t *out);

/* softmax -> inclusive cumulative frequencies (softmax_cdf.rs:85-139) */
void czo_build_cumfreqs(const int32_t *logits, int V, const uint16_t *lut,
                        uint32_t coef_q24, uint32_t target_total, uint32_t *cum);
uint32_t czo_default_coef_q24(void);                          /* softmax_cdf.rs:23-28 */
uint32_t czo_default_target_total(int V);                     /* softmax_cdf.rs:39-46 */

/* ---- model (rust/src/model.rs) ---- */
typedef struct {
    const int8_t *attn_norm, *post_attn_norm, *ffn_norm, *post_ffn_norm;
    const int8_t *qkv_w;   /* [d + 2*n_kv*64, d] */
    const int8_t *out_w;   /* [d, d] */
    const int8_t *up_w;    /* [2*d_ff, d] */
    const int8_t *down_w;  /* [d, d_ff] */
    const int32_t *score_mult; /* [n_heads] */
    const int8_t *sink_key;    /* [64] or NULL */
    int32_t qkv_mult, out_mult, up_mult, down_mult;
    int32_t qkv_shift, out_shift, up_shift, down_shift;
} czo_layer;

typedef struct {
    int32_t vocab, n_layers, n_heads, n_kv_heads, d_model, d_ff, head_dim;
    int32_t max_seq_len, context_length;
    uint32_t coef_q24, target_total;
    int32_t eps_scaled;
    const int8_t *embed;     /* [V, d] */
    const int8_t *final_norm;/* [d] */
    const int8_t *head_w;    /* [V, d] */
    const uint16_t *exp2_lut;/* [256] */
    const int16_t *rope_cos; /* [context_length, 32] */
    const int16_t *rope_sin;
    czo_layer layers[CZO_MAX_LAYERS];
} czo_model;

/* Returns 0 when the model shape is one the reference runs without a panic. */
int czo_model_check(const czo_model *m);

/* KV state for one chunk: n_layers x [max_seq_len][64] K and V. */
size_t czo_kv_bytes(const czo_model *m);

/* One token at one position (model.rs:362-480). kv must hold czo_kv_bytes. */
void czo_forward(const czo_model *m, int8_t *kv, uint32_t token, int pos, int32_t *logits);

/* ---- arithmetic coder (rust/src/arith_coder.rs) ---- */
typedef struct {
    uint64_t low, high;
    uint32_t underflow;
    uint8_t *out;
    size_t len, cap;
    uint8_t cur;
    int bit_pos;
    int overflow;
} czo_encoder;
void czo_enc_init(czo_encoder *e, uint8_t *buf, size_t cap);           /* arith_coder.rs:28-37 */
void czo_enc_encode(czo_encoder *e, const uint32_t *cum, int V, int sym); /* arith_coder.rs:80-98 */
void czo_enc_encode_range(czo_encoder *e, uint32_t lo, uint32_t hi, uint32_t total);
void czo_enc_finish(czo_encoder *e);                                   /* arith_coder.rs:122-130 */

typedef struct {
    uint64_t low, high, code;
    const uint8_t *in;
    size_t len, byte_pos;
    int bit_pos;
} czo_decoder;
void czo_dec_init(czo_decoder *d, const uint8_t *in, size_t len);      /* arith_coder.rs:153-174 */
int czo_dec_decode(czo_decoder *d, const uint32_t *cum, int V);        /* arith_coder.rs:195-222 */

/* ---- chunk drivers (rust/src/main.rs:206-238 and 377-396) ----
 * chunk_starts has n_chunks+1 entries; chunk i is tokens[starts[i]..starts[i+1]).
 * Compressed chunk i is written to out + i*slot_cap, its length to out_lens[i].
 * Returns 0, or -1 when a slot overflowed / an input was out of range. */
int czo_compress_chunks(const czo_model *m, const uint32_t *tokens, const uint64_t *chunk_starts,
                        uint32_t n_chunks, uint8_t *out, uint64_t slot_cap, uint32_t *out_lens,
                        int nthreads);
/* data_starts has n_chunks+1 entries; decoded tokens of chunk i land at
 * out_tokens + (sum of n_tokens[0..i)). */
int czo_decompress_chunks(const czo_model *m, const uint8_t *data, const uint64_t *data_starts,
                          const uint32_t *n_tokens, uint32_t n_chunks, uint32_t *out_tokens,
                          int nthreads);

/* Per-position intermediates of one chunk, for localising a mismatch.
 * Any output pointer may be NULL.  logits: [n][V]; lohi: [n][2] (the coder's
 * sym_low, sym_high); attn: [n][n_layers][d] attention outputs;
 * final_in: [n][d] the final-norm output that feeds the LM head. */
void czo_chunk_trace(const czo_model *m, const uint32_t *tokens, int n, int32_t *logits,
                     uint32_t *lohi, int8_t *attn, int8_t *final_in);

#ifdef __cplusplus
}
#endif
#endif
