/*
 * zonos2_oracle.h -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * CPU restatement of zonos2.cpp's per-decode-step output path: the 9-codebook
 * output head with its tanh softcap, the Xoshiro256** generator and the
 * sampler.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs load this code.  The CUDA library never links it.
 *
 * Parity pin: the restatement is checked against the reference itself,
 * compiled unmodified from its own sources into oracle/_ref/ (see Makefile),
 * and against golden vectors generated from that build (tests/golden/).
 */
#ifndef ZONOS2_ORACLE_H
#define ZONOS2_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Row flags (same bit meaning as the CUDA library's ZONOS2CU_FLAG_*). */
#define ORC_FLAG_ALL_MASKED 1 /* no logit >= -1e9 survived: token = pad id  */
#define ORC_FLAG_NONFINITE  2 /* a NaN / +inf logit was treated as masked   */

/* Sampler knobs.  Field meaning follows Zonos2GenParams (src/zonos2.h:244-254). */
typedef struct {
    float temperature;
    int   top_k;
    float top_p;
    float min_p;
    float repetition_penalty; /* build-defined; 1.0 = off */
    int   pad_id;             /* token forced by the delay-pattern mask / all-masked rows */
} orc_params;

/* Per-row diagnostics used by the tests to classify GPU/oracle mismatches. */
typedef struct {
    int   token;
    int   n_topk;      /* candidates after top-k                                 */
    int   n_final;     /* candidates the draw walked over                        */
    int   pos;         /* position of the drawn token in the sorted list, -1 = fell through to back() */
    float r;           /* the uniform                                             */
    float margin;      /* smallest distance of r / top_p / min-p threshold to a decision boundary */
    int   tie;         /* 1 if an equal-probability group touches a cut or the drawn position */
} orc_diag;

/* Xoshiro256** with the reference's seeding (src/zonos2_generate.cpp:11-33). */
void     orc_rng_seed(uint64_t seed, uint64_t st[4]);
uint64_t orc_rng_next(uint64_t st[4]);
float    orc_randf(uint64_t st[4]);
/* Stream s of a batch is seeded with seed + s (build definition for B > 1). */
void     orc_rng_seed_streams(uint64_t seed, int n, uint64_t *st);

/* exp_mode: 0 = libm expf (what the reference calls), 1 = correctly rounded
 * (float)exp((double)x), which is what the CUDA sampler computes. */
float orc_exp(float x, int exp_mode);

/* sample_token (src/zonos2_generate.cpp:36-93) with the uniform passed in and
 * equal probabilities ordered by ascending token id. */
int orc_sample_token_r(float r, const float *logits, int vocab, float temp, int top_k,
                       float top_p, float min_p, int exp_mode, orc_diag *diag);
/* Same, drawing r from the generator after filtering, as the reference does. */
int orc_sample_token(uint64_t st[4], const float *logits, int vocab, float temp, int top_k,
                     float top_p, float min_p, int exp_mode, orc_diag *diag);

/* One row with the build-defined prologue: repetition penalty over the
 * history window, allow bitmask, delay-pattern forcing, non-finite guard. */
int orc_sample_row(float r, const float *logits, int vocab, const orc_params *p,
                   const int32_t *hist, int hist_len, const uint32_t *allow,
                   int force_pad, int exp_mode, orc_diag *diag, int *flags);

/* One decode step over [n_streams, n_cb] rows (row r at logits + r*row_stride).
 * rng [n_streams][4] advanced by n_cb draws (codebook order), history ring
 * [n_streams][n_cb][hist_len] read then appended at hist_pos, allow
 * [n_streams][allow_words] or NULL, delay_step < 0 disables the delay mask. */
int orc_step(const float *logits, int n_streams, int n_cb, int vocab, long row_stride,
             const orc_params *p, uint64_t *rng, int32_t *hist, int hist_len, int hist_pos,
             const uint32_t *allow, int allow_words, int delay_step, int32_t *codes,
             int32_t *flags, int exp_mode, orc_diag *diags, int nthreads);

/* Output head + softcap (src/zonos2_model.cpp:200-216, :687-703) for the
 * sampled rows: out[b][c][v] = cap*tanhf(dot(h[b], W[c*rows_per_cb+v]) / cap),
 * sequential f32 dot in input order. */
void orc_head_softcap(const float *W, int rows_per_cb, int n_cb, int vocab, int dim,
                      const float *h, int batch, float softcap, float *out, int nthreads);

/* rms_norm_per_token (src/zonos2_model.cpp:19-35) over n_rows rows, in place;
 * weight may be NULL. */
void orc_out_norm(float *x, int dim, int n_rows, float eps, const float *weight);

/* out = uncond + scale * (cond - uncond), element by element
 * (src/zonos2_generate.cpp:178-183). */
void orc_cfg_blend(const float *cond, const float *uncond, long n, float scale, float *out);

/* embedding_sum (src/zonos2_model.cpp:116-151) of n frames ids [n][n_cb+1]:
 * cb_tables [n_cb][audio_vocab][dim], text_table [text_vocab+1][dim], out [n][dim]. */
void orc_embed_frames(const float *cb_tables, const float *text_table, int n_cb, int audio_vocab,
                      int text_vocab, int dim, const int32_t *ids, int n, float *out);

/* shear_up (scripts/dac_decode.py:23-30) of codes [n_frames][n_cb]. */
void orc_shear_up(const int32_t *codes, int n_frames, int n_cb, int32_t pad, int32_t *out);

#ifdef __cplusplus
}
#endif
#endif
