/*
 * zonos2_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Plain-C restatement of zonos2.cpp's per-decode-step output path.  Each
 * function cites the reference file:line it restates.  Built with
 * -ffp-contract=off so every f32 operation rounds exactly where the
 * reference's (non-FMA, non-fast-math) build rounds.
 *
 * Where the restatement deliberately differs from the reference:
 *   - equal probabilities are ordered by ascending token id; the reference's
 *     std::sort (src/zonos2_generate.cpp:51-52) leaves their order to
 *     libstdc++'s introsort.  diag->tie marks rows where that matters.
 *   - exp_mode 1 uses a correctly rounded exp; the reference's expf (glibc)
 *     is misrounded by one ulp on about 1e-4 of its inputs in [-104, 0].
 * Repetition penalty, masks and per-stream generators do not exist in the
 * reference; they follow the build's written definition in prologue.h.
 */
#include "zonos2_oracle.h"
#include "prologue.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- Xoshiro256** : src/zonos2_generate.cpp:11-33 ---------------------- */

static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t orc_rng_next(uint64_t st[4])
{
    /* output scrambler and state transition: src/zonos2_generate.cpp:20-31 */
    const uint64_t out = rotl64(st[1] * 5u, 7) * 9u;
    const uint64_t t = st[1] << 17;
    st[2] ^= st[0];
    st[3] ^= st[1];
    st[1] ^= st[2];
    st[0] ^= st[3];
    st[2] ^= t;
    st[3] = rotl64(st[3], 45);
    return out;
}

void orc_rng_seed(uint64_t seed, uint64_t st[4])
{
    /* seed xor four fixed words, then 20 discarded outputs: :13-19 */
    static const uint64_t salt[4] = {0x9E3779B97F4A7C15ULL, 0xBF58476D1CE4E5B9ULL,
                                     0x94D049BB133111EBULL, 0x3243F6A8885A308DULL};
    for (int i = 0; i < 4; i++) st[i] = seed ^ salt[i];
    for (int i = 0; i < 20; i++) (void)orc_rng_next(st);
}

float orc_randf(uint64_t st[4])
{
    /* 53-bit double in [0,1), then narrowed to float (may round to 1.0f): :32 */
    const double d = (double)(orc_rng_next(st) >> 11) * 0x1.0p-53;
    return (float)d;
}

void orc_rng_seed_streams(uint64_t seed, int n, uint64_t *st)
{
    for (int s = 0; s < n; s++) orc_rng_seed(seed + (uint64_t)s, st + 4 * (size_t)s);
}

float orc_exp(float x, int exp_mode)
{
    return exp_mode ? (float)exp((double)x) : expf(x);
}

/* ---- sample_token : src/zonos2_generate.cpp:36-93 ------------------------ */

typedef struct {
    float p;
    int idx;
} orc_cand;

static int cand_order(const void *a, const void *b)
{
    const orc_cand *x = (const orc_cand *)a, *y = (const orc_cand *)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}

static float sum_prefix(const orc_cand *c, int n)
{
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += c[i].p;
    return s;
}

static inline float fminabs(float m, float v)
{
    v = fabsf(v);
    return v < m ? v : m;
}

int orc_sample_token_r(float r, const float *logits, int vocab, float temp, int top_k,
                       float top_p, float min_p, int exp_mode, orc_diag *diag)
{
    orc_cand *c = (orc_cand *)malloc(sizeof(orc_cand) * (size_t)vocab);
    float margin = INFINITY;
    int tie = 0;

    /* :41-42 running max from -1e9 (a NaN never replaces it) */
    float mx = -1e9f;
    for (int i = 0; i < vocab; i++)
        if (mx < logits[i]) mx = logits[i];

    /* :44-49 unnormalised probabilities, index-order sum */
    float sum = 0.0f;
    for (int i = 0; i < vocab; i++) {
        c[i].p = orc_exp((logits[i] - mx) / temp, exp_mode);
        c[i].idx = i;
        sum += c[i].p;
    }

    /* :51-52 descending probability (ties: ascending id) */
    qsort(c, (size_t)vocab, sizeof(orc_cand), cand_order);

    int n = vocab;
    /* :55-59 top-k */
    if (top_k > 0 && top_k < vocab) {
        n = top_k;
        if (c[n - 1].p == c[n].p) tie = 1;
        if (c[n - 1].p > 0.0f) margin = fminf(margin, (c[n - 1].p - c[n].p) / c[n - 1].p);
        sum = sum_prefix(c, n);
    }
    const int n_topk = n;

    /* :62-73 top-p: cut right after the first prefix whose mass reaches top_p */
    if (top_p < 1.0f) {
        float cum = 0.0f;
        int cut = 0;
        for (int i = 0; i < n; i++) {
            const float prev = cum;
            cum += c[i].p / sum;
            cut = i + 1;
            if (cum >= top_p) {
                margin = fminabs(margin, cum - top_p);
                margin = fminabs(margin, prev - top_p);
                break;
            }
        }
        if (cut < n && c[cut - 1].p == c[cut].p) tie = 1;
        n = cut;
        sum = sum_prefix(c, n);
    }

    /* :76-84 min-p: longest prefix with p/sum >= (p0/sum)*min_p */
    if (min_p > 0.0f && n > 0) {
        const float thresh = (c[0].p / sum) * min_p;
        int j = 0;
        while (j < n && c[j].p / sum >= thresh) j++;
        if (j < n) margin = fminabs(margin, (c[j].p / sum - thresh) / (thresh > 0 ? thresh : 1.0f));
        if (j > 0) margin = fminabs(margin, (c[j - 1].p / sum - thresh) / (thresh > 0 ? thresh : 1.0f));
        n = j;
        sum = sum_prefix(c, n);
    }

    /* :86-92 one uniform, CDF walk, fall through to the last candidate */
    int tok = -1, pos = -1;
    float cum = 0.0f;
    for (int i = 0; i < n; i++) {
        const float prev = cum;
        cum += c[i].p / sum;
        if (r <= cum) {
            tok = c[i].idx;
            pos = i;
            margin = fminabs(margin, r - cum);
            margin = fminabs(margin, r - prev);
            break;
        }
    }
    if (pos < 0 && n > 0) {
        tok = c[n - 1].idx;
        margin = fminabs(margin, r - cum);
    }
    const int at = pos >= 0 ? pos : n - 1;
    if (at >= 0) {
        if (at > 0 && c[at - 1].p == c[at].p) tie = 1;
        if (at + 1 < vocab && c[at + 1].p == c[at].p) tie = 1;
    }
    if (diag) {
        diag->token = tok;
        diag->n_topk = n_topk;
        diag->n_final = n;
        diag->pos = pos;
        diag->r = r;
        diag->margin = margin;
        diag->tie = tie;
    }
    free(c);
    return tok;
}

int orc_sample_token(uint64_t st[4], const float *logits, int vocab, float temp, int top_k,
                     float top_p, float min_p, int exp_mode, orc_diag *diag)
{
    const float r = orc_randf(st);
    return orc_sample_token_r(r, logits, vocab, temp, top_k, top_p, min_p, exp_mode, diag);
}

/* ---- one row with the build-defined prologue (prologue.h) -------------- */

int orc_sample_row(float r, const float *logits, int vocab, const orc_params *p,
                   const int32_t *hist, int hist_len, const uint32_t *allow,
                   int force_pad, int exp_mode, orc_diag *diag, int *flags)
{
    float *l = (float *)malloc(sizeof(float) * (size_t)vocab);
    int f = 0;
    const int live = zonos2_row_prologue(logits, vocab, p->repetition_penalty, hist, hist_len,
                                         allow, force_pad, p->pad_id, l, &f);
    int tok;
    if (!live) {
        tok = p->pad_id;
        if (diag) {
            memset(diag, 0, sizeof(*diag));
            diag->token = tok;
            diag->pos = -1;
            diag->r = r;
            diag->margin = INFINITY;
        }
    } else {
        tok = orc_sample_token_r(r, l, vocab, p->temperature, p->top_k, p->top_p, p->min_p,
                                 exp_mode, diag);
    }
    free(l);
    if (flags) *flags = f;
    return tok;
}

int orc_step(const float *logits, int n_streams, int n_cb, int vocab, long row_stride,
             const orc_params *p, uint64_t *rng, int32_t *hist, int hist_len, int hist_pos,
             const uint32_t *allow, int allow_words, int delay_step, int32_t *codes,
             int32_t *flags, int exp_mode, orc_diag *diags, int nthreads)
{
    if (n_streams < 0 || n_cb <= 0 || vocab <= 0) return -1;
    if (hist_len > 0 && (hist_pos < 0 || hist_pos >= hist_len)) return -1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads)
#endif
    for (int s = 0; s < n_streams; s++) {
        uint64_t *st = rng + 4 * (size_t)s;
        for (int c = 0; c < n_cb; c++) {
            const size_t row = (size_t)s * (size_t)n_cb + (size_t)c;
            const float r = orc_randf(st); /* codebook order: src/zonos2_generate.cpp:259-267 */
            int32_t *h = hist ? hist + row * (size_t)hist_len : NULL;
            const uint32_t *a = allow ? allow + (size_t)s * (size_t)allow_words : NULL;
            const int force = delay_step >= 0 && delay_step < c;
            int f = 0;
            const int tok = orc_sample_row(r, logits + row * (size_t)row_stride, vocab, p, h,
                                           hist_len, a, force, exp_mode,
                                           diags ? diags + row : NULL, &f);
            codes[row] = tok;
            if (flags) flags[row] = f;
            if (h && hist_len > 0) h[hist_pos] = tok;
        }
    }
    return 0;
}

/* ---- output head + softcap : src/zonos2_model.cpp:200-216, :687-703 ------ */

void orc_head_softcap(const float *W, int rows_per_cb, int n_cb, int vocab, int dim,
                      const float *h, int batch, float softcap, float *out, int nthreads)
{
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads)
#endif
    for (int b = 0; b < batch; b++)
        for (int c = 0; c < n_cb; c++) {
            const float *x = h + (size_t)b * (size_t)dim;
            float *o = out + ((size_t)b * (size_t)n_cb + (size_t)c) * (size_t)vocab;
            for (int v = 0; v < vocab; v++) {
                const float *w = W + ((size_t)c * (size_t)rows_per_cb + (size_t)v) * (size_t)dim;
                float s = 0.0f;
                for (int i = 0; i < dim; i++) s += x[i] * w[i];
                o[v] = softcap > 0.0f ? softcap * tanhf(s / softcap) : s;
            }
        }
}


/* The output RMSNorm applied to the hidden states before the head
 * (src/zonos2_model.cpp:684-685 calling rms_norm_per_token, :19-35): per row,
 * the f32 sum of squares in index order, rms = sqrt(ss / dim + eps), rcp =
 * 1 / rms, then x * rcp (times the scale weight when there is one).  In place. */
void orc_out_norm(float *x, int dim, int n_rows, float eps, const float *weight)
{
    for (int t = 0; t < n_rows; t++) {
        float *xt = x + (size_t)t * (size_t)dim;
        float ss = 0.0f;
        for (int d = 0; d < dim; d++) ss += xt[d] * xt[d];
        const float rms = sqrtf(ss / (float)dim + eps);
        const float rcp = 1.0f / rms;
        if (weight)
            for (int d = 0; d < dim; d++) xt[d] = xt[d] * rcp * weight[d];
        else
            for (int d = 0; d < dim; d++) xt[d] *= rcp;
    }
}

/* Classifier-free guidance on softcapped logits, as the reference blends its
 * prefill logits (src/zonos2_generate.cpp:178-183): out = u + s * (c - u). */
void orc_cfg_blend(const float *cond, const float *uncond, long n, float scale, float *out)
{
    for (long i = 0; i < n; i++) out[i] = uncond[i] + scale * (cond[i] - uncond[i]);
}


/* embedding_sum (src/zonos2_model.cpp:116-151): the input embedding of each
 * frame, out[t] = sum over codebooks cb (in order) of cb_tables[cb][id_cb]
 * (ids outside [0, audio_vocab) add nothing), then the text column: a text
 * token (< text_vocab) adds 5 x its row, the padding id (== text_vocab) adds its
 * row once, anything else nothing.  Tables are row-major [rows][dim]. */
void orc_embed_frames(const float *cb_tables, const float *text_table, int n_cb, int audio_vocab,
                      int text_vocab, int dim, const int32_t *ids, int n, float *out)
{
    const int fw = n_cb + 1;
    for (int t = 0; t < n; t++) {
        float *o = out + (size_t)t * (size_t)dim;
        for (int d = 0; d < dim; d++) o[d] = 0.0f;
        for (int cb = 0; cb < n_cb; cb++) {
            const int tid = ids[(size_t)t * fw + cb];
            if (tid >= 0 && tid < audio_vocab) {
                const float *row = cb_tables + ((size_t)cb * audio_vocab + tid) * (size_t)dim;
                for (int d = 0; d < dim; d++) o[d] += row[d];
            }
        }
        const int tid = ids[(size_t)t * fw + n_cb];
        if (tid >= 0 && tid < text_vocab) {
            const float *row = text_table + (size_t)tid * (size_t)dim;
            for (int d = 0; d < dim; d++) o[d] += row[d] * 5.0f;
        } else if (tid == text_vocab) {
            const float *row = text_table + (size_t)tid * (size_t)dim;
            for (int d = 0; d < dim; d++) o[d] += row[d];
        }
    }
}

/* shear_up (scripts/dac_decode.py:23-30): undo the delay pattern of n_frames
 * frames of n_cb codes, out[t][j] = codes[t + j][j] while t + j < n_frames,
 * pad elsewhere. */
void orc_shear_up(const int32_t *codes, int n_frames, int n_cb, int32_t pad, int32_t *out)
{
    for (int t = 0; t < n_frames; t++)
        for (int j = 0; j < n_cb; j++)
            out[(size_t)t * n_cb + j] =
                t + j < n_frames ? codes[(size_t)(t + j) * n_cb + j] : pad;
}
