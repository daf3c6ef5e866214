/*
 * ref_harness.cpp -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Compiles the reference's own, unmodified sources for the per-decode-step
 * output path into oracle/_ref/libzonos2_ref.so (recipe: oracle/Makefile,
 * include path = the reference's src/ directory).  The reference's sampler
 * and GEMM are file-static, so they are reached by including the two
 * translation units here and exporting thin C wrappers:
 *   - Xoshiro256                  src/zonos2_generate.cpp:11-33
 *   - sample_token                src/zonos2_generate.cpp:36-93
 *   - linear_forward              src/zonos2_model.cpp:200-216
 * The softcap expression of src/zonos2_model.cpp:692-703 lives inside
 * zonos2_forward (which needs a full checkpoint), so ref_head_softcap applies
 * that one expression itself after the reference's linear_forward.
 * ref_step wraps the unmodified sample_token in the build-defined prologue
 * (prologue.h) and is the CPU baseline timed beside the CUDA path.
 */
#include <cstdint>
#include <cstring>
#include <vector>

#include "zonos2_model.cpp"
#include "zonos2_generate.cpp"

#include "prologue.h"

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

void ref_rng_seed(uint64_t seed, uint64_t out[4])
{
    Xoshiro256 r(seed);
    std::memcpy(out, r.s, sizeof(r.s));
}

uint64_t ref_rng_next(uint64_t st[4])
{
    Xoshiro256 r;
    std::memcpy(r.s, st, sizeof(r.s));
    const uint64_t v = r.next();
    std::memcpy(st, r.s, sizeof(r.s));
    return v;
}

float ref_randf(uint64_t st[4])
{
    Xoshiro256 r;
    std::memcpy(r.s, st, sizeof(r.s));
    const float v = r.randf();
    std::memcpy(st, r.s, sizeof(r.s));
    return v;
}

int ref_sample_token(uint64_t st[4], const float *logits, int vocab, float temp, int top_k,
                     float top_p, float min_p)
{
    Xoshiro256 r;
    std::memcpy(r.s, st, sizeof(r.s));
    const int tok = sample_token(r, logits, vocab, temp, top_k, top_p, min_p);
    std::memcpy(st, r.s, sizeof(r.s));
    return tok;
}

void ref_linear_forward(const float *W, int in_f, int out_f, const float *x, int n_tok,
                        float *out)
{
    linear_forward(W, in_f, out_f, x, n_tok, out);
}

/* The reference's own rms_norm_per_token, in place (weight may be NULL). */
void ref_out_norm(float *x, int dim, int n_rows, float eps, const float *weight)
{
    rms_norm_per_token(x, dim, n_rows, eps, weight);
}

/* The reference's own embedding_sum on tables given as plain arrays
 * (cb_tables [n_cb][audio_vocab][dim], text_table [text_vocab+1][dim]). */
void ref_embed_frames(const float *cb_tables, const float *text_table, int n_cb, int audio_vocab,
                      int text_vocab, int dim, const int32_t *ids, int n, float *out)
{
    Zonos2Weights w;
    w.cfg.dim = dim;
    w.cfg.n_codebooks = n_cb;
    w.cfg.audio_vocab = audio_vocab;
    w.cfg.text_vocab = text_vocab;
    for (int cb = 0; cb < n_cb; cb++)
        w.codebook_embeds[cb].weight.data.assign(cb_tables + (size_t)cb * audio_vocab * dim,
                                                 cb_tables + (size_t)(cb + 1) * audio_vocab * dim);
    w.text_embed.weight.data.assign(text_table, text_table + (size_t)(text_vocab + 1) * dim);
    embedding_sum(w, w.cfg, ids, n, n_cb + 1, out);
}

/* The reference's own codes.bin writer (decode_dac_to_wav writes
 * `stem`.codes.bin); returns 1 on success. */
int ref_write_codes(const char *stem, const int32_t *frames, int n_frames, int n_cb)
{
    std::vector<std::vector<int32_t>> codes((size_t)n_frames);
    for (int t = 0; t < n_frames; t++)
        codes[t].assign(frames + (size_t)t * n_cb, frames + (size_t)(t + 1) * n_cb);
    return decode_dac_to_wav(codes, std::string(stem)) ? 1 : 0;
}

/* W: [n_cb*rows_per_cb, dim]; out: [batch][n_cb][vocab] (the sampled rows). */
void ref_head_softcap(const float *W, int rows_per_cb, int n_cb, int vocab, int dim,
                      const float *h, int batch, float softcap, float *out, int nthreads)
{
    const int out_dim = rows_per_cb * n_cb;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int b = 0; b < batch; b++) {
        std::vector<float> flat((size_t)out_dim);
        linear_forward(W, dim, out_dim, h + (size_t)b * dim, 1, flat.data());
        for (int c = 0; c < n_cb; c++)
            for (int v = 0; v < vocab; v++) {
                float l = flat[(size_t)c * rows_per_cb + v];
                if (softcap > 0) l = softcap * std::tanh(l / softcap);
                out[((size_t)b * n_cb + c) * vocab + v] = l;
            }
    }
}

/* One decode step over [n_streams, n_cb] rows through the unmodified
 * sample_token; same argument meaning as orc_step in zonos2_oracle.h. */
int ref_step(const float *logits, int n_streams, int n_cb, int vocab, long row_stride,
             float temp, int top_k, float top_p, float min_p, float rho, int pad_id,
             uint64_t *rng, int32_t *hist, int hist_len, int hist_pos, const uint32_t *allow,
             int allow_words, int delay_step, int32_t *codes, int32_t *flags, int nthreads)
{
    if (n_streams < 0 || n_cb <= 0 || vocab <= 0) return -1;
    if (hist_len > 0 && (hist_pos < 0 || hist_pos >= hist_len)) return -1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
    {
        std::vector<float> row((size_t)vocab);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (int s = 0; s < n_streams; s++) {
            Xoshiro256 r;
            std::memcpy(r.s, rng + 4 * (size_t)s, sizeof(r.s));
            for (int c = 0; c < n_cb; c++) {
                const size_t ridx = (size_t)s * n_cb + c;
                int32_t *h = hist ? hist + ridx * (size_t)hist_len : nullptr;
                const uint32_t *a = allow ? allow + (size_t)s * allow_words : nullptr;
                const int force = delay_step >= 0 && delay_step < c;
                int f = 0;
                const int live = zonos2_row_prologue(logits + ridx * (size_t)row_stride, vocab,
                                                     rho, h, hist_len, a, force, pad_id,
                                                     row.data(), &f);
                int tok;
                if (live) {
                    tok = sample_token(r, row.data(), vocab, temp, top_k, top_p, min_p);
                } else {
                    (void)r.randf(); /* the row's uniform is consumed either way */
                    tok = pad_id;
                }
                codes[ridx] = tok;
                if (flags) flags[ridx] = f;
                if (h && hist_len > 0) h[hist_pos] = tok;
            }
            std::memcpy(rng + 4 * (size_t)s, r.s, sizeof(r.s));
        }
    }
    return 0;
}

int ref_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

} /* extern "C" */
