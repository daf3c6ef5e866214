/*
 * prologue.h -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Build-defined row prologue shared by the C restatement (zonos2_oracle.c)
 * and the harness around the unmodified reference (ref_harness.cpp).
 *
 * Zonos2GenParams declares repetition_penalty / repetition_window
 * (src/zonos2.h:251-252) but nothing reads them, and the reference has no
 * token masks.  The build defines, per (stream, codebook) row:
 *   1. NaN / +inf logits are masked (-inf) and flagged;
 *   2. every distinct token id in [0, vocab) found in the history window is
 *      penalised once: l > 0 ? l * RN(1/rho) : l * rho;
 *   3. tokens whose allow bit is clear are masked;
 *   4. when the delay-pattern mask is active only pad_id survives;
 *   5. a row with no logit >= -1e9 (the reference's initial running max,
 *      src/zonos2_generate.cpp:41) is "all masked": the sampler returns
 *      pad_id, because the reference's sample_token is undefined there;
 * and the row's uniform is consumed in every case.
 */
#ifndef ZONOS2_PROLOGUE_H
#define ZONOS2_PROLOGUE_H

#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#define PROLOGUE_FLAG_ALL_MASKED 1
#define PROLOGUE_FLAG_NONFINITE 2

/* Writes the masked/penalised row to out[vocab]; returns 1 if the row is live. */
static inline int zonos2_row_prologue(const float *logits, int vocab, float rho,
                                      const int32_t *hist, int hist_len,
                                      const uint32_t *allow, int force_pad, int pad_id,
                                      float *out, int *flags)
{
    int f = 0;
    for (int i = 0; i < vocab; i++) {
        float v = logits[i];
        if (isnan(v) || v == INFINITY) {
            v = -INFINITY;
            f |= PROLOGUE_FLAG_NONFINITE;
        }
        out[i] = v;
    }
    if (hist_len > 0 && rho != 1.0f) {
        unsigned char *seen = (unsigned char *)calloc((size_t)vocab, 1);
        for (int j = 0; j < hist_len; j++) {
            const int t = hist[j];
            if (t >= 0 && t < vocab) seen[t] = 1;
        }
        const float inv = 1.0f / rho;
        for (int i = 0; i < vocab; i++)
            if (seen[i]) out[i] = out[i] > 0.0f ? out[i] * inv : out[i] * rho;
        free(seen);
    }
    if (allow)
        for (int i = 0; i < vocab; i++)
            if (!((allow[i >> 5] >> (i & 31)) & 1u)) out[i] = -INFINITY;
    if (force_pad)
        for (int i = 0; i < vocab; i++)
            if (i != pad_id) out[i] = -INFINITY;
    int live = 0;
    for (int i = 0; i < vocab; i++)
        if (out[i] >= -1e9f) live = 1;
    if (!live) f |= PROLOGUE_FLAG_ALL_MASKED;
    if (flags) *flags = f;
    return live;
}

#endif
