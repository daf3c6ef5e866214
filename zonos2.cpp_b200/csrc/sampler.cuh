// sampler.cuh -- launcher interface of the fused sampler kernel (sampler.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace z2 {

constexpr int kSamplerVocabMax = 1024;
constexpr int kSamplerCbMax = 16;

struct SampleArgs {
    const float *logits;
    long long row_stride;
    int n_streams, n_cb, vocab;
    float temperature, top_p, min_p, rho, inv_rho;
    double inv_temp;         // RN_f64(1 / temperature): (l - max) / T as one f64 multiply
    int top_k, pad_id;
    uint64_t *rng;           // [n_streams][4]
    int32_t *hist;           // [n_streams][n_cb][hist_len] or nullptr
    int hist_len, hist_pos;
    const uint32_t *allow;   // [n_streams][allow_words] or nullptr
    int allow_words;
    int delay_step;
    int32_t *codes;          // [n_streams][n_cb]
    int32_t *flags;          // [n_streams][n_cb] or nullptr
    int vec_logits;          // rows 16-byte aligned and vocab % 4 == 0
    int vec_hist;            // history rows 16-byte aligned and hist_len % 4 == 0
    // Incremental history (the decode context): per row, how often each token
    // occurs in the ring and a bitmap of the tokens that occur.  When set, the
    // penalty reads the bitmap instead of scanning the ring, and the kernel
    // updates counts and bitmap for the token it evicts and the one it appends.
    uint16_t *counts;        // [n_streams][n_cb][vocab] or nullptr
    uint32_t *presence;      // [n_streams][n_cb][allow_words] or nullptr
};

// Enqueues one sampling step; returns the cudaError_t of the launch.
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t stream);

// Shared memory bytes the kernel uses for n_cb codebooks per CTA.
size_t sample_smem_bytes(int n_cb);

// Rebuilds counts / presence of `rows` history rings ([rows][hist_len] i32,
// entries outside [0, vocab) ignored).  hist_len <= 65535.
cudaError_t launch_history_index(const int32_t *hist, long long rows, int hist_len, int vocab,
                                 uint16_t *counts, uint32_t *presence, cudaStream_t stream);

}  // namespace z2
