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
    const uint32_t *allow;   // [n_streams][allow_words] or, lane-major, [n_streams][32]
    int allow_words;
    int allow_lane_major;    // allow holds lane-major words (word l, bit 4*j + e: token
                             // 4*(l + 32*j) + e), 32 per stream
    int delay_step;
    int32_t *codes;          // [n_streams][n_cb]; also carries each row's uniform between
                             // the two kernels of a step
    int32_t *flags;          // [n_streams][n_cb] or nullptr
    int vec_logits;          // rows 16-byte aligned and vocab % 4 == 0
    int vec_hist;            // history rows 16-byte aligned and hist_len % 4 == 0
    // Incremental history (the decode context): per row, how often each token
    // occurs in the ring and a bitmap of the tokens that occur.  When set, the
    // penalty reads the bitmap instead of scanning the ring, and the kernel
    // updates counts and bitmap for the token it evicts and the one it appends.
    uint16_t *counts;        // [n_streams][n_cb][1024] or nullptr
    uint32_t *presence;      // [n_streams][n_cb][32] lane-major, or nullptr
    // Uniforms drawn one step ahead (the decode context).  When u_cur is set the
    // step is one launch: row r reads its uniform from u_cur[r]; warp 0 of each
    // CTA sets rng to rng_ahead (the state after this step's draws) for its slice
    // of streams, draws the next step's uniforms into u_next and leaves rng_ahead
    // the state after them.  When u_cur is nullptr a draw kernel precedes the
    // sampler and parks the uniforms in the code slots.
    const float *u_cur;      // [n_streams][n_cb] or nullptr
    float *u_next;           // [n_streams][n_cb]
    uint64_t *rng_ahead;     // [n_streams][4]
};

// Enqueues one sampling step (the uniform draw, then the persistent sampler
// under programmatic dependent launch); returns the cudaError_t of the launches.
cudaError_t launch_sample(const SampleArgs &a, cudaStream_t stream);

// Draws one step's uniforms from rng_in into u ([n_streams][n_cb] f32) and
// writes the advanced states to rng_out (rng_in is left as it is): the decode
// context's first step, and the first after its generators are set.
cudaError_t launch_draw_ahead(const uint64_t *rng_in, uint64_t *rng_out, int n_streams, int n_cb,
                              float *u, cudaStream_t stream);

// Shared memory bytes of one sampler CTA.
size_t sample_smem_bytes();

// Reads and clears the sampler's device error word (1: a row copy did not
// complete within ~2 s).  Returns a cudaError_t.
int read_and_clear_sampler_error(int *value);

// Rebuilds counts / lane-major presence of `rows` history rings
// ([rows][hist_len] i32, entries outside [0, vocab) ignored).  hist_len <= 65535.
cudaError_t launch_history_index(const int32_t *hist, long long rows, int hist_len, int vocab,
                                 uint16_t *counts, uint32_t *presence, cudaStream_t stream);

}  // namespace z2
