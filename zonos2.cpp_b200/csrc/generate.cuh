// generate.cuh -- launchers of the generation-loop kernels (generate.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace z2 {

// Appends each stream's sampled frame codes [n_streams][n_cb] to frames
// [n_streams][max_frames][n_cb] (clamp, end-of-audio, frame count) and writes
// its next input frame next_in [n_streams][n_cb + 1].
cudaError_t launch_gen_append(const int32_t *codes, int n_streams, int n_cb, int codebook_size,
                              int eoa_id, int text_pad_id, int max_frames, int32_t *frames,
                              int32_t *n_frames, int32_t *eos_at, int32_t *next_in,
                              cudaStream_t stream);

// Input embeddings out [n][dim] f32 of frames ids [n][n_cb + 1]; cb_tables
// [n_cb][audio_vocab][dim], text_table [text_vocab + 1][dim], f32 row-major.
cudaError_t launch_embed_frames(const float *cb_tables, const float *text_table, int n_cb,
                                int audio_vocab, int text_vocab, int dim, const int32_t *ids,
                                int n, float *out, cudaStream_t stream);

// out [n_streams][max_frames][n_cb]: each stream's frames with the delay
// pattern removed, pad past its own frame count.
cudaError_t launch_shear_up(const int32_t *frames, const int32_t *n_frames, int n_streams,
                            int max_frames, int n_cb, int32_t pad, int32_t *out,
                            cudaStream_t stream);

}  // namespace z2
