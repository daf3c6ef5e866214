// head.cuh -- launcher interface of the output-head kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace z2 {

struct HeadArgs {
    const void *W;        // [n_cb*rows_per_cb][dim] row-major
    int rows_per_cb, n_cb, vocab, dim;
    const void *hidden;   // [batch][dim]
    int batch;
    float softcap;        // <= 0: no cap
    float *out;           // [batch][n_cb][vocab] f32, or [batch/2][..] with cfg
    // Classifier-free guidance: hidden rows come in pairs (2s conditional,
    // 2s+1 unconditional) and out row s is u + cfg_scale * (c - u) of the two
    // softcapped rows (src/zonos2_generate.cpp:178-183).  batch is even.
    int cfg = 0;
    float cfg_scale = 1.0f;
    // Per hidden row, a factor applied to the row's dot products before the
    // softcap (bf16 kernel only): the output RMSNorm's 1 / rms when its weight has
    // been folded into the columns of W.  nullptr: none.
    const float *row_scale = nullptr;
};

// The output RMSNorm of rows x [rows][dim] (f32, or bf16 when `bf16`) into y of
// the same type, with the optional f32 scale weight w [dim]
// (head_prologue.cu).
cudaError_t launch_out_norm(const void *x, bool bf16, int rows, int dim, float eps,
                            const float *w, void *y, cudaStream_t stream);

// 1 / rms of each row of x [rows][dim] (bf16), rms = sqrt(mean of squares + eps),
// into rcp [rows] f32: the output RMSNorm's row factor, applied by the bf16 head's
// epilogue when the norm's weight is folded into W (head_prologue.cu).
cudaError_t launch_row_rcp_rms(const void *x, int rows, int dim, float eps, float *rcp,
                               cudaStream_t stream);

// W'[r][k] = bf16(W[r][k] * w[k]) for rows x dim bf16 W and f32 w: the output
// RMSNorm's weight folded into the columns of the head (head_prologue.cu).
cudaError_t launch_fold_columns(const void *W, const float *w, int rows, int dim, void *out,
                                cudaStream_t stream);

// f32 weights and hidden states: one warp per output row, f64 accumulation
// (head_gemv.cu).
cudaError_t launch_head_gemv_f32(const HeadArgs &a, cudaStream_t stream);

// bf16 weights and hidden states: tcgen05 tensor-core GEMM with the softcap in
// the TMEM epilogue (head_tc.cu).  Returns cudaErrorNotSupported for shapes it
// does not implement.
cudaError_t launch_head_tc_bf16(const HeadArgs &a, cudaStream_t stream);

// Reads and clears the device error word written by the tcgen05 kernel's
// bounded waits (head_tc.cu).
int read_and_clear_device_error(int *value);

}  // namespace z2
