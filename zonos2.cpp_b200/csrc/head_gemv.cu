// head_gemv.cu -- f32 output head + softcap for small batches (sm_100a).
//
// Restates linear_forward for the multi_output head (src/zonos2_model.cpp:
// 200-216, :687-690) followed by the softcap l = 15*tanh(l/15) of
// src/zonos2_model.cpp:692-703, for the sampled rows of each codebook.
// The head is a GEMV at decode batch sizes: every weight row is read once
// from HBM by one warp with coalesced 128-bit loads (the bound is the
// 4*n_cb*vocab*dim bytes of W), and the dot product is accumulated in f64 so
// the f32 result is the correctly rounded dot product -- within the
// reference's own sequential-f32 rounding error of its value.  With
// classifier-free guidance, rows 2s and 2s+1 (conditional, unconditional) are
// blended into output row s after the softcap (src/zonos2_generate.cpp:178-183).
#include <math.h>

#include "common.cuh"
#include "head.cuh"

namespace z2 {

namespace {

constexpr int kGemvWarps = 8;

__global__ void __launch_bounds__(32 * kGemvWarps)
    head_gemv_f32_kernel(const float *__restrict__ W, int rows_per_cb, int n_cb, int vocab,
                         int dim, const float *__restrict__ hid, int batch, float cap,
                         float *__restrict__ out, int vec, int cfg, float cfg_scale)
{
    const int lane = threadIdx.x & 31;
    const int o = blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
    if (o >= n_cb * vocab) return;
    const int c = o / vocab, v = o - c * vocab;
    const float *w = W + ((size_t)c * rows_per_cb + v) * (size_t)dim;
    float cond = 0.0f;   // with cfg: the softcapped logit of the pair's conditional row
    for (int b = 0; b < batch; b++) {
        const float *h = hid + (size_t)b * dim;
        double acc = 0.0;
        if (vec) {
            for (int i = 4 * lane; i < dim; i += 128) {
                const float4 wv = __ldg(reinterpret_cast<const float4 *>(w + i));
                const float4 hv = __ldg(reinterpret_cast<const float4 *>(h + i));
                acc += (double)wv.x * (double)hv.x;
                acc += (double)wv.y * (double)hv.y;
                acc += (double)wv.z * (double)hv.z;
                acc += (double)wv.w * (double)hv.w;
            }
        } else {
            for (int i = lane; i < dim; i += 32) acc += (double)__ldg(w + i) * (double)__ldg(h + i);
        }
#pragma unroll
        for (int s = 16; s; s >>= 1) acc += __shfl_xor_sync(kFull, acc, s);
        if (lane == 0) {
            float l = __double2float_rn(acc);
            if (cap > 0.0f) l = cap * tanhf(l / cap);
            if (!cfg) {
                out[((size_t)b * n_cb + c) * vocab + v] = l;
            } else if ((b & 1) == 0) {
                cond = l;
            } else {   // u + s * (c - u), rounded step by step like the reference
                out[((size_t)(b >> 1) * n_cb + c) * vocab + v] =
                    __fadd_rn(l, __fmul_rn(cfg_scale, __fsub_rn(cond, l)));
            }
        }
    }
}

}  // namespace

cudaError_t launch_head_gemv_f32(const HeadArgs &a, cudaStream_t stream)
{
    const int rows = a.n_cb * a.vocab;
    if (rows == 0 || a.batch == 0) return cudaSuccess;
    const int vec = (a.dim % 4 == 0) && ((uintptr_t)a.W % 16 == 0) &&
                    ((uintptr_t)a.hidden % 16 == 0);
    const int blocks = (rows + kGemvWarps - 1) / kGemvWarps;
    head_gemv_f32_kernel<<<blocks, 32 * kGemvWarps, 0, stream>>>(
        static_cast<const float *>(a.W), a.rows_per_cb, a.n_cb, a.vocab, a.dim,
        static_cast<const float *>(a.hidden), a.batch, a.softcap, a.out, vec, a.cfg,
        a.cfg_scale);
    return cudaGetLastError();
}

}  // namespace z2
