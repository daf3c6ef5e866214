// generate.cu -- the batched generation loop around the decode step (sm_100a).
//
// gen_append_kernel restates, for a batch of streams, what the reference's loop
// does with each sampled frame (src/zonos2_generate.cpp:209-226, :259-276):
// codes clamped to codebook_size - 1, the frame kept, the stream ended after a
// frame holding the end-of-audio id, and the next step's input frame built
// from it -- the codes plus the text padding id (:238-243).  One thread per
// stream; an ended stream (or one with max_frames frames) keeps nothing more.
//
// embed_frames_kernel restates embedding_sum (src/zonos2_model.cpp:116-151),
// the model's input embedding of a frame: the codebook rows added in codebook
// order, then the text row (5x for a text token, once for the padding id).  One
// thread per (frame, element), so the adds of each element run in the
// reference's order; built with -fmad=false, so `row * 5 + acc` rounds twice
// like the reference's.
//
// shear_up_kernel restates shear_up (scripts/dac_decode.py:23-30): codebook j
// advanced by j frames, the vacated tail filled with the padding id.
#include "common.cuh"
#include "generate.cuh"

namespace z2 {

namespace {

__global__ void __launch_bounds__(128)
    gen_append_kernel(const int32_t *__restrict__ codes, int n_streams, int n_cb,
                      int codebook_size, int eoa_id, int text_pad_id, int max_frames,
                      int32_t *__restrict__ frames, int32_t *__restrict__ n_frames,
                      int32_t *__restrict__ eos_at, int32_t *__restrict__ next_in)
{
    const int s = blockIdx.x * 128 + threadIdx.x;
    if (s >= n_streams) return;
    const int n = n_frames[s];
    if (eos_at[s] >= 0 || n >= max_frames) return;
    const int32_t *c = codes + (size_t)s * n_cb;
    int32_t *f = frames + ((size_t)s * max_frames + n) * n_cb;
    int32_t *in = next_in + (size_t)s * (n_cb + 1);
    bool eos = false;
    for (int cb = 0; cb < n_cb; cb++) {
        int tok = c[cb];
        if (tok >= codebook_size) tok = codebook_size - 1;
        f[cb] = tok;
        in[cb] = tok;
        eos |= tok == eoa_id;
    }
    in[n_cb] = text_pad_id;
    if (eos) eos_at[s] = n;
    n_frames[s] = n + 1;
}

__global__ void __launch_bounds__(256)
    embed_frames_kernel(const float *__restrict__ cb_tables, const float *__restrict__ text_table,
                        int n_cb, int audio_vocab, int text_vocab, int dim,
                        const int32_t *__restrict__ ids, int n, float *__restrict__ out)
{
    const int d = blockIdx.x * 256 + threadIdx.x;
    const int t = blockIdx.y;
    if (d >= dim || t >= n) return;
    const int32_t *id = ids + (size_t)t * (n_cb + 1);
    float acc = 0.0f;
    for (int cb = 0; cb < n_cb; cb++) {
        const int tid = __ldg(id + cb);
        if (tid >= 0 && tid < audio_vocab)
            acc = __fadd_rn(acc, __ldg(cb_tables + ((size_t)cb * audio_vocab + tid) * dim + d));
    }
    const int tid = __ldg(id + n_cb);
    if (tid >= 0 && tid < text_vocab)
        acc = __fadd_rn(acc, __fmul_rn(__ldg(text_table + (size_t)tid * dim + d), 5.0f));
    else if (tid == text_vocab)
        acc = __fadd_rn(acc, __ldg(text_table + (size_t)tid * dim + d));
    out[(size_t)t * dim + d] = acc;
}

__global__ void __launch_bounds__(256)
    shear_up_kernel(const int32_t *__restrict__ frames, const int32_t *__restrict__ n_frames,
                    int n_streams, int max_frames, int n_cb, int32_t pad, int32_t *__restrict__ out)
{
    const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
    const long long total = (long long)n_streams * max_frames * n_cb;
    if (i >= total) return;
    const int j = (int)(i % n_cb);
    const long long st = i / n_cb;
    const int t = (int)(st % max_frames);
    const int s = (int)(st / max_frames);
    const int nf = n_frames[s];
    out[i] = t + j < nf ? frames[((size_t)s * max_frames + t + j) * n_cb + j] : pad;
}

}  // namespace

cudaError_t launch_gen_append(const int32_t *codes, int n_streams, int n_cb, int codebook_size,
                              int eoa_id, int text_pad_id, int max_frames, int32_t *frames,
                              int32_t *n_frames, int32_t *eos_at, int32_t *next_in,
                              cudaStream_t stream)
{
    if (n_streams == 0) return cudaSuccess;
    gen_append_kernel<<<(unsigned)((n_streams + 127) / 128), 128, 0, stream>>>(
        codes, n_streams, n_cb, codebook_size, eoa_id, text_pad_id, max_frames, frames, n_frames,
        eos_at, next_in);
    return cudaGetLastError();
}

cudaError_t launch_embed_frames(const float *cb_tables, const float *text_table, int n_cb,
                                int audio_vocab, int text_vocab, int dim, const int32_t *ids,
                                int n, float *out, cudaStream_t stream)
{
    if (n == 0 || dim == 0) return cudaSuccess;
    const dim3 grid((unsigned)((dim + 255) / 256), (unsigned)n);
    embed_frames_kernel<<<grid, 256, 0, stream>>>(cb_tables, text_table, n_cb, audio_vocab,
                                                 text_vocab, dim, ids, n, out);
    return cudaGetLastError();
}

cudaError_t launch_shear_up(const int32_t *frames, const int32_t *n_frames, int n_streams,
                            int max_frames, int n_cb, int32_t pad, int32_t *out,
                            cudaStream_t stream)
{
    const long long total = (long long)n_streams * max_frames * n_cb;
    if (total == 0) return cudaSuccess;
    shear_up_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
        frames, n_frames, n_streams, max_frames, n_cb, pad, out);
    return cudaGetLastError();
}

}  // namespace z2
