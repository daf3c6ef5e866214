// capi.cu -- the extern "C" boundary declared in include/zonos2_cuda.h.
//
// Host-side argument checks, the per-device staging of the sample_token
// drop-in, and the context that keeps a shard of decode streams' generator
// states, history rings and masks resident in HBM.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <new>

#include "common.cuh"
#include "head.cuh"
#include "generate.cuh"
#include "sampler.cuh"
#include "zonos2_cuda.h"

namespace {

thread_local char tl_error[256] = "";

}  // namespace

// The message zonos2cu_last_error returns on this thread (the other .cu files
// of the library report through it).
__attribute__((visibility("hidden"))) const char *z2_set_error(const char *fmt, const char *a,
                                                               const char *b)
{
    snprintf(tl_error, sizeof(tl_error), fmt, a, b);
    return tl_error;
}

namespace {

int cuda_fail(cudaError_t e, const char *what)
{
    snprintf(tl_error, sizeof(tl_error), "%s: %s", what, cudaGetErrorString(e));
    // A failed call (cudaMalloc out of memory, say) also leaves its error in the
    // thread's last-error slot, where the next launch's cudaGetLastError would
    // find it and fail an unrelated call: the error is reported here, so clear it
    // (a sticky error stays in the context regardless).
    (void)cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? ZONOS2CU_ENOMEM : ZONOS2CU_ECUDA;
}

#define Z2_CK(call)                                               \
    do {                                                          \
        const cudaError_t e_ = (call);                            \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);       \
    } while (0)

int check_params(const zonos2cu_sample_params *p, int vocab)
{
    if (!p) return ZONOS2CU_EINVAL;
    if (!(p->temperature > 0.0f) || !isfinite(p->temperature)) return ZONOS2CU_EINVAL;
    if (isnan(p->top_p)) return ZONOS2CU_EINVAL;
    // min_p > 1 empties the candidate list: undefined in the reference
    if (isnan(p->min_p) || p->min_p > 1.0f) return ZONOS2CU_EINVAL;
    if (!(p->repetition_penalty > 0.0f) || !isfinite(p->repetition_penalty))
        return ZONOS2CU_EINVAL;
    if (p->pad_id < 0 || p->pad_id >= vocab) return ZONOS2CU_EINVAL;
    return ZONOS2CU_OK;
}

void fill_sample_args(z2::SampleArgs &a, const zonos2cu_sample_params *p)
{
    a.temperature = p->temperature;
    a.top_k = p->top_k;
    a.top_p = p->top_p;
    a.min_p = p->min_p;
    a.rho = p->repetition_penalty;
    a.inv_rho = 1.0f / p->repetition_penalty;
    a.inv_temp = 1.0 / (double)p->temperature;
    a.pad_id = p->pad_id;
}

int check_rows(const float *logits, int n_streams, int n_cb, int vocab, long long row_stride,
               uint64_t *rng, int32_t *hist, int hist_len, int hist_pos, int32_t *codes)
{
    if (n_streams < 0 || n_cb < 1 || n_cb > z2::kSamplerCbMax) return ZONOS2CU_EINVAL;
    if (vocab < 1) return ZONOS2CU_EINVAL;
    if (vocab > z2::kSamplerVocabMax) return ZONOS2CU_EUNSUPPORTED;
    if (row_stride < vocab) return ZONOS2CU_EINVAL;
    if (hist_len < 0) return ZONOS2CU_EINVAL;
    if (hist_len > 0 && (!hist || hist_pos < 0 || hist_pos >= hist_len)) return ZONOS2CU_EINVAL;
    if (n_streams > 0 && (!logits || !rng || !codes)) return ZONOS2CU_EINVAL;
    if ((uintptr_t)rng % 16 != 0) return ZONOS2CU_EINVAL;  // generator states load as 16-byte pairs
    return ZONOS2CU_OK;
}

int launch_rows(const float *logits, int n_streams, int n_cb, int vocab, long long row_stride,
                const zonos2cu_sample_params *params, uint64_t *rng, int32_t *hist,
                int hist_len, int hist_pos, const uint32_t *allow, int delay_step,
                int32_t *codes, int32_t *flags, cudaStream_t stream,
                uint16_t *counts = nullptr, uint32_t *presence = nullptr,
                bool allow_lane_major = false, const float *u_cur = nullptr,
                float *u_next = nullptr, uint64_t *rng_ahead = nullptr)
{
    z2::SampleArgs a{};
    a.logits = logits;
    a.row_stride = row_stride;
    a.n_streams = n_streams;
    a.n_cb = n_cb;
    a.vocab = vocab;
    fill_sample_args(a, params);
    a.rng = rng;
    a.hist = hist_len > 0 ? hist : nullptr;
    a.hist_len = hist_len;
    a.hist_pos = hist_pos;
    a.allow = allow;
    a.allow_words = (vocab + 31) / 32;
    a.allow_lane_major = allow_lane_major ? 1 : 0;
    a.delay_step = delay_step;
    a.codes = codes;
    a.flags = flags;
    a.vec_logits = (row_stride % 4 == 0) && (vocab % 4 == 0) && ((uintptr_t)logits % 16 == 0);
    a.vec_hist = hist_len > 0 && (hist_len % 4 == 0) && ((uintptr_t)hist % 16 == 0);
    a.counts = hist_len > 0 ? counts : nullptr;
    a.presence = hist_len > 0 ? presence : nullptr;
    a.u_cur = u_cur;
    a.u_next = u_next;
    a.rng_ahead = rng_ahead;
    Z2_CK(z2::launch_sample(a, stream));
    return ZONOS2CU_OK;
}

// n elements of device memory; *p is written only on success
template <class T>
cudaError_t dev_alloc(T **p, size_t n)
{
    void *q = nullptr;
    const cudaError_t e = cudaMalloc(&q, sizeof(T) * n);
    if (e == cudaSuccess) *p = static_cast<T *>(q);
    return e;
}

// ---- per-device staging for the sample_token drop-in --------------------
// One row per call: the uniform is drawn on the host from the caller's generator
// (the reference's own draw), the row and its uniform go over in one copy from
// page-locked memory, the sampler runs the row with that uniform (the decode
// context's drawn-ahead path; the generator words it advances there are scratch)
// and writes the code and flag straight into mapped page-locked memory, so no
// copy comes back.
struct Staging {   // created on the first call on the device and kept until exit
    std::mutex mu;
    bool ready = false;
    cudaStream_t stream = nullptr;
    float *h_in = nullptr;      // page-locked [1024] logits + [1] uniform
    int32_t *h_out = nullptr;   // page-locked and mapped [2] code, flag
    int32_t *h_out_dev = nullptr;   // h_out as the device sees it
    float *d_in = nullptr;      // [1024] logits, [1024] the uniform, [1025] scratch uniform
    uint64_t *d_rng = nullptr;  // [8] scratch generator words
};
Staging g_staging[64];

// The generator's next f32 uniform, as the reference draws it
// (src/zonos2_generate.cpp:20-33): 53-bit double in [0, 1), narrowed to float.
float host_randf(uint64_t st[4])
{
    const uint64_t s1 = st[1];
    const uint64_t x = s1 * 5u;
    const uint64_t out = ((x << 7) | (x >> 57)) * 9u;
    const uint64_t t = st[1] << 17;
    st[2] ^= st[0];
    st[3] ^= st[1];
    st[1] ^= st[2];
    st[0] ^= st[3];
    st[2] ^= t;
    st[3] = (st[3] << 45) | (st[3] >> 19);
    return (float)((double)(out >> 11) * 0x1.0p-53);
}

}  // namespace

extern "C" {

void zonos2cu_default_params(zonos2cu_sample_params *p)
{
    if (!p) return;
    p->temperature = 0.7f;
    p->top_k = 50;
    p->top_p = 0.9f;
    p->min_p = 0.02f;
    p->repetition_penalty = 1.0f;
    p->pad_id = 1023;
}

const char *zonos2cu_version(void) { return "zonos2cu 0.1 (sm_100a)"; }

const char *zonos2cu_last_error(void) { return tl_error; }

void zonos2cu_rng_seed(uint64_t seed, uint64_t state[4])
{
    // src/zonos2_generate.cpp:13-19
    uint64_t s0 = seed ^ 0x9E3779B97F4A7C15ULL, s1 = seed ^ 0xBF58476D1CE4E5B9ULL,
             s2 = seed ^ 0x94D049BB133111EBULL, s3 = seed ^ 0x3243F6A8885A308DULL;
    for (int i = 0; i < 20; i++) {
        const uint64_t t = s1 << 17;
        s2 ^= s0;
        s3 ^= s1;
        s1 ^= s2;
        s0 ^= s3;
        s2 ^= t;
        s3 = (s3 << 45) | (s3 >> 19);
    }
    state[0] = s0;
    state[1] = s1;
    state[2] = s2;
    state[3] = s3;
}

int zonos2cu_sample_rows(const float *logits_dev, int n_streams, int n_cb, int vocab,
                         long long row_stride, const zonos2cu_sample_params *params,
                         uint64_t *rng_dev, int32_t *hist_dev, int hist_len, int hist_pos,
                         const uint32_t *allow_dev, int delay_step, int32_t *codes_dev,
                         int32_t *flags_dev, void *stream)
{
    int rc = check_rows(logits_dev, n_streams, n_cb, vocab, row_stride, rng_dev, hist_dev,
                        hist_len, hist_pos, codes_dev);
    if (rc) return rc;
    if ((rc = check_params(params, vocab))) return rc;
    return launch_rows(logits_dev, n_streams, n_cb, vocab, row_stride, params, rng_dev, hist_dev,
                       hist_len, hist_pos, allow_dev, delay_step, codes_dev, flags_dev,
                       (cudaStream_t)stream);
}

int zonos2cu_sample_token(uint64_t rng_state[4], const float *logits, int vocab_size,
                          float temp, int top_k, float top_p, float min_p)
{
    if (!rng_state || !logits || vocab_size < 1) return ZONOS2CU_EINVAL;
    if (vocab_size > z2::kSamplerVocabMax) return ZONOS2CU_EUNSUPPORTED;
    zonos2cu_sample_params p;
    p.temperature = temp;
    p.top_k = top_k;
    p.top_p = top_p;
    p.min_p = min_p;
    p.repetition_penalty = 1.0f;
    p.pad_id = 0;
    int rc = check_params(&p, vocab_size);
    if (rc) return rc;
    int dev = 0;
    Z2_CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return ZONOS2CU_EINVAL;
    Staging &st = g_staging[dev];
    std::lock_guard<std::mutex> lock(st.mu);
    // first call on this device: the staging area (a call that failed part way
    // keeps what it made, and the next one makes the rest)
    if (!st.ready) {
        if (!st.stream) {
            cudaStream_t s = nullptr;
            Z2_CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
            st.stream = s;
        }
        if (!st.h_in) {
            void *h = nullptr;
            Z2_CK(cudaHostAlloc(&h, sizeof(float) * (z2::kSamplerVocabMax + 4), cudaHostAllocDefault));
            st.h_in = static_cast<float *>(h);
        }
        if (!st.h_out) {
            void *h = nullptr;
            Z2_CK(cudaHostAlloc(&h, sizeof(int32_t) * 2, cudaHostAllocMapped));
            st.h_out = static_cast<int32_t *>(h);
        }
        if (!st.h_out_dev) {
            void *d = nullptr;
            Z2_CK(cudaHostGetDevicePointer(&d, st.h_out, 0));
            st.h_out_dev = static_cast<int32_t *>(d);
        }
        if (!st.d_in) Z2_CK(dev_alloc(&st.d_in, z2::kSamplerVocabMax + 4));
        if (!st.d_rng) {
            Z2_CK(dev_alloc(&st.d_rng, 8));
            Z2_CK(cudaMemsetAsync(st.d_rng, 0, sizeof(uint64_t) * 8, st.stream));
        }
        st.ready = true;
    }
    uint64_t rs[4];
    memcpy(rs, rng_state, sizeof(rs));
    const float u = host_randf(rs);   // the call's one draw
    memcpy(st.h_in, logits, sizeof(float) * vocab_size);
    st.h_in[z2::kSamplerVocabMax] = u;
    // one copy: the row, then (past the row's vocab_size entries, which the sampler
    // does not read) the uniform at entry 1024
    Z2_CK(cudaMemcpyAsync(st.d_in, st.h_in, sizeof(float) * (z2::kSamplerVocabMax + 1),
                          cudaMemcpyHostToDevice, st.stream));
    rc = launch_rows(st.d_in, 1, 1, vocab_size, vocab_size, &p, st.d_rng, nullptr, 0, 0, nullptr,
                     -1, st.h_out_dev, st.h_out_dev + 1, st.stream, nullptr, nullptr, false,
                     st.d_in + z2::kSamplerVocabMax, st.d_in + z2::kSamplerVocabMax + 1,
                     st.d_rng + 4);
    if (rc) return rc;
    Z2_CK(cudaStreamSynchronize(st.stream));   // the code and flag are in h_out
    memcpy(rng_state, rs, sizeof(rs));
    if (st.h_out[1] & ZONOS2CU_FLAG_ALL_MASKED) return ZONOS2CU_EINVAL;
    return st.h_out[0];
}

}  // extern "C"

namespace {

int check_head(const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb, int n_cb, int vocab,
               int dim, const void *hidden_dev, int batch, float softcap, const float *logits_dev)
{
    if (n_cb < 1 || vocab < 1 || dim < 1 || batch < 0 || rows_per_cb < vocab)
        return ZONOS2CU_EINVAL;
    if (isnan(softcap)) return ZONOS2CU_EINVAL;
    if (dtype != ZONOS2CU_F32 && dtype != ZONOS2CU_BF16) return ZONOS2CU_EINVAL;
    if (batch > 0 && (!W_dev || !hidden_dev || !logits_dev)) return ZONOS2CU_EINVAL;
    return ZONOS2CU_OK;
}

// The head on `batch` hidden rows; with cfg, rows pair up and `logits_dev` gets
// batch / 2 blended rows.
int launch_head(const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb, int n_cb, int vocab,
                int dim, const void *hidden_dev, int batch, float softcap, float *logits_dev,
                void *stream, bool cfg, float cfg_scale, const float *row_scale = nullptr)
{
    int rc = check_head(W_dev, dtype, rows_per_cb, n_cb, vocab, dim, hidden_dev, batch, softcap,
                        logits_dev);
    if (rc) return rc;
    z2::HeadArgs a{W_dev, rows_per_cb, n_cb, vocab, dim, hidden_dev, batch, softcap, logits_dev};
    a.cfg = cfg ? 1 : 0;
    a.cfg_scale = cfg_scale;
    a.row_scale = row_scale;
    cudaError_t e;
    if (dtype == ZONOS2CU_F32) {
        e = z2::launch_head_gemv_f32(a, (cudaStream_t)stream);
    } else if (dtype == ZONOS2CU_BF16) {
        e = z2::launch_head_tc_bf16(a, (cudaStream_t)stream);
        if (e == cudaErrorNotSupported) return ZONOS2CU_EUNSUPPORTED;
    } else {
        return ZONOS2CU_EINVAL;
    }
    if (e != cudaSuccess) return cuda_fail(e, "head launch");
    return ZONOS2CU_OK;
}

}  // namespace

// Every check that zonos2cu_head_softcap and then zonos2cu_sample_rows would make
// on these arguments, with `logits_dev` standing for the buffer between them:
// zonos2cu_step_noalloc runs it before it launches anything.
__attribute__((visibility("hidden"))) int z2_check_head_then_sample(
    const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb, int n_cb, int vocab, int dim,
    const void *hidden_dev, int n_streams, float softcap, const float *logits_dev,
    const zonos2cu_sample_params *params, uint64_t *rng_dev, int32_t *hist_dev, int hist_len,
    int hist_pos, int32_t *codes_dev)
{
    int rc = check_head(W_dev, dtype, rows_per_cb, n_cb, vocab, dim, hidden_dev, n_streams,
                        softcap, logits_dev);
    if (rc) return rc;
    rc = check_rows(logits_dev, n_streams, n_cb, vocab, vocab, rng_dev, hist_dev, hist_len,
                    hist_pos, codes_dev);
    if (rc) return rc;
    return check_params(params, vocab);
}

extern "C" {

int zonos2cu_head_softcap(const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb, int n_cb,
                          int vocab, int dim, const void *hidden_dev, int batch, float softcap,
                          float *logits_dev, void *stream)
{
    return launch_head(W_dev, dtype, rows_per_cb, n_cb, vocab, dim, hidden_dev, batch, softcap,
                       logits_dev, stream, false, 1.0f);
}

int zonos2cu_embed_frames(const float *codebook_tables_dev, const float *text_table_dev,
                          int n_cb, int audio_vocab, int text_vocab, int dim,
                          const int32_t *ids_dev, int n_frames, float *out_dev, void *stream)
{
    if (n_cb < 1 || audio_vocab < 1 || text_vocab < 0 || dim < 1 || n_frames < 0)
        return ZONOS2CU_EINVAL;
    if (n_frames > 0 && (!codebook_tables_dev || !text_table_dev || !ids_dev || !out_dev))
        return ZONOS2CU_EINVAL;
    Z2_CK(z2::launch_embed_frames(codebook_tables_dev, text_table_dev, n_cb, audio_vocab,
                                  text_vocab, dim, ids_dev, n_frames, out_dev,
                                  (cudaStream_t)stream));
    return ZONOS2CU_OK;
}

int zonos2cu_write_codes_bin(const char *path, const int32_t *frames_host, int n_frames, int n_cb)
{
    if (!path || n_frames < 0 || n_cb < 0 || (n_frames > 0 && n_cb > 0 && !frames_host))
        return ZONOS2CU_EINVAL;
    FILE *f = fopen(path, "wb");
    if (!f) return ZONOS2CU_EINVAL;
    const size_t n = (size_t)n_frames * (size_t)n_cb;
    const bool ok = fwrite(&n_frames, sizeof(int), 1, f) == 1 &&
                    fwrite(&n_cb, sizeof(int), 1, f) == 1 &&
                    (n == 0 || fwrite(frames_host, sizeof(int32_t), n, f) == n);
    if (fclose(f) != 0 || !ok) return ZONOS2CU_EINVAL;
    return ZONOS2CU_OK;
}

int zonos2cu_device_error(void)
{
    Z2_CK(cudaDeviceSynchronize());
    int v = 0, vs = 0;
    int e = z2::read_and_clear_device_error(&v);
    if (!e) e = z2::read_and_clear_sampler_error(&vs);
    if (e) return cuda_fail((cudaError_t)e, "device error word");
    return v ? v : vs;
}

}  // extern "C"

// ---- context --------------------------------------------------------------

struct zonos2cu_ctx {
    int device = 0;
    zonos2cu_dims dims{};
    cudaStream_t stream = nullptr;
    uint64_t *rng = nullptr;     // [S][4]
    int32_t *hist = nullptr;     // [S][C][H]
    int hist_pos = 0;
    uint16_t *counts = nullptr;  // [S][C][1024] occurrences of each token in the ring
    uint32_t *presence = nullptr;// [S][C][32] tokens with a nonzero count, lane-major
    // Uniforms drawn one step ahead: u_ahead[ahead_par] holds the next step's,
    // rng_ahead the generators after them (rng stays the state after the steps taken).
    float *u_ahead = nullptr;    // [2][S][C]
    uint64_t *rng_ahead = nullptr;
    bool ahead_valid = false;    // u_ahead[ahead_par] and rng_ahead follow from rng
    int ahead_par = 0;
    uint32_t *allow = nullptr;   // [S][32] lane-major (word l, bit 4j+e: token 4(l+32j)+e)
    bool allow_on = false;
    void *head = nullptr;        // [C*V][D] of head_dtype
    zonos2cu_dtype head_dtype = ZONOS2CU_F32;
    float *logits = nullptr;     // [S][C][V] fused-step intermediate
    // output RMSNorm ahead of the head (zonos2cu_set_out_norm)
    bool norm_on = false;
    float norm_eps = 1e-5f;
    float *norm_w = nullptr;     // [D] or unused
    bool norm_has_w = false;
    void *normed = nullptr;      // [2S][D] f32: the normalised rows (f32 head)
    void *head_folded = nullptr; // bf16 head with the norm weight folded into its columns
    float *row_rcp = nullptr;    // [2S]: 1 / rms of each hidden row (bf16 head)
    // classifier-free guidance (zonos2cu_set_cfg): steps take 2S hidden rows
    bool cfg_on = false;
    float cfg_scale = 1.0f;
    // generation loop state (zonos2cu_gen_begin)
    bool gen_on = false;
    int gen_max_frames = 0, gen_eoa = 1024, gen_pad = 1025, gen_text_pad = 519;
    size_t gen_cap = 0;               // frame slots allocated per stream x streams
    int32_t *gen_frames = nullptr;    // [S][max_frames][C]
    int32_t *gen_count = nullptr;     // [2][S]: frames kept, end-of-audio frame (-1: none)
    int32_t *gen_next = nullptr;      // [S][C+1]: the next step's input frame
    // input embedding tables (zonos2cu_set_embeddings), f32 row-major
    float *emb_cb = nullptr;          // [C][audio_vocab][D]
    float *emb_text = nullptr;        // [text_vocab+1][D]
    int emb_audio_vocab = 0, emb_text_vocab = 0;
    // host-path staging, grown on demand
    float *in_logits = nullptr;
    size_t in_logits_bytes = 0;
    void *in_hidden = nullptr;
    size_t in_hidden_bytes = 0;
    int32_t *out = nullptr;      // [2][S][C] codes, flags, as the device writes them
    int32_t *out_host = nullptr; // the same memory, page-locked and mapped, for small batches
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev)
    {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard()
    {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

size_t n_rows(const zonos2cu_ctx *c) { return (size_t)c->dims.n_streams * c->dims.n_cb; }

int grow(void **p, size_t *cap, size_t want)
{
    if (*cap >= want) return ZONOS2CU_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    Z2_CK(cudaMalloc(p, want));
    *cap = want;
    return ZONOS2CU_OK;
}

// The bf16 head with the output norm's weight folded into its columns, when both
// are set (synchronises the context's stream).
int refold_head(zonos2cu_ctx *c)
{
    if (!c->norm_on || !c->norm_has_w || !c->head || c->head_dtype != ZONOS2CU_BF16)
        return ZONOS2CU_OK;
    const size_t rows = (size_t)c->dims.n_cb * c->dims.vocab, D = (size_t)c->dims.dim;
    if (!c->head_folded) Z2_CK(cudaMalloc(&c->head_folded, 2 * rows * D));
    Z2_CK(z2::launch_fold_columns(c->head, c->norm_w, (int)rows, (int)D, c->head_folded,
                                  c->stream));
    Z2_CK(cudaStreamSynchronize(c->stream));
    return ZONOS2CU_OK;
}

// Small batches: the host path's codes and flags are written by the kernels
// straight into mapped page-locked memory, so no copy comes back (a frame of a
// one-stream context, 45 -> 35 us per call).  Larger batches copy them back in
// one piece each, which beats that many scattered writes over PCIe.
constexpr size_t kMappedOutRows = 2304;

int ensure_out(zonos2cu_ctx *c)
{
    if (c->out) return ZONOS2CU_OK;
    const size_t n = 2 * (n_rows(c) ? n_rows(c) : 1);
    if (n_rows(c) <= kMappedOutRows) {
        void *h = nullptr, *d = nullptr;
        Z2_CK(cudaHostAlloc(&h, sizeof(int32_t) * n, cudaHostAllocMapped));
        const cudaError_t e = cudaHostGetDevicePointer(&d, h, 0);
        if (e != cudaSuccess) {
            cudaFreeHost(h);
            return cuda_fail(e, "mapped output");
        }
        c->out_host = static_cast<int32_t *>(h);
        c->out = static_cast<int32_t *>(d);
        return ZONOS2CU_OK;
    }
    Z2_CK(cudaMalloc(&c->out, sizeof(int32_t) * n));
    return ZONOS2CU_OK;
}

// The host path's codes (and flags) of the step just enqueued on c->stream, on
// the host when it returns.
int finish_host_step(zonos2cu_ctx *c, size_t rows, int32_t *codes_host, int32_t *flags_host)
{
    if (c->out_host) {
        Z2_CK(cudaStreamSynchronize(c->stream));
        memcpy(codes_host, c->out_host, sizeof(int32_t) * rows);
        if (flags_host) memcpy(flags_host, c->out_host + rows, sizeof(int32_t) * rows);
        return ZONOS2CU_OK;
    }
    Z2_CK(cudaMemcpyAsync(codes_host, c->out, sizeof(int32_t) * rows, cudaMemcpyDeviceToHost,
                          c->stream));
    if (flags_host)
        Z2_CK(cudaMemcpyAsync(flags_host, c->out + rows, sizeof(int32_t) * rows,
                              cudaMemcpyDeviceToHost, c->stream));
    Z2_CK(cudaStreamSynchronize(c->stream));
    return ZONOS2CU_OK;
}

}  // namespace

extern "C" {

int zonos2cu_ctx_create(int device, const zonos2cu_dims *d, zonos2cu_ctx **out)
{
    if (!d || !out) return ZONOS2CU_EINVAL;
    *out = nullptr;
    if (d->n_streams < 0 || d->n_cb < 1 || d->n_cb > z2::kSamplerCbMax || d->vocab < 1 ||
        d->dim < 0 || d->hist_len < 0)
        return ZONOS2CU_EINVAL;
    if (d->vocab > z2::kSamplerVocabMax) return ZONOS2CU_EUNSUPPORTED;
    if (d->hist_len > 65535) return ZONOS2CU_EUNSUPPORTED;  // 16-bit token counts
    int ndev = 0;
    Z2_CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return ZONOS2CU_EINVAL;
    DeviceGuard g(device);
    zonos2cu_ctx *c = new (std::nothrow) zonos2cu_ctx();
    if (!c) return ZONOS2CU_ENOMEM;
    c->device = device;
    c->dims = *d;
    int rc = ZONOS2CU_OK;
    do {
        cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) { rc = cuda_fail(e, "stream"); break; }
        const size_t S = (size_t)d->n_streams;
        if (S == 0) break;
        e = cudaMalloc(&c->rng, sizeof(uint64_t) * 4 * S);
        if (e == cudaSuccess) e = cudaMalloc(&c->rng_ahead, sizeof(uint64_t) * 4 * S);
        if (e == cudaSuccess) e = cudaMalloc(&c->u_ahead, sizeof(float) * 2 * S * d->n_cb);
        if (e != cudaSuccess) { rc = cuda_fail(e, "rng"); break; }
        uint64_t *h = new (std::nothrow) uint64_t[4 * S];
        if (!h) { rc = ZONOS2CU_ENOMEM; break; }
        for (size_t s = 0; s < S; s++) zonos2cu_rng_seed(d->seed + d->first_stream + s, h + 4 * s);
        e = cudaMemcpyAsync(c->rng, h, sizeof(uint64_t) * 4 * S, cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        delete[] h;
        if (e != cudaSuccess) { rc = cuda_fail(e, "rng upload"); break; }
        if (d->hist_len > 0) {
            const size_t rows = S * d->n_cb;
            const size_t hb = sizeof(int32_t) * rows * (size_t)d->hist_len;
            // u16 counts, rows 1024 wide (word-aligned pairs for the sampler's atomics)
            const size_t cbytes = sizeof(uint16_t) * rows * (size_t)z2::kSamplerVocabMax;
            const size_t pbytes = sizeof(uint32_t) * rows * 32;   // lane-major 1024-bit map
            e = cudaMalloc(&c->hist, hb);
            if (e == cudaSuccess) e = cudaMemsetAsync(c->hist, 0xff, hb, c->stream);  // -1: empty
            if (e == cudaSuccess) e = cudaMalloc(&c->counts, cbytes);
            if (e == cudaSuccess) e = cudaMemsetAsync(c->counts, 0, cbytes, c->stream);
            if (e == cudaSuccess) e = cudaMalloc(&c->presence, pbytes);
            if (e == cudaSuccess) e = cudaMemsetAsync(c->presence, 0, pbytes, c->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
            if (e != cudaSuccess) { rc = cuda_fail(e, "history"); break; }
        }
    } while (0);
    if (rc) {
        zonos2cu_ctx_destroy(c);
        return rc;
    }
    *out = c;
    return ZONOS2CU_OK;
}

int zonos2cu_ctx_destroy(zonos2cu_ctx *c)
{
    if (!c) return ZONOS2CU_OK;
    DeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    cudaFree(c->rng);
    cudaFree(c->rng_ahead);
    cudaFree(c->u_ahead);
    cudaFree(c->hist);
    cudaFree(c->counts);
    cudaFree(c->presence);
    cudaFree(c->allow);
    cudaFree(c->head);
    cudaFree(c->logits);
    cudaFree(c->norm_w);
    cudaFree(c->normed);
    cudaFree(c->head_folded);
    cudaFree(c->row_rcp);
    cudaFree(c->gen_frames);
    cudaFree(c->gen_count);
    cudaFree(c->gen_next);
    cudaFree(c->emb_cb);
    cudaFree(c->emb_text);
    cudaFree(c->in_logits);
    cudaFree(c->in_hidden);
    if (c->out_host)
        cudaFreeHost(c->out_host);
    else
        cudaFree(c->out);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return ZONOS2CU_OK;
}

void *zonos2cu_ctx_stream(zonos2cu_ctx *c) { return c ? (void *)c->stream : nullptr; }

int zonos2cu_set_head(zonos2cu_ctx *c, const void *W_host, zonos2cu_dtype dtype, int rows_per_cb)
{
    if (!c || !W_host || c->dims.dim < 1 || rows_per_cb < c->dims.vocab) return ZONOS2CU_EINVAL;
    if (dtype != ZONOS2CU_F32 && dtype != ZONOS2CU_BF16) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // no step may still be using the state
    const size_t es = dtype == ZONOS2CU_F32 ? 4 : 2;
    const size_t row_bytes = es * (size_t)c->dims.dim;
    const size_t V = (size_t)c->dims.vocab, C = (size_t)c->dims.n_cb;
    cudaFree(c->head);
    c->head = nullptr;
    Z2_CK(cudaMalloc(&c->head, row_bytes * V * C));
    // keep the sampled rows of each codebook: one 2-D copy per codebook
    for (size_t cb = 0; cb < C; cb++) {
        const char *src = static_cast<const char *>(W_host) + cb * (size_t)rows_per_cb * row_bytes;
        Z2_CK(cudaMemcpyAsync(static_cast<char *>(c->head) + cb * V * row_bytes, src, V * row_bytes,
                              cudaMemcpyHostToDevice, c->stream));
    }
    Z2_CK(cudaStreamSynchronize(c->stream));
    c->head_dtype = dtype;
    if (!c->logits && n_rows(c)) Z2_CK(cudaMalloc(&c->logits, sizeof(float) * n_rows(c) * V));
    if (c->norm_on && dtype == ZONOS2CU_F32 && !c->normed && n_rows(c))
        Z2_CK(cudaMalloc(&c->normed, sizeof(float) * 2 * (size_t)c->dims.n_streams * c->dims.dim));
    return refold_head(c);
}

int zonos2cu_set_history(zonos2cu_ctx *c, const int32_t *hist_host, int hist_pos)
{
    if (!c || !hist_host || c->dims.hist_len < 1) return ZONOS2CU_EINVAL;
    if (hist_pos < 0 || hist_pos >= c->dims.hist_len) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // no step may still be using the state
    if (n_rows(c)) {
        Z2_CK(cudaMemcpyAsync(c->hist, hist_host, sizeof(int32_t) * n_rows(c) * c->dims.hist_len,
                              cudaMemcpyHostToDevice, c->stream));
        Z2_CK(z2::launch_history_index(c->hist, (long long)n_rows(c), c->dims.hist_len,
                                       c->dims.vocab, c->counts, c->presence, c->stream));
        Z2_CK(cudaStreamSynchronize(c->stream));
    }
    c->hist_pos = hist_pos;
    return ZONOS2CU_OK;
}

int zonos2cu_get_history(zonos2cu_ctx *c, int32_t *hist_host, int *hist_pos)
{
    if (!c || c->dims.hist_len < 1) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // steps may have run on any stream
    if (hist_host && n_rows(c))
        Z2_CK(cudaMemcpy(hist_host, c->hist, sizeof(int32_t) * n_rows(c) * c->dims.hist_len,
                         cudaMemcpyDeviceToHost));
    if (hist_pos) *hist_pos = c->hist_pos;
    return ZONOS2CU_OK;
}

int zonos2cu_set_rng(zonos2cu_ctx *c, const uint64_t *state_host)
{
    if (!c || !state_host) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // no step may still be using the state
    if (c->dims.n_streams)
        Z2_CK(cudaMemcpyAsync(c->rng, state_host, sizeof(uint64_t) * 4 * c->dims.n_streams,
                              cudaMemcpyHostToDevice, c->stream));
    Z2_CK(cudaStreamSynchronize(c->stream));
    c->ahead_valid = false;   // the next step draws from the new state
    return ZONOS2CU_OK;
}

int zonos2cu_get_rng(zonos2cu_ctx *c, uint64_t *state_host)
{
    if (!c || !state_host) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // steps may have run on any stream
    if (c->dims.n_streams)
        Z2_CK(cudaMemcpy(state_host, c->rng, sizeof(uint64_t) * 4 * c->dims.n_streams,
                         cudaMemcpyDeviceToHost));
    return ZONOS2CU_OK;
}

int zonos2cu_set_allow(zonos2cu_ctx *c, const uint32_t *bits_host)
{
    if (!c) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // no step may still be using the state
    if (!bits_host) {
        c->allow_on = false;
        return ZONOS2CU_OK;
    }
    // stored lane-major: the sampler's lane l reads word l of its stream
    const size_t S = (size_t)c->dims.n_streams;
    const int V = c->dims.vocab, words = (V + 31) / 32;
    if (S) {
        uint32_t *lm = new (std::nothrow) uint32_t[32 * S]();
        if (!lm) return ZONOS2CU_ENOMEM;
        for (size_t st = 0; st < S; st++)
            for (int t = 0; t < V; t++)
                if ((bits_host[st * words + (t >> 5)] >> (t & 31)) & 1u)
                    lm[st * 32 + ((t >> 2) & 31)] |= 1u << (4 * (t >> 7) + (t & 3));
        cudaError_t e = cudaSuccess;
        if (!c->allow) e = cudaMalloc(&c->allow, sizeof(uint32_t) * 32 * S);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(c->allow, lm, sizeof(uint32_t) * 32 * S, cudaMemcpyHostToDevice,
                                c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        delete[] lm;
        if (e != cudaSuccess) return cuda_fail(e, "allow upload");
    }
    c->allow_on = true;
    return ZONOS2CU_OK;
}

int zonos2cu_set_out_norm(zonos2cu_ctx *c, int enable, const float *weight_host, float eps)
{
    if (!c || c->dims.dim < 1) return ZONOS2CU_EINVAL;
    if (enable && (!(eps >= 0.0f) || !isfinite(eps))) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // no step may still be using the state
    if (!enable) {
        c->norm_on = false;
        return ZONOS2CU_OK;
    }
    const size_t D = (size_t)c->dims.dim;
    const size_t S2 = 2 * (size_t)c->dims.n_streams;   // rows with guidance on
    // the f32 head normalises into a copy (room for 2S rows covers every mode);
    // the bf16 head takes the rows' 1 / rms and, with a weight, a folded head
    if (!c->normed && n_rows(c) && (!c->head || c->head_dtype == ZONOS2CU_F32))
        Z2_CK(cudaMalloc(&c->normed, sizeof(float) * S2 * D));
    if (!c->row_rcp && n_rows(c)) Z2_CK(cudaMalloc(&c->row_rcp, sizeof(float) * S2));
    if (weight_host) {
        if (!c->norm_w) Z2_CK(cudaMalloc(&c->norm_w, sizeof(float) * D));
        Z2_CK(cudaMemcpyAsync(c->norm_w, weight_host, sizeof(float) * D, cudaMemcpyHostToDevice,
                              c->stream));
        Z2_CK(cudaStreamSynchronize(c->stream));
    }
    c->norm_has_w = weight_host != nullptr;
    c->norm_eps = eps;
    c->norm_on = true;
    return refold_head(c);
}

int zonos2cu_set_cfg(zonos2cu_ctx *c, int enable, float scale)
{
    if (!c || (enable && !isfinite(scale))) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // no step may still be using the state
    c->cfg_on = enable != 0;
    c->cfg_scale = scale;
    return ZONOS2CU_OK;
}

int zonos2cu_gen_begin(zonos2cu_ctx *c, int max_frames, int eoa_id, int audio_pad_id,
                       int text_pad_id)
{
    if (!c || max_frames < 1) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());   // no step may still be using the state
    const size_t S = (size_t)c->dims.n_streams, Cb = (size_t)c->dims.n_cb;
    const size_t need = S * (size_t)max_frames * Cb;
    if (need > c->gen_cap) {
        cudaFree(c->gen_frames);
        c->gen_frames = nullptr;
        c->gen_cap = 0;
        if (need) Z2_CK(cudaMalloc(&c->gen_frames, sizeof(int32_t) * need));
        c->gen_cap = need;
    }
    if (!c->gen_count && S) Z2_CK(cudaMalloc(&c->gen_count, sizeof(int32_t) * 2 * S));
    if (!c->gen_next && S) Z2_CK(cudaMalloc(&c->gen_next, sizeof(int32_t) * S * (Cb + 1)));
    if (S) {
        int32_t *h = new (std::nothrow) int32_t[S * (Cb + 1)];
        if (!h) return ZONOS2CU_ENOMEM;
        for (size_t s = 0; s < S; s++) {   // before the first frame: padding everywhere
            for (size_t cb = 0; cb < Cb; cb++) h[s * (Cb + 1) + cb] = audio_pad_id;
            h[s * (Cb + 1) + Cb] = text_pad_id;
        }
        cudaError_t e = cudaMemsetAsync(c->gen_count, 0, sizeof(int32_t) * S, c->stream);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(c->gen_count + S, 0xff, sizeof(int32_t) * S, c->stream);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(c->gen_frames, 0xff, sizeof(int32_t) * need, c->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(c->gen_next, h, sizeof(int32_t) * S * (Cb + 1),
                                cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        delete[] h;
        if (e != cudaSuccess) return cuda_fail(e, "generation state");
    }
    c->gen_max_frames = max_frames;
    c->gen_eoa = eoa_id;
    c->gen_pad = audio_pad_id;
    c->gen_text_pad = text_pad_id;
    c->gen_on = true;
    return ZONOS2CU_OK;
}

int zonos2cu_gen_end(zonos2cu_ctx *c)
{
    if (!c) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());
    c->gen_on = false;
    return ZONOS2CU_OK;
}

int zonos2cu_gen_read(zonos2cu_ctx *c, int32_t *frames_host, int32_t *n_frames_host,
                      int32_t *eos_at_host)
{
    if (!c || !c->gen_count) return ZONOS2CU_ESTATE;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());
    const size_t S = (size_t)c->dims.n_streams;
    if (frames_host && S)
        Z2_CK(cudaMemcpy(frames_host, c->gen_frames,
                         sizeof(int32_t) * S * (size_t)c->gen_max_frames * c->dims.n_cb,
                         cudaMemcpyDeviceToHost));
    if (n_frames_host && S)
        Z2_CK(cudaMemcpy(n_frames_host, c->gen_count, sizeof(int32_t) * S, cudaMemcpyDeviceToHost));
    if (eos_at_host && S)
        Z2_CK(cudaMemcpy(eos_at_host, c->gen_count + S, sizeof(int32_t) * S,
                         cudaMemcpyDeviceToHost));
    return ZONOS2CU_OK;
}

const int32_t *zonos2cu_gen_next_input(zonos2cu_ctx *c) { return c ? c->gen_next : nullptr; }

int zonos2cu_gen_shear_up(zonos2cu_ctx *c, int32_t *out_dev, void *stream)
{
    if (!c || !out_dev) return ZONOS2CU_EINVAL;
    if (!c->gen_count) return ZONOS2CU_ESTATE;
    DeviceGuard g(c->device);
    Z2_CK(z2::launch_shear_up(c->gen_frames, c->gen_count, c->dims.n_streams, c->gen_max_frames,
                              c->dims.n_cb, c->gen_pad, out_dev, (cudaStream_t)stream));
    return ZONOS2CU_OK;
}

int zonos2cu_set_embeddings(zonos2cu_ctx *c, const float *codebook_tables_host,
                            const float *text_table_host, int audio_vocab, int text_vocab)
{
    if (!c || !codebook_tables_host || !text_table_host || c->dims.dim < 1 || audio_vocab < 1 ||
        text_vocab < 0)
        return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    Z2_CK(cudaDeviceSynchronize());
    const size_t D = (size_t)c->dims.dim, Cb = (size_t)c->dims.n_cb;
    const size_t nb = sizeof(float) * Cb * (size_t)audio_vocab * D;
    const size_t tb = sizeof(float) * ((size_t)text_vocab + 1) * D;
    cudaFree(c->emb_cb);
    cudaFree(c->emb_text);
    c->emb_cb = nullptr;
    c->emb_text = nullptr;
    Z2_CK(cudaMalloc(&c->emb_cb, nb));
    Z2_CK(cudaMalloc(&c->emb_text, tb));
    Z2_CK(cudaMemcpyAsync(c->emb_cb, codebook_tables_host, nb, cudaMemcpyHostToDevice, c->stream));
    Z2_CK(cudaMemcpyAsync(c->emb_text, text_table_host, tb, cudaMemcpyHostToDevice, c->stream));
    Z2_CK(cudaStreamSynchronize(c->stream));
    c->emb_audio_vocab = audio_vocab;
    c->emb_text_vocab = text_vocab;
    return ZONOS2CU_OK;
}

int zonos2cu_gen_embed_next(zonos2cu_ctx *c, float *out_dev, void *stream)
{
    if (!c || !out_dev) return ZONOS2CU_EINVAL;
    if (!c->gen_next || !c->emb_cb) return ZONOS2CU_ESTATE;
    DeviceGuard g(c->device);
    Z2_CK(z2::launch_embed_frames(c->emb_cb, c->emb_text, c->dims.n_cb, c->emb_audio_vocab,
                                  c->emb_text_vocab, c->dims.dim, c->gen_next, c->dims.n_streams,
                                  out_dev, (cudaStream_t)stream));
    return ZONOS2CU_OK;
}

int zonos2cu_ctx_sample(zonos2cu_ctx *c, const float *logits_dev, long long row_stride,
                        const zonos2cu_sample_params *params, int delay_step, int32_t *codes_dev,
                        int32_t *flags_dev, void *stream)
{
    if (!c) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    const zonos2cu_dims &d = c->dims;
    int rc = check_rows(logits_dev, d.n_streams, d.n_cb, d.vocab, row_stride, c->rng, c->hist,
                        d.hist_len, c->hist_pos, codes_dev);
    if (rc) return rc;
    if ((rc = check_params(params, d.vocab))) return rc;
    const size_t rows = (size_t)d.n_streams * d.n_cb;
    if (!c->ahead_valid && d.n_streams) {   // this step's uniforms, once
        Z2_CK(z2::launch_draw_ahead(c->rng, c->rng_ahead, d.n_streams, d.n_cb,
                                    c->u_ahead + rows * c->ahead_par, (cudaStream_t)stream));
        c->ahead_valid = true;
    }
    rc = launch_rows(logits_dev, d.n_streams, d.n_cb, d.vocab, row_stride, params, c->rng,
                     c->hist, d.hist_len, c->hist_pos, c->allow_on ? c->allow : nullptr,
                     delay_step, codes_dev, flags_dev, (cudaStream_t)stream, c->counts,
                     c->presence, /*allow_lane_major*/ true, c->u_ahead + rows * c->ahead_par,
                     c->u_ahead + rows * (c->ahead_par ^ 1), c->rng_ahead);
    if (rc) {
        c->ahead_valid = false;
        return rc;
    }
    c->ahead_par ^= 1;
    if (c->gen_on)   // the generation loop keeps this step's frame
        Z2_CK(z2::launch_gen_append(codes_dev, d.n_streams, d.n_cb, d.vocab, c->gen_eoa,
                                    c->gen_text_pad, c->gen_max_frames, c->gen_frames,
                                    c->gen_count, c->gen_count + d.n_streams, c->gen_next,
                                    (cudaStream_t)stream));
    if (d.hist_len > 0) c->hist_pos = (c->hist_pos + 1) % d.hist_len;
    return ZONOS2CU_OK;
}

int zonos2cu_ctx_sample_host(zonos2cu_ctx *c, const float *logits_host, long long row_stride,
                             const zonos2cu_sample_params *params, int delay_step,
                             int32_t *codes_host, int32_t *flags_host)
{
    if (!c || !logits_host || !codes_host) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    const size_t rows = n_rows(c);
    if (row_stride < c->dims.vocab) return ZONOS2CU_EINVAL;
    int rc = check_params(params, c->dims.vocab);
    if (rc) return rc;
    if (rows == 0) return ZONOS2CU_OK;
    const size_t bytes = sizeof(float) * rows * (size_t)row_stride;
    if ((rc = grow((void **)&c->in_logits, &c->in_logits_bytes, bytes))) return rc;
    if ((rc = ensure_out(c))) return rc;
    Z2_CK(cudaMemcpyAsync(c->in_logits, logits_host, bytes, cudaMemcpyHostToDevice, c->stream));
    rc = zonos2cu_ctx_sample(c, c->in_logits, row_stride, params, delay_step, c->out,
                             c->out + rows, c->stream);
    if (rc) return rc;
    return finish_host_step(c, rows, codes_host, flags_host);
}

int zonos2cu_ctx_step(zonos2cu_ctx *c, const void *hidden_dev, zonos2cu_dtype dtype,
                      const zonos2cu_sample_params *params, int delay_step, int32_t *codes_dev,
                      int32_t *flags_dev, float *logits_out_dev, void *stream)
{
    if (!c || !hidden_dev) return ZONOS2CU_EINVAL;
    if (!c->head) return ZONOS2CU_ESTATE;
    if (dtype != c->head_dtype) return ZONOS2CU_EINVAL;
    DeviceGuard g(c->device);
    const zonos2cu_dims &d = c->dims;
    int rc = check_params(params, d.vocab);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    float *lg = logits_out_dev ? logits_out_dev : c->logits;
    const int rows_in = (c->cfg_on ? 2 : 1) * d.n_streams;
    const void *h = hidden_dev;
    const void *W = c->head;
    const float *row_scale = nullptr;
    if (c->norm_on && rows_in > 0) {   // rms_norm_per_token (src/zonos2_model.cpp:684-685)
        if (dtype == ZONOS2CU_BF16) {   // folded: the weight in W's columns, 1 / rms per row
            Z2_CK(z2::launch_row_rcp_rms(hidden_dev, rows_in, d.dim, c->norm_eps, c->row_rcp, st));
            if (c->norm_has_w) W = c->head_folded;
            row_scale = c->row_rcp;
        } else {                        // the exact restatement into a normalised copy
            Z2_CK(z2::launch_out_norm(hidden_dev, false, rows_in, d.dim, c->norm_eps,
                                      c->norm_has_w ? c->norm_w : nullptr, c->normed, st));
            h = c->normed;
        }
    }
    rc = launch_head(W, dtype, d.vocab, d.n_cb, d.vocab, d.dim, h, rows_in, 15.0f, lg, st,
                     c->cfg_on, c->cfg_scale, row_scale);
    if (rc) return rc;
    return zonos2cu_ctx_sample(c, lg, d.vocab, params, delay_step, codes_dev, flags_dev, st);
}

int zonos2cu_ctx_step_host(zonos2cu_ctx *c, const void *hidden_host, zonos2cu_dtype dtype,
                           const zonos2cu_sample_params *params, int delay_step,
                           int32_t *codes_host, int32_t *flags_host)
{
    if (!c || !hidden_host || !codes_host) return ZONOS2CU_EINVAL;
    if (!c->head) return ZONOS2CU_ESTATE;
    DeviceGuard g(c->device);
    const size_t rows = n_rows(c);
    if (rows == 0) return ZONOS2CU_OK;
    const size_t bytes = (dtype == ZONOS2CU_F32 ? 4 : 2) * (size_t)(c->cfg_on ? 2 : 1) *
                         (size_t)c->dims.n_streams * c->dims.dim;
    int rc = grow(&c->in_hidden, &c->in_hidden_bytes, bytes);
    if (rc) return rc;
    if ((rc = ensure_out(c))) return rc;
    Z2_CK(cudaMemcpyAsync(c->in_hidden, hidden_host, bytes, cudaMemcpyHostToDevice, c->stream));
    rc = zonos2cu_ctx_step(c, c->in_hidden, dtype, params, delay_step, c->out, c->out + rows,
                           nullptr, c->stream);
    if (rc) return rc;
    return finish_host_step(c, rows, codes_host, flags_host);
}

}  // extern "C"
