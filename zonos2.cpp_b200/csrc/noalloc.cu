// noalloc.cu -- zonos2cu_step_noalloc: the fused decode step without any
// device allocation, for callers that may not allocate (their device memory
// is owned by another framework's pool, or they decode under real-time
// constraints where an allocation could block the device).
//
// The head writes its logits into a fixed array compiled into the library
// instead of a caller or context buffer; the sampler reads them from there.
// Every call shares the array, so calls whose work overlaps on the GPU race;
// nothing in it has to start at zero (the head overwrites every logit the
// sampler reads).
//
// The array's device address belongs to the CUDA context current at the call.
// Outside stream capture every call looks it up again (cudaGetSymbolAddress
// allocates nothing), so a context made after cudaDeviceReset, or a different
// context made current on the same device, gets its own address.  Under
// capture no lookup is made: the address recorded by the last call outside
// capture in the same context is used, and a context that has never made one
// gets ZONOS2CU_ESTATE.
#include <cuda.h>

#include <mutex>

#include "zonos2_cuda.h"

int z2_check_head_then_sample(const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb, int n_cb,
                              int vocab, int dim, const void *hidden_dev, int n_streams,
                              float softcap, const float *logits_dev,
                              const zonos2cu_sample_params *params, uint64_t *rng_dev,
                              int32_t *hist_dev, int hist_len, int hist_pos, int32_t *codes_dev);

namespace {

static __device__ __align__(256) float g_noalloc_logits[ZONOS2CU_NOALLOC_MAX_LOGITS];

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

struct ScratchAddr {
    std::mutex mu;
    bool looked_up = false;
    CtxGetCurrentFn ctx_get_current = nullptr;
    struct Entry {
        CUcontext ctx;
        float *addr;
    };
    Entry seen[64] = {};   // the address last found in each context, most recent first
    int n_seen = 0;
};
ScratchAddr g_addr;

// The context current on this thread (null if the driver entry point is missing).
CUcontext current_context()
{
    if (!g_addr.looked_up) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_addr.ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
        g_addr.looked_up = true;
    }
    CUcontext c = nullptr;
    if (!g_addr.ctx_get_current || g_addr.ctx_get_current(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// The array's device address in the current context.
int scratch_in_current_context(cudaStream_t stream, float **out)
{
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
        (void)cudaGetLastError();   // reported here: not left for the next launch
        return ZONOS2CU_ECUDA;
    }
    std::lock_guard<std::mutex> lock(g_addr.mu);
    const CUcontext ctx = current_context();
    if (cap == cudaStreamCaptureStatusNone) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_logits) != cudaSuccess || !p) {
            (void)cudaGetLastError();
            return ZONOS2CU_ECUDA;
        }
        *out = static_cast<float *>(p);
        if (!ctx) return ZONOS2CU_OK;
        int i = 0;   // record it, most recent first
        while (i < g_addr.n_seen && g_addr.seen[i].ctx != ctx) i++;
        if (i == g_addr.n_seen && g_addr.n_seen < 64) g_addr.n_seen++;
        if (i == 64) i = 63;   // forget the oldest context
        for (; i > 0; i--) g_addr.seen[i] = g_addr.seen[i - 1];
        g_addr.seen[0] = {ctx, *out};
        return ZONOS2CU_OK;
    }
    for (int i = 0; ctx && i < g_addr.n_seen; i++)
        if (g_addr.seen[i].ctx == ctx) {
            *out = g_addr.seen[i].addr;
            return ZONOS2CU_OK;
        }
    return ZONOS2CU_ESTATE;
}

}  // namespace

extern "C" int zonos2cu_step_noalloc(const void *W_dev, zonos2cu_dtype dtype, int rows_per_cb,
                                     int n_cb, int vocab, int dim, const void *hidden_dev,
                                     int n_streams, float softcap,
                                     const zonos2cu_sample_params *params, uint64_t *rng_dev,
                                     int32_t *hist_dev, int hist_len, int hist_pos,
                                     const uint32_t *allow_dev, int delay_step, int32_t *codes_dev,
                                     int32_t *flags_dev, void *stream)
{
    // Every argument is checked before anything is launched: an invalid sampler
    // argument must not cost a head launch, nor overwrite the shared array.  The
    // array's address stands in for the logits buffer (it is never null).
    const float *placeholder = reinterpret_cast<const float *>(256);
    int rc = z2_check_head_then_sample(W_dev, dtype, rows_per_cb, n_cb, vocab, dim, hidden_dev,
                                       n_streams, softcap, placeholder, params, rng_dev, hist_dev,
                                       hist_len, hist_pos, codes_dev);
    if (rc) return rc;
    if ((long long)n_streams * n_cb * vocab > (long long)ZONOS2CU_NOALLOC_MAX_LOGITS)
        return ZONOS2CU_ETOOBIG;
    if (n_streams == 0) return ZONOS2CU_OK;
    float *logits = nullptr;
    rc = scratch_in_current_context((cudaStream_t)stream, &logits);
    if (rc) return rc;
    rc = zonos2cu_head_softcap(W_dev, dtype, rows_per_cb, n_cb, vocab, dim, hidden_dev, n_streams,
                               softcap, logits, stream);
    if (rc) return rc;
    return zonos2cu_sample_rows(logits, n_streams, n_cb, vocab, vocab, params, rng_dev, hist_dev,
                                hist_len, hist_pos, allow_dev, delay_step, codes_dev, flags_dev,
                                stream);
}
