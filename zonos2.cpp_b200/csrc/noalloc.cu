// noalloc.cu -- zonos2cu_step_noalloc: the fused decode step without any
// device allocation, for callers that may not allocate (their device memory
// is owned by another framework's pool, or they decode under real-time
// constraints where an allocation could block the device).
//
// The head writes its logits into a fixed array compiled into the library
// instead of a caller or context buffer; the sampler reads them from there.
// The array's device address is looked up once per device, on the first
// call, with that device current.  Every call shares the array, so calls
// whose work overlaps on the GPU race; nothing in it has to start at zero
// (the head overwrites every logit the sampler reads).
#include <mutex>

#include "zonos2_cuda.h"

namespace {

static __device__ __align__(256) float g_noalloc_logits[ZONOS2CU_NOALLOC_MAX_LOGITS];

struct ScratchAddr {
    std::mutex mu;
    float *dev[64] = {};
};
ScratchAddr g_addr;

// The array's device address on the current device (set up on first use).
int scratch_on_current_device(float **out)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return ZONOS2CU_ECUDA;
    std::lock_guard<std::mutex> lock(g_addr.mu);
    if (!g_addr.dev[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_logits) != cudaSuccess || !p) return ZONOS2CU_ECUDA;
        g_addr.dev[dev] = static_cast<float *>(p);
    }
    *out = g_addr.dev[dev];
    return ZONOS2CU_OK;
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
    if (n_streams < 0 || n_cb < 1 || vocab < 1) return ZONOS2CU_EINVAL;
    if ((long long)n_streams * n_cb * vocab > (long long)ZONOS2CU_NOALLOC_MAX_LOGITS)
        return ZONOS2CU_ETOOBIG;
    if (n_streams == 0) return ZONOS2CU_OK;
    float *logits = nullptr;
    int rc = scratch_on_current_device(&logits);
    if (rc) return rc;
    rc = zonos2cu_head_softcap(W_dev, dtype, rows_per_cb, n_cb, vocab, dim, hidden_dev, n_streams,
                               softcap, logits, stream);
    if (rc) return rc;
    return zonos2cu_sample_rows(logits, n_streams, n_cb, vocab, vocab, params, rng_dev, hist_dev,
                                hist_len, hist_pos, allow_dev, delay_step, codes_dev, flags_dev,
                                stream);
}
