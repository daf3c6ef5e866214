// head_prologue.cu -- the output RMSNorm ahead of the head (sm_100a).
//
// Restates rms_norm_per_token (src/zonos2_model.cpp:19-35), which the
// reference applies to the last hidden states before the multi_output head
// (src/zonos2_model.cpp:684-685): per row, the f32 sum of squares in index
// order, rms = sqrt(ss / dim + eps), rcp = 1 / rms, then x * rcp * w.  One
// warp per row: lane 0 accumulates the sum term by term in the reference's
// order (the other lanes have nothing to add without changing its rounding),
// then the warp writes the normalised row.  Built with -fmad=false, so every
// operation rounds where the reference's does; bf16 rows are widened to f32
// first and the result is rounded back to bf16 for the tensor-core head.
#include <cuda_bf16.h>
#include <math.h>

#include "common.cuh"
#include "head.cuh"

namespace z2 {

namespace {

constexpr int kNormWarps = 4;

__device__ __forceinline__ float load_f(const float *p) { return __ldg(p); }
__device__ __forceinline__ float load_f(const __nv_bfloat16 *p)
{
    return __bfloat162float(*p);
}
__device__ __forceinline__ void store_f(float *p, float v) { *p = v; }
__device__ __forceinline__ void store_f(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(32 * kNormWarps)
    out_norm_kernel(const T *__restrict__ x, int rows, int dim, float eps,
                    const float *__restrict__ w, T *__restrict__ y)
{
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const T *xr = x + (size_t)row * dim;
    float rcp = 0.0f;
    if (lane == 0) {
        float ss = 0.0f;
        int d = 0;
        for (; d + 4 <= dim; d += 4) {   // four independent loads, one chain of adds
            const float a = load_f(xr + d), b = load_f(xr + d + 1);
            const float c = load_f(xr + d + 2), e = load_f(xr + d + 3);
            ss = __fadd_rn(ss, __fmul_rn(a, a));
            ss = __fadd_rn(ss, __fmul_rn(b, b));
            ss = __fadd_rn(ss, __fmul_rn(c, c));
            ss = __fadd_rn(ss, __fmul_rn(e, e));
        }
        for (; d < dim; d++) {
            const float a = load_f(xr + d);
            ss = __fadd_rn(ss, __fmul_rn(a, a));
        }
        const float rms = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)dim), eps));
        rcp = __fdiv_rn(1.0f, rms);
    }
    rcp = __shfl_sync(kFull, rcp, 0);
    T *yr = y + (size_t)row * dim;
    for (int d = lane; d < dim; d += 32) {
        const float v = __fmul_rn(load_f(xr + d), rcp);
        store_f(yr + d, w ? __fmul_rn(v, __ldg(w + d)) : v);
    }
}

}  // namespace

cudaError_t launch_out_norm(const void *x, bool bf16, int rows, int dim, float eps,
                            const float *w, void *y, cudaStream_t stream)
{
    if (rows == 0) return cudaSuccess;
    const unsigned blocks = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
    if (bf16)
        out_norm_kernel<__nv_bfloat16><<<blocks, 32 * kNormWarps, 0, stream>>>(
            static_cast<const __nv_bfloat16 *>(x), rows, dim, eps, w,
            static_cast<__nv_bfloat16 *>(y));
    else
        out_norm_kernel<float><<<blocks, 32 * kNormWarps, 0, stream>>>(
            static_cast<const float *>(x), rows, dim, eps, w, static_cast<float *>(y));
    return cudaGetLastError();
}

}  // namespace z2
