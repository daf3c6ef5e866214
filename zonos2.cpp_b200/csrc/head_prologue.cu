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
// first and the result is rounded back to bf16 for the tensor-core head when
// the norm has no weight to fold.  With a weight, the bf16 head takes the
// weight folded into its columns (fold_columns_kernel, once) and the rows'
// 1 / rms (row_rcp_rms_kernel, per step) in its epilogue: no normalised copy of
// the hidden states is written or read.
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

// One warp per bf16 row: the sum of squares (lanes take eight elements at a
// time, then a shuffle tree; the bf16 path is held to its stated tolerance,
// not to the reference's order of additions), rms = sqrt(ss / dim + eps),
// rcp = 1 / rms.
__global__ void __launch_bounds__(32 * kNormWarps)
    row_rcp_rms_kernel(const __nv_bfloat16 *__restrict__ x, int rows, int dim, float eps,
                       float *__restrict__ rcp)
{
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const __nv_bfloat16 *xr = x + (size_t)row * dim;
    float ss = 0.0f;
    if (dim % 8 == 0 && ((uintptr_t)xr & 15u) == 0) {
        for (int d = 8 * lane; d < dim; d += 256) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(xr + d));
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float a = __uint_as_float(w4[k] << 16), b = __uint_as_float(w4[k] & 0xffff0000u);
                ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)));
            }
        }
    } else {
        for (int d = lane; d < dim; d += 32) {
            const float a = __bfloat162float(xr[d]);
            ss = __fadd_rn(ss, __fmul_rn(a, a));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(kFull, ss, o));
    if (lane == 0) rcp[row] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(ss, (float)dim), eps)));
}

// W'[r][k] = bf16(W[r][k] * w[k]), one thread per element.
__global__ void fold_columns_kernel(const __nv_bfloat16 *__restrict__ W, const float *__restrict__ w,
                                    long long n, int dim, __nv_bfloat16 *__restrict__ out)
{
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int k = (int)(i % dim);
    out[i] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(W[i]), __ldg(w + k)));
}

}  // namespace

cudaError_t launch_row_rcp_rms(const void *x, int rows, int dim, float eps, float *rcp,
                               cudaStream_t stream)
{
    if (rows == 0) return cudaSuccess;
    const unsigned blocks = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
    row_rcp_rms_kernel<<<blocks, 32 * kNormWarps, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(x), rows, dim, eps, rcp);
    return cudaGetLastError();
}

cudaError_t launch_fold_columns(const void *W, const float *w, int rows, int dim, void *out,
                                cudaStream_t stream)
{
    const long long n = (long long)rows * dim;
    if (n == 0) return cudaSuccess;
    fold_columns_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16 *>(W), w, n, dim, static_cast<__nv_bfloat16 *>(out));
    return cudaGetLastError();
}

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
