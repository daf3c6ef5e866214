// head_tc.cu -- bf16 output head + softcap on the tcgen05 tensor cores (sm_100a).
#include "common.cuh"
#include "head.cuh"

namespace z2 {

__device__ int g_device_error = 0;

int read_and_clear_device_error(int *value)
{
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
    if (e != cudaSuccess) return (int)e;
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return (int)e;
    *value = v;
    return 0;
}

cudaError_t launch_head_tc_bf16(const HeadArgs &, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace z2
