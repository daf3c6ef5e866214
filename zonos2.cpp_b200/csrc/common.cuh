// common.cuh -- shared helpers for the zonos2 B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace z2 {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- Xoshiro256** with the reference's output and transition
// (src/zonos2_generate.cpp:20-32).
__device__ __forceinline__ uint64_t rotl64(uint64_t x, int k)
{
    return (x << k) | (x >> (64 - k));
}

struct Xo256 {
    uint64_t s0, s1, s2, s3;
    __device__ __forceinline__ uint64_t next()
    {
        const uint64_t out = rotl64(s1 * 5u, 7) * 9u;
        const uint64_t t = s1 << 17;
        s2 ^= s0;
        s3 ^= s1;
        s1 ^= s2;
        s0 ^= s3;
        s2 ^= t;
        s3 = rotl64(s3, 45);
        return out;
    }
    // 53-bit double in [0, 1) narrowed to float with round-to-nearest, as the
    // reference's implicit double -> float conversion does.
    __device__ __forceinline__ float randf()
    {
        return __double2float_rn((double)(next() >> 11) * 0x1.0p-53);
    }
};

}  // namespace z2
