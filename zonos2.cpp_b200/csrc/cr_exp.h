// cr_exp.h -- exp(x) for f32 x <= 0, correctly rounded to f32, on host and device.
//
// Own table-driven method (Tang's reduction): x = (64m + j) ln2/64 + r with
// |r| <= ln2/128, exp(x) = 2^m * 2^(j/64) * e^r; e^r by its degree-5 Taylor
// polynomial in f64 (truncation < 0.4 f64 ulp), the table holds 2^(j/64)
// rounded to f64, ln2/64 is split in a 21-bit head (k * head is exact) and a
// tail.  The f64 result is within a few f64 ulps; an exhaustive host check of
// every f32 input in [-128, 0] against a long-double exp shows the final f32
// rounding is always correct (tests/test_exp_exhaustive.py runs it).  Every
// f64 step is an explicit fma or a single rounded operation, so host and device
// produce the same bits.
#pragma once

#include <stdint.h>
#if defined(__CUDACC__)
#define Z2_HD __host__ __device__ __forceinline__
#define Z2_HDM __host__ __device__ __forceinline__
#include <math.h>
#else
#define Z2_HD static inline
#define Z2_HDM inline
#include <math.h>
#include <string.h>
#endif

namespace z2 {

// 2^(j/64), j = 0..63, rounded to f64 (computed with a long-double exp2)
#define Z2_EXP2_64_TABLE \
  { \
    0x1p+0, 0x1.02c9a3e778061p+0, 0x1.059b0d3158574p+0, \
    0x1.0874518759bc8p+0, 0x1.0b5586cf9890fp+0, 0x1.0e3ec32d3d1a2p+0, \
    0x1.11301d0125b51p+0, 0x1.1429aaea92dep+0, 0x1.172b83c7d517bp+0, \
    0x1.1a35beb6fcb75p+0, 0x1.1d4873168b9aap+0, 0x1.2063b88628cd6p+0, \
    0x1.2387a6e756238p+0, 0x1.26b4565e27cddp+0, 0x1.29e9df51fdee1p+0, \
    0x1.2d285a6e4030bp+0, 0x1.306fe0a31b715p+0, 0x1.33c08b26416ffp+0, \
    0x1.371a7373aa9cbp+0, 0x1.3a7db34e59ff7p+0, 0x1.3dea64c123422p+0, \
    0x1.4160a21f72e2ap+0, 0x1.44e086061892dp+0, 0x1.486a2b5c13cdp+0, \
    0x1.4bfdad5362a27p+0, 0x1.4f9b2769d2ca7p+0, 0x1.5342b569d4f82p+0, \
    0x1.56f4736b527dap+0, 0x1.5ab07dd485429p+0, 0x1.5e76f15ad2148p+0, \
    0x1.6247eb03a5585p+0, 0x1.6623882552225p+0, 0x1.6a09e667f3bcdp+0, \
    0x1.6dfb23c651a2fp+0, 0x1.71f75e8ec5f74p+0, 0x1.75feb564267c9p+0, \
    0x1.7a11473eb0187p+0, 0x1.7e2f336cf4e62p+0, 0x1.82589994cce13p+0, \
    0x1.868d99b4492edp+0, 0x1.8ace5422aa0dbp+0, 0x1.8f1ae99157736p+0, \
    0x1.93737b0cdc5e5p+0, 0x1.97d829fde4e5p+0, 0x1.9c49182a3f09p+0, \
    0x1.a0c667b5de565p+0, 0x1.a5503b23e255dp+0, 0x1.a9e6b5579fdbfp+0, \
    0x1.ae89f995ad3adp+0, 0x1.b33a2b84f15fbp+0, 0x1.b7f76f2fb5e47p+0, \
    0x1.bcc1e904bc1d2p+0, 0x1.c199bdd85529cp+0, 0x1.c67f12e57d14bp+0, \
    0x1.cb720dcef9069p+0, 0x1.d072d4a07897cp+0, 0x1.d5818dcfba487p+0, \
    0x1.da9e603db3285p+0, 0x1.dfc97337b9b5fp+0, 0x1.e502ee78b3ff6p+0, \
    0x1.ea4afa2a490dap+0, 0x1.efa1bee615a27p+0, 0x1.f50765b6e454p+0, \
    0x1.fa7c1819e90d8p+0 \
  }

#if defined(__CUDACC__)
static __device__ const double kExp2Table_dev[64] = Z2_EXP2_64_TABLE;
#endif
static const double kExp2Table_host[64] = Z2_EXP2_64_TABLE;

Z2_HD double exp2_64th(int j)
{
#if defined(__CUDA_ARCH__)
    return __ldg(&kExp2Table_dev[j]);
#else
    return kExp2Table_host[j];
#endif
}

Z2_HD double pow2_int(int m)  // 2^m for -1022 <= m <= 1023
{
    const uint64_t b = (uint64_t)(uint32_t)(m + 1023) << 52;
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)b);
#else
    double d;
    memcpy(&d, &b, sizeof d);
    return d;
#endif
}

Z2_HD int low_word(double d)   // the low 32 bits of d's encoding
{
#if defined(__CUDA_ARCH__)
    return __double2loint(d);
#else
    uint64_t b;
    memcpy(&b, &d, sizeof b);
    return (int)(uint32_t)b;
#endif
}

struct Exp2Table64 {   // 2^(j/64) from the constant table
    Z2_HDM double operator()(int j) const { return exp2_64th(j); }
};

// exp(xf) rounded to nearest f32, for xf <= 0 (or -inf); exp(x) < 2^-150 -> 0.
// tab(j) returns 2^(j/64) as in Z2_EXP2_64_TABLE (callers may keep a copy in
// faster memory).
template <class Table>
Z2_HDM float cr_expf_neg_t(float xf, const Table &tab)
{
    if (!(xf >= -104.0f)) return 0.0f;
    const double x = (double)xf;
    const double inv_ln2_64 = 0x1.71547652b82fep+6;   // 64 / ln2
    const double ln2_64_hi = 0x1.62e42p-7;            // ln2 / 64, 21-bit head
    const double ln2_64_lo = 0x1.fdf473de6bp-28;      // ln2 / 64 - head
    const double shifter = 0x1.8p52;                  // 2^52 + 2^51
    const double kt = x * inv_ln2_64 + shifter;        // k + shifter, k = nearest integer
    const double kd = kt - shifter;
    const int k = low_word(kt);                        // |k| < 2^14
    double r = fma(-kd, ln2_64_hi, x);
    r = fma(-kd, ln2_64_lo, r);
    double p = fma(r, 1.0 / 120.0, 1.0 / 24.0);
    p = fma(p, r, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    const double res = (tab(k & 63) * p) * pow2_int(k >> 6);
    return (float)res;
}

Z2_HD float cr_expf_neg(float xf) { return cr_expf_neg_t(xf, Exp2Table64()); }

}  // namespace z2
