// sampler.cu -- fused per-row sampler for the zonos2 decode step (sm_100a).
//
// Restates, per (stream, codebook) row, the reference's sample_token
// (src/zonos2_generate.cpp:36-93) fed through the build-defined prologue
// (repetition penalty over the history window, allow bitmask, delay-pattern
// forcing, non-finite guard), with the row's uniform drawn from a per-stream
// Xoshiro256** in codebook order (src/zonos2_generate.cpp:259-267).
//
// sample_rows_kernel is persistent: one CTA of 28 warps per SM, whose warps
// take the SM's rows from a shared counter; no warp waits for another.  The
// uniforms come one of two ways:
//  - the decode context draws them one step ahead: warp 0 of each CTA draws the
//    next step's uniforms for a slice of streams, so a step is one launch (the
//    first step after the generators are set is preceded by draw_ahead_kernel);
//    the kernel runs under programmatic dependent launch and waits for the grid
//    before it at its start, so only its launch overlaps that grid's tail;
//  - otherwise draw_uniforms_kernel (one thread per stream) draws the stream's
//    n_cb uniforms in codebook order, advances its generator and parks each
//    uniform in the row's code slot, and the sampler, launched behind it under
//    programmatic dependent launch, waits for it only before it first reads a
//    uniform.
//
// Per row: one bulk copy (TMA) lands the logits in the warp's shared memory
// while the warp finishes its previous row.  Lane l holds slots
// 4*(l + 32*j) + e, j < 8, e < 4, so every access is a conflict-free 128-bit
// one, and a lane-major bitmap (word l, bit 4*j + e) gives a lane all its mask
// bits in one load; the decode context keeps its history set and allow mask in
// that layout.  After the prologue and the row max, a 128-bucket histogram of
// the gap (max - l), in buckets T/8 wide (the last one open-ended), finds the
// bucket B* holding the k-th largest logit.  Buckets <= B*+1 are the
// candidates: a superset of the top-k that also holds every logit whose
// probability could round equal to the k-th one's (equal probabilities need
// logits far closer than a bucket).  In the common case (<= 128 candidates)
// they are scattered in bucket order as 32-bit keys, four per lane, and sorted
// in registers; the decisions are certified on fixed-point prefix sums of
// hardware-exp2 probabilities against the reference's own error margins, and
// the rows no margin settles take an exact form out of line (exact
// probabilities, f64 prefix sums, and where those cannot decide either, the
// reference's f32 running sums term by term).  Other rows (top-k off, > 128
// candidates) take a slower general path; delay-forced rows return the pad
// token once the row has been checked for non-finite logits.
//
// Exactness: the token is the one the reference's own f32 operations give --
// (l - max) / T, exp rounded correctly to f32, sums accumulated one term at a
// time in sorted order, p / sum divisions, the CDF walk -- either because a
// certified margin shows the decision cannot differ or because those
// operations are carried out as written; so for equal inputs the token equals
// the reference's up to (a) equal-probability ties, taken in ascending token
// order, and (b) the reference's expf being misrounded by one ulp (glibc, on
// about 1e-4 of its inputs).  (l - max) / T is computed as an f64 product
// with RN(1/T) rounded to f32: the f64 error (< 2^-52 relative) cannot reach
// an f32 rounding boundary, which a quotient of two f32 values never comes
// closer to than 2^-48 relative, nor hits exactly.  Compiled with -fmad=false:
// no multiply-add is contracted (the one explicit fma places a logit in a
// bucket, which decides no token).
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "cr_exp.h"
#include "sampler.cuh"

namespace z2 {

__device__ int g_sampler_error = 0;

int read_and_clear_sampler_error(int *value)
{
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_sampler_error, sizeof(int));
    if (e != cudaSuccess) return (int)e;
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_sampler_error, &zero, sizeof(int));
    if (e != cudaSuccess) return (int)e;
    *value = v;
    return 0;
}

namespace {

// Per-warp shared-memory region (bytes).  Common path:
//   [0, 4096)      the row: the bulk copy lands the logits, the prologue
//                  rewrites them in place; free once the candidates are
//                  compacted (the next row's copy lands here meanwhile)
//   [4096, 5120)   the bucket byte of every slot (a scanned history's
//                  seen-bytes during the prologue), then the sorted keys
//   [5120, 5632)   128 bucket counters, then the sorted probabilities
//   [5632, 6656)   compacted candidates (logit, token); after the sort the
//                  prefix sums [5632, 6144) and p / sum [6144, 6656)
//   [8192, 8200)   the row copy's mbarrier
// General path: up to 1024 keys over [0, 8192) (no copy is in flight then).
constexpr int kRegion = 8192;
constexpr int kWarpStride = kRegion + 16;
constexpr int kCtaHeader = 528;          // 2^(j/64), j < 64, shared by the CTA's warps; the item counter
constexpr int kCtrOffset = 512;
constexpr int kRowOffset = 0;
constexpr int kBktOffset = 4096;
constexpr int kKeysOffset = 4096;
constexpr int kHistOffset = 5120;
constexpr int kPsOffset = 5120;
constexpr int kStageOffset = 5632;
constexpr int kPfOffset = 5632;
constexpr int kQOffset = 6144;
constexpr int kBarOffset = kRegion;
constexpr int kBuckets = 128;    // gap buckets: 0..126 finite, 127 marks a masked slot
constexpr int kRegSortMax = 128; // candidates sorted in registers (four per lane)
constexpr int kWarps = 28;      // warps per CTA: one CTA per SM, so the rows of a whole SM are
                                // shared out by one counter (9-warp CTAs, three per SM, left
                                // more of the SM idle at the end of a launch)
constexpr int kCtasPerSm = 1;   // shared memory and <= 72 registers
constexpr unsigned long long kWaitNs = 2000000000ull;

enum : int { kErrTimeout = 1 };

__device__ __forceinline__ uint64_t make_key(float p, int tok)
{
    return ((uint64_t)__float_as_uint(p) << 32) | (uint64_t)(0xffffffffu - (uint32_t)tok);
}
__device__ __forceinline__ float key_p(uint64_t k) { return __uint_as_float((uint32_t)(k >> 32)); }
__device__ __forceinline__ int key_tok(uint64_t k) { return (int)(0xffffffffu - (uint32_t)k); }
__device__ __forceinline__ uint64_t make_ent(float v, int tok)
{
    return ((uint64_t)__float_as_uint(v) << 32) | (uint32_t)tok;
}
__device__ __forceinline__ float ent_v(uint64_t e) { return __uint_as_float((uint32_t)(e >> 32)); }

// The slot -> token map of the register layout.
__device__ __forceinline__ int slot_token(int lane, int i)
{
    return 4 * (lane + 32 * (i >> 2)) + (i & 3);
}

// Word and bit of token t in a lane-major 1024-bit map.
__device__ __forceinline__ int lm_word(int t) { return (t >> 2) & 31; }
__device__ __forceinline__ uint32_t lm_bit(int t) { return 1u << (4 * (t >> 7) + (t & 3)); }

__device__ __forceinline__ int warp_incl_scan(int x, int lane)
{
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    return x;
}

struct SmemExpTable {
    const double *t;
    __device__ __forceinline__ double operator()(int j) const { return t[j]; }
};

// p = exp((l - max) / T) exactly as the reference rounds it (see the header).
template <class Table>
__device__ __forceinline__ float row_prob(float l, float M, double inv_temp, const Table &tab)
{
    return cr_expf_neg_t(__double2float_rn((double)__fsub_rn(l, M) * inv_temp), tab);
}

// The build-defined prologue of one logit (slot i of this lane): non-finite
// guard, repetition penalty (a factor of exactly 1 when the token is unseen),
// allow / delay mask.
__device__ __forceinline__ float prologue(float x, int i, uint32_t seenm, uint32_t allowm,
                                          float rho, float inv_rho)
{
    const bool fin = x < INFINITY;  // false for NaN and +inf
    const float f = ((seenm >> i) & 1u) ? (x > 0.0f ? inv_rho : rho) : 1.0f;
    return (fin && ((allowm >> i) & 1u)) ? __fmul_rn(x, f) : -INFINITY;
}

// Gap bucket of a logit: u = sat(fma(-v, s, max * s)) in [0, 1] with
// s = 1 / (126 * width), and the bucket is round(126 u), read from the low byte
// of 126 u + 2^23 (the histogram does this two slots at a time); -inf and gaps
// past 126 widths land in 126, the open-ended last bucket.  The saturating fma
// clamps on the fma pipe.  The scatter's sort key carries the same coordinate
// 126 u + 1/2 rounded to a multiple of 2^-15 (an integer below 2^22, monotone
// non-increasing in v) and recomputes the bucket bit for bit.

// a * b + c on both halves, each saturated to [0, 1] (the packed f32x2 fma has
// no saturating form, so two scalar ones: still the fma pipe, not the ALU's)
__device__ __forceinline__ float2 ffma2_sat(float2 a, float2 b, float2 c)
{
    float2 d;
    asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d.x) : "f"(a.x), "f"(b.x), "f"(c.x));
    asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d.y) : "f"(a.y), "f"(b.y), "f"(c.y));
    return d;
}

// Bit e of the result is set iff byte e of pk is <= bc (bytes and bc < 128).
__device__ __forceinline__ uint32_t bytes_le(uint32_t pk, uint32_t bc4)
{
    const uint32_t le = ((bc4 - pk) & 0x80808080u) >> 7;
    return (le * 0x10204080u) >> 28;
}

__device__ __forceinline__ void mark_seen(unsigned char *seen, int t, int vocab)
{
    if ((unsigned)t < (unsigned)vocab) seen[t] = 1;
}

// ---- bulk copy, mbarrier, programmatic launch
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// The whole warp waits for the phase with this parity; false (warp-uniform,
// error word set) after ~2 s.
__device__ __noinline__ bool mbar_wait_warp_slow(uint32_t bar, uint32_t parity, int lane)
{
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; it++) {
        if (__all_sync(kFull, mbar_try_wait(bar, parity))) return true;
        if ((it & 255u) == 0u &&
            __shfl_sync(kFull, (int)(globaltimer_ns() - t0 > kWaitNs), 0)) {
            if (lane == 0) atomicCAS(&g_sampler_error, 0, kErrTimeout);
            return false;
        }
    }
}
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, int lane)
{
    if (__all_sync(kFull, mbar_try_wait(bar, parity))) return true;
    return mbar_wait_warp_slow(bar, parity, lane);
}
// One bulk copy global -> this CTA's shared memory, completing on `bar`
// (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(dst), "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// Orders this warp's earlier generic accesses to its region before the next
// bulk copy writes it.
__device__ __forceinline__ void fence_proxy_async()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Descending bitonic sort of n (power of two, <= 1024) keys in shared memory.
__device__ __noinline__ void bitonic_smem_desc(uint64_t *keys, int n, int lane)
{
    for (int size = 2; size <= n; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int q = lane; q < (n >> 1); q += 32) {
                const int i = 2 * q - (q & (stride - 1));
                const int j = i + stride;
                const uint64_t x = keys[i], y = keys[j];
                const bool desc = (i & size) == 0;
                if (desc ? (x < y) : (x > y)) {
                    keys[i] = y;
                    keys[j] = x;
                }
            }
            __syncwarp();
        }
}

// Sequential f32 sum of the probabilities of keys[0..m), one term at a time.
__device__ float seq_sum(const uint64_t *keys, int m)
{
    float s = 0.0f;
    int i = 0;
    for (; i + 2 <= m; i += 2) {
        const ulonglong2 kk = *reinterpret_cast<const ulonglong2 *>(keys + i);
        s += key_p(kk.x);
        s += key_p(kk.y);
    }
    if (i < m) s += key_p(keys[i]);
    return s;
}

// Running f32 prefix sums pf[i] = ps[0] + ... + ps[i], one term at a time (one lane).
__device__ __forceinline__ void prefix_sums(const float *ps, float *pf, int m)
{
    float P = 0.0f;
    int i = 0;
#pragma unroll 2
    for (; i + 4 <= m; i += 4) {
        const float4 p4 = *reinterpret_cast<const float4 *>(ps + i);
        float4 o;
        P += p4.x;
        o.x = P;
        P += p4.y;
        o.y = P;
        P += p4.z;
        o.z = P;
        P += p4.w;
        o.w = P;
        *reinterpret_cast<float4 *>(pf + i) = o;
    }
    for (; i < m; i++) {
        P += ps[i];
        pf[i] = P;
    }
}

// 1 + the first i < len whose running sum of ps[j] / S (j <= i, accumulated in
// order in f32) is >= thr; -1 if none.  The warp divides 32 terms at a time
// into q, lane 0 accumulates them.
__device__ __noinline__ int walk_cdf(const float *ps, float *q, int len, float S, float thr,
                                     int lane)
{
    float cum = 0.0f;
    for (int base = 0; base < len; base += 32) {
        const int e = min(base + 32, len);
        if (base + lane < e) q[base + lane] = ps[base + lane] / S;
        __syncwarp();
        int hit = -1;
        if (lane == 0) {
            int k = base;
            for (; k + 4 <= e; k += 4) {
                const float4 qq = *reinterpret_cast<const float4 *>(q + k);
                const float c0 = cum + qq.x, c1 = c0 + qq.y, c2 = c1 + qq.z, c3 = c2 + qq.w;
                if (c3 >= thr) {
                    hit = c0 >= thr ? k + 1 : c1 >= thr ? k + 2 : c2 >= thr ? k + 3 : k + 4;
                    break;
                }
                cum = c3;
            }
            if (hit < 0)
                for (; k < e; k++) {
                    cum += q[k];
                    if (cum >= thr) {
                        hit = k + 1;
                        break;
                    }
                }
        }
        hit = __shfl_sync(kFull, hit, 0);
        if (hit > 0) return hit;
    }
    return -1;
}

// First index i < mm with !(p_i / S >= thresh) (the min-p cut), mm if none.
__device__ __forceinline__ int minp_cut(const float *ps, int mm, float S, float thresh, int lane)
{
    for (int base = 0; base < mm; base += 32) {
        const int i = base + lane;
        const uint32_t fails = __ballot_sync(kFull, i < mm && !(ps[i] / S >= thresh));
        if (fails) return base + __ffs(fails) - 1;
    }
    return mm;
}

// The (want)-th token, in token order, outside the positive set of a row
// (keys[0..n_pos)); -1 if there is none.  The whole warp: lane l holds the
// positive bits of tokens 32l .. 32l + 31.
__device__ __noinline__ int zero_tail_token(const uint64_t *keys, int n_pos, int V, int want,
                                            int lane)
{
    uint32_t pm = 0u;
    for (int i = 0; i < n_pos; i++) {
        const int t = key_tok(keys[i]);
        if ((t >> 5) == lane) pm |= 1u << (t & 31);
    }
    const int lo = 32 * lane;
    const uint32_t valid = lo >= V ? 0u : (V - lo >= 32 ? ~0u : ((1u << (V - lo)) - 1u));
    uint32_t z = ~pm & valid;
    const int c = __popc(z);
    const int incl = warp_incl_scan(c, lane);
    const bool mine = want >= incl - c && want < incl;
    const uint32_t b = __ballot_sync(kFull, mine);
    int tok = -1;
    if (mine) {
        for (int k = want - (incl - c); k > 0; k--) z &= z - 1;
        tok = lo + __ffs(z) - 1;
    }
    return b ? __shfl_sync(kFull, tok, __ffs(b) - 1) : -1;
}

// The token once the list is settled: position pos, or the last of n entries
// (a zero-probability token when the walk fell past the m positive ones).
// The whole warp, with warp-uniform arguments.
__device__ __forceinline__ int pick_token(const uint64_t *keys, int pos, int n, int m, int n_pos,
                                          int V, int pad, int lane)
{
    const int m3 = min(n, m);
    if (pos >= 0) return key_tok(keys[pos]);
    if (n > m3) return zero_tail_token(keys, n_pos, V, n - 1 - m3, lane);
    return n > 0 ? key_tok(keys[n - 1]) : pad;
}

struct RowKnobs {
    int V, K;
    bool topk_on;
    float top_p, min_p, rho, inv_rho;
    double inv_temp;
    int pad;
};

// The general path for rows the common path does not take (top-k off, more
// than 128 candidates): candidates compacted from a fresh read of the logits,
// bitonic sort, sums recomputed from the sorted keys.  Returns the token in
// every lane.
__device__ __noinline__ int general_path(const RowKnobs &kn, unsigned char *region,
                                         const float *lrow, uint32_t selm, int n_c, float M,
                                         uint32_t seenm, uint32_t allowm, int lane, float u)
{
    uint64_t *ent = reinterpret_cast<uint64_t *>(region);
    __syncwarp();
    if (kn.topk_on) {   // lane-major compaction
        const int cnt = __popc(selm);
        int off = warp_incl_scan(cnt, lane) - cnt;
        uint32_t sm = selm;
        while (sm) {
            const int i = __ffs(sm) - 1;
            sm &= sm - 1;
            const int t = slot_token(lane, i);
            ent[off++] = make_ent(prologue(__ldg(lrow + t), i, seenm, allowm, kn.rho, kn.inv_rho), t);
        }
    } else {            // every finite logit, in token order (the top-k-off sum runs in it)
        int base = 0;
        for (int j = 0; j < 8; j++) {
            const uint32_t nib = (selm >> (4 * j)) & 0xfu;
            const int cnt = __popc(nib);
            const int inc = warp_incl_scan(cnt, lane);
            int off = base + inc - cnt;
            for (int e = 0; e < 4; e++)
                if ((nib >> e) & 1u) {
                    const int t = 4 * (lane + 32 * j) + e;
                    ent[off++] = make_ent(prologue(__ldg(lrow + t), 4 * j + e, seenm, allowm,
                                                   kn.rho, kn.inv_rho), t);
                }
            base += __shfl_sync(kFull, inc, 31);
        }
    }
    __syncwarp();
    int np = 0;
    for (int q = lane; q < n_c; q += 32) {
        const uint64_t en = ent[q];
        const float p = row_prob(ent_v(en), M, kn.inv_temp, Exp2Table64());
        np += p > 0.0f;
        ent[q] = make_key(p, (int)(uint32_t)en);
    }
    const int n_pos = __reduce_add_sync(kFull, np);
    __syncwarp();
    float S = 0.0f;
    if (!kn.topk_on && lane == 0) S = seq_sum(ent, n_c);  // token-order sum: :44-49
    int N = 32;
    while (N < n_c) N <<= 1;
    for (int i = n_c + lane; i < N; i += 32) ent[i] = 0ull;
    __syncwarp();
    bitonic_smem_desc(ent, N, lane);

    const int n_list = kn.topk_on ? kn.K : kn.V;
    const int m = min(n_pos, n_list);
    if (kn.topk_on && lane == 0) S = seq_sum(ent, m);
    S = __shfl_sync(kFull, S, 0);
    int n = n_list;
    if (kn.top_p < 1.0f) {
        int cut = -1;
        if (lane == 0) {
            float cum = 0.0f;
            for (int i = 0; i < m; i++) {
                cum += key_p(ent[i]) / S;
                if (cum >= kn.top_p) {
                    cut = i + 1;
                    break;
                }
            }
            S = seq_sum(ent, min(cut > 0 ? cut : n, m));
        }
        cut = __shfl_sync(kFull, cut, 0);
        S = __shfl_sync(kFull, S, 0);
        if (cut > 0) n = cut;
    }
    if (kn.min_p > 0.0f && n > 0) {
        const float thresh = (key_p(ent[0]) / S) * kn.min_p;
        const int mm = min(n, m);
        int j = mm;
        for (int base = 0; base < mm; base += 32) {
            const int i = base + lane;
            const uint32_t fails = __ballot_sync(kFull, i < mm && !(key_p(ent[i]) / S >= thresh));
            if (fails) {
                j = base + __ffs(fails) - 1;
                break;
            }
        }
        if (j == mm && n > mm) j = (0.0f >= thresh) ? n : mm;
        n = j;
        if (lane == 0) S = seq_sum(ent, min(n, m));
        S = __shfl_sync(kFull, S, 0);
    }
    int pos = -1;
    if (lane == 0) {
        float cum = 0.0f;
        for (int i = 0; i < min(n, m); i++) {
            cum += key_p(ent[i]) / S;
            if (u <= cum) {
                pos = i;
                break;
            }
        }
    }
    pos = __shfl_sync(kFull, pos, 0);
    return pick_token(ent, pos, n, m, n_pos, kn.V, kn.pad, lane);
}

}  // namespace

// One thread per stream: the stream's n_cb uniforms in codebook order, each
// parked in its row's code slot (as f32 bits) for sample_rows_kernel, and the
// advanced generator state.
__global__ void __launch_bounds__(128) draw_uniforms_kernel(uint64_t *rng, int n_streams, int n_cb,
                                                            uint32_t *slots)
{
    grid_dep_launch();   // the sampler may start; it waits for this grid before reading a slot
    const int s = blockIdx.x * 128 + threadIdx.x;
    if (s >= n_streams) return;
    ulonglong2 *sp = reinterpret_cast<ulonglong2 *>(rng + 4 * (size_t)s);
    const ulonglong2 st01 = sp[0], st23 = sp[1];
    Xo256 g{st01.x, st01.y, st23.x, st23.y};
    uint32_t *out = slots + (size_t)s * n_cb;
    for (int c = 0; c < n_cb; c++) out[c] = __float_as_uint(g.randf());
    sp[0] = make_ulonglong2(g.s0, g.s1);
    sp[1] = make_ulonglong2(g.s2, g.s3);
}

// One stream's n_cb uniforms in codebook order from rng_in into u; the advanced
// state goes to rng_out.
__device__ __forceinline__ void draw_stream(const uint64_t *rng_in, uint64_t *rng_out, int s,
                                            int n_cb, float *u)
{
    const ulonglong2 *sp = reinterpret_cast<const ulonglong2 *>(rng_in + 4 * (size_t)s);
    const ulonglong2 st01 = sp[0], st23 = sp[1];
    Xo256 g{st01.x, st01.y, st23.x, st23.y};
    for (int c = 0; c < n_cb; c++) u[(size_t)s * n_cb + c] = g.randf();
    ulonglong2 *op = reinterpret_cast<ulonglong2 *>(rng_out + 4 * (size_t)s);
    op[0] = make_ulonglong2(g.s0, g.s1);
    op[1] = make_ulonglong2(g.s2, g.s3);
}

// Warp 0 of each sampler CTA, when the uniforms run one step ahead: for the
// CTA's slice of streams, the state after this step's draws becomes the
// stream's state, and the next step's uniforms are drawn from it.
__device__ __noinline__ void draw_ahead_slice(uint64_t *rng, uint64_t *rng_ahead, float *u_next,
                                              int n_streams, int n_cb, int lane)
{
    const int per = (n_streams + gridDim.x - 1) / gridDim.x;
    const int s_end = min(n_streams, (int)blockIdx.x * per + per);
    for (int s = (int)blockIdx.x * per + lane; s < s_end; s += 32) {
        const ulonglong2 *ap = reinterpret_cast<const ulonglong2 *>(rng_ahead + 4 * (size_t)s);
        ulonglong2 *cp = reinterpret_cast<ulonglong2 *>(rng + 4 * (size_t)s);
        const ulonglong2 st01 = ap[0], st23 = ap[1];
        cp[0] = st01;
        cp[1] = st23;
        draw_stream(rng_ahead, rng_ahead, s, n_cb, u_next);
    }
}

__global__ void __launch_bounds__(128) draw_ahead_kernel(const uint64_t *rng_in, uint64_t *rng_out,
                                                         int n_streams, int n_cb, float *u)
{
    const int s = blockIdx.x * 128 + threadIdx.x;
    if (s < n_streams) draw_stream(rng_in, rng_out, s, n_cb, u);
}

// Descending bitonic sort of 128 keys held four per lane (key e of lane l is
// element 4*l + e): compare-exchanges inside a lane for distances 1 and 2,
// shuffles across lanes for the rest.
template <class Key>
__device__ __forceinline__ void cmpx(Key &a, Key &b, bool desc)
{
    const bool sw = desc ? (a < b) : (a > b);
    const Key x = sw ? b : a;
    const Key y = sw ? a : b;
    a = x;
    b = y;
}
template <class Key, int K, int J>
__device__ __forceinline__ void bitonic_stage(Key key[4], int lane)
{
    const bool desc = ((4 * lane) & K) == 0;   // element 4l + e, K >= 4
    if constexpr (J >= 4) {
        constexpr int lj = J >> 2;
        const bool keep_max = desc == ((lane & lj) == 0);
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const Key o = __shfl_xor_sync(kFull, key[e], lj);
            key[e] = ((key[e] > o) == keep_max) ? key[e] : o;
        }
    } else if constexpr (J == 2) {
        cmpx(key[0], key[2], desc);
        cmpx(key[1], key[3], desc);
    } else if constexpr (K == 2) {
        cmpx(key[0], key[1], true);
        cmpx(key[2], key[3], false);
    } else {
        cmpx(key[0], key[1], desc);
        cmpx(key[2], key[3], desc);
    }
}
template <class Key, int K>
__device__ __forceinline__ void bitonic_merge(Key key[4], int lane)
{
    if constexpr (K >= 128) bitonic_stage<Key, K, 64>(key, lane);
    if constexpr (K >= 64) bitonic_stage<Key, K, 32>(key, lane);
    if constexpr (K >= 32) bitonic_stage<Key, K, 16>(key, lane);
    if constexpr (K >= 16) bitonic_stage<Key, K, 8>(key, lane);
    if constexpr (K >= 8) bitonic_stage<Key, K, 4>(key, lane);
    if constexpr (K >= 4) bitonic_stage<Key, K, 2>(key, lane);
    bitonic_stage<Key, K, 1>(key, lane);
}
// Bit i set for the slots of this lane that hold a token < V.
__device__ __forceinline__ uint32_t valid_slots(int lane, int V)
{
    uint32_t m = 0u;
#pragma unroll
    for (int i = 0; i < 32; i++) m |= (slot_token(lane, i) < V ? 1u : 0u) << i;
    return m;
}

// The row's slots -> registers when V < 1024 (slots past V read 0).
__device__ __forceinline__ void load_row_partial(const float *rowf, int lane, int V, float v[32])
{
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int t0 = 4 * (lane + 32 * j);
        float4 f = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (t0 < V) f = *reinterpret_cast<const float4 *>(rowf + t0);
        v[4 * j + 0] = f.x;
        v[4 * j + 1] = f.y;
        v[4 * j + 2] = f.z;
        v[4 * j + 3] = f.w;
    }
}

// The prologue logit by logit, with the non-finite guard: for rows holding a
// NaN or infinite logit, and for a penalty < 1.  Reloads the raw row, returns
// this lane's max; drops non-finite slots from *km, flags them in *nonfin.
__device__ __forceinline__ float careful_prologue(const float *rowf, int lane, int V, uint32_t seenm,
                                               uint32_t allowm, uint32_t validm, float rho,
                                               float inv_rho, float v[32], uint32_t *km,
                                               bool *nonfin)
{
    float mx = -INFINITY;
    uint32_t finm = 0u;
    bool nf = false;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int t0 = 4 * (lane + 32 * j);
        float4 f = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (t0 < V) f = *reinterpret_cast<const float4 *>(rowf + t0);
        v[4 * j + 0] = f.x;
        v[4 * j + 1] = f.y;
        v[4 * j + 2] = f.z;
        v[4 * j + 3] = f.w;
    }
#pragma unroll
    for (int i = 0; i < 32; i++) {
        const bool fin = v[i] < INFINITY;
        nf |= !fin;
        finm |= (fin ? 1u : 0u) << i;
        v[i] = prologue(v[i], i, seenm, allowm & validm, rho, inv_rho);
        mx = fmaxf(mx, v[i]);
    }
    *km &= finm;
    *nonfin = nf;
    return mx;
}

// One odd-even transposition round (descending) on 128 keys held four per lane
// (element 4*l + e): pairs (0,1) (2,3), then (1,2) (3, next lane's 0).  With
// kCheck, returns whether it swapped anything in this lane.
template <bool kCheck>
__device__ __forceinline__ bool oets_round(uint32_t k[4], int lane)
{
    bool moved = false;
    if (kCheck) moved = k[0] < k[1] || k[2] < k[3];
    const uint32_t a0 = max(k[0], k[1]), a1 = min(k[0], k[1]);
    const uint32_t a2 = max(k[2], k[3]), a3 = min(k[2], k[3]);
    if (kCheck) moved = moved || a1 < a2;
    k[1] = max(a1, a2);
    k[2] = min(a1, a2);
    const uint32_t nx = __shfl_down_sync(kFull, a0, 1);   // the next lane's first
    const uint32_t pv = __shfl_up_sync(kFull, a3, 1);     // the previous lane's last
    if (kCheck) moved = moved || (lane < 31 && a3 < nx);
    k[3] = lane < 31 ? max(a3, nx) : a3;
    k[0] = lane > 0 ? min(a0, pv) : a0;
    return moved;
}

// Odd-even transposition rounds until one swaps nothing; true if sorted within
// `cap` rounds.  Bucket order leaves only keys inside a bucket out of order, a
// few rounds from sorted, and the check (a vote and the branch on it) costs more
// than a round: rounds 0-2 run unchecked, then every second round is checked
// (the constrained 4096-stream step: 4.8 rounds per row, 0.0682 against
// 0.0698 ms checking every round; the head's flatter logits take 8.2).
__device__ __forceinline__ bool oets_desc(uint32_t k[4], int lane, int cap)
{
    for (int round = 0; round < cap; round++) {
        if (round < 3 || !(round & 1)) {
            oets_round<false>(k, lane);
        } else if (!__any_sync(kFull, oets_round<true>(k, lane))) {
            return true;
        }
    }
    return false;
}

// Odd-even transposition rounds on 128 64-bit keys (descending), as oets_desc.
__device__ __forceinline__ bool oets_desc64(uint64_t k[4], int lane, int cap)
{
    for (int round = 0; round < cap; round++) {
        bool moved = (k[0] < k[1]) || (k[2] < k[3]);
        const uint64_t a0 = max(k[0], k[1]), a1 = min(k[0], k[1]);
        const uint64_t a2 = max(k[2], k[3]), a3 = min(k[2], k[3]);
        moved = moved || (a1 < a2);
        k[1] = max(a1, a2);
        k[2] = min(a1, a2);
        const uint64_t nx = __shfl_down_sync(kFull, a0, 1);
        const uint64_t pv = __shfl_up_sync(kFull, a3, 1);
        moved = moved || (lane < 31 && a3 < nx);
        k[3] = lane < 31 ? max(a3, nx) : a3;
        k[0] = lane > 0 ? min(a0, pv) : a0;
        if (!__any_sync(kFull, moved)) return true;
    }
    return false;
}

// Out of line: the exact-key sort for the rare rows whose quantized order fails.
__device__ __noinline__ void sort_keys_exact(uint64_t key[4], int lane);

template <class Key>
__device__ __forceinline__ void bitonic128_desc(Key key[4], int lane)
{
    bitonic_merge<Key, 2>(key, lane);
    bitonic_merge<Key, 4>(key, lane);
    bitonic_merge<Key, 8>(key, lane);
    bitonic_merge<Key, 16>(key, lane);
    bitonic_merge<Key, 32>(key, lane);
    bitonic_merge<Key, 64>(key, lane);
    bitonic_merge<Key, 128>(key, lane);
}

// Inclusive prefix sums, in f64, of the sorted probabilities at positions < m
// (position 4*lane + e).  At most 128 f32 terms: each f64 add is exact or off by
// 2^-53 relative, far inside the margins they are used with.
__device__ __forceinline__ void prefix_f64(const uint64_t key[4], int m, int lane, double P[4])
{
    double run = 0.0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        run = __dadd_rn(run, (4 * lane + e < m) ? (double)key_p(key[e]) : 0.0);
        P[e] = run;
    }
    double incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl = __dadd_rn(incl, y);
    }
    double excl = __shfl_up_sync(kFull, incl, 1);
    if (lane == 0) excl = 0.0;
#pragma unroll
    for (int e = 0; e < 4; e++) P[e] = __dadd_rn(P[e], excl);
}

__device__ __forceinline__ double sel4(const double P[4], int e)
{
    return e == 0 ? P[0] : e == 1 ? P[1] : e == 2 ? P[2] : P[3];
}

// P at position i, in every lane.
__device__ __forceinline__ double prefix_at(const double P[4], int i)
{
    return __shfl_sync(kFull, sel4(P, i & 3), i >> 2);
}

// Smallest position 4*l + e whose bit e is set in lane l's f4; 128 if none.
__device__ __forceinline__ int first_flagged(uint32_t f4)
{
    const uint32_t b = __ballot_sync(kFull, f4 != 0u);
    if (b == 0u) return 128;
    const int fl = __ffs(b) - 1;
    return 4 * fl + __ffs(__shfl_sync(kFull, f4, fl)) - 1;
}

// max(a, b, c) in one instruction (sm_100); a NaN operand is ignored as by fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c)
{
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ uint32_t sel4u(const uint32_t x[4], int e)
{
    return e == 0 ? x[0] : e == 1 ? x[1] : e == 2 ? x[2] : x[3];
}
__device__ __forceinline__ float sel4f(const float x[4], int e)
{
    return e == 0 ? x[0] : e == 1 ? x[1] : e == 2 ? x[2] : x[3];
}

// 2^a by the hardware approximation (relative error far below 2^-20 for
// results in the normal range).
__device__ __forceinline__ float ex2_approx(float a)
{
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
    return r;
}

// A partial sum the reference accumulates term by term in f32 over a sorted list
// of len probabilities p_j, each divided by the list's own f32 sum S', is at
// position i < len P_i / S * (1 + d), with P_i, S the exact sums and
// |d| <= (len - 1 + 1 + i) * 2^-24 * (1 + O(2^-24)): len - 1 roundings in S', one
// per division, i in the running sum.  sum_eta(len) bounds it for every i < len
// (the factor covers the second-order terms); decisions clear of the threshold
// by this margin equal the reference's, the rest are made term by term.
__device__ __forceinline__ float sum_eta(int len)
{
    return (float)(2 * len) * (1.01f * 0x1p-24f);
}

// min-p keeps position i while fl(p_i / S) >= fl(fl(p_0 / S) * min_p); the sum S
// cancels, so p_i >= p_0 * min_p * (1 + 2^-24) keeps it and
// p_i < p_0 * min_p * (1 - 3 * 2^-24) drops it; the margin is taken 5x.
constexpr double kMinpEta = 16.0 * 0x1p-24;

// The probability at sorted position i, in every lane.
__device__ __forceinline__ float key_p_at(const uint64_t key[4], int i)
{
    const int e = i & 3;
    const uint64_t k = e == 0 ? key[0] : e == 1 ? key[1] : e == 2 ? key[2] : key[3];
    return __shfl_sync(kFull, key_p(k), i >> 2);
}

__device__ __noinline__ void sort_keys_exact(uint64_t key[4], int lane)
{
    bitonic128_desc(key, lane);
}

// Steps 6-8 in exact arithmetic, for the rows the certified form cannot settle.
// Lane l holds candidates 4l + e (token t_e, penalized logit l_e) in the
// quantized order.  Exact probabilities make exact keys; where the quantized order
// breaks theirs, odd-even rounds restore it (only neighbours within a quantum
// are out of order), with a full sort after 8 rounds; decisions come from exact
// f64 prefix sums
// where the reference's margin allows, else term by term with the reference's
// f32 sums.  The row's logits are no longer in shared memory: the next row's
// copy may be landing there.  Returns the token in every lane.
__device__ __noinline__ int exact_decide(unsigned char *region, const double *exptab, int n_c, int K,
                                         int V, int pad, float top_p, float min_p, double inv_temp,
                                         float M, float u, int lane, float l0, float l1, float l2,
                                         float l3, uint32_t t0, uint32_t t1, uint32_t t2,
                                         uint32_t t3)
{
    const float lv[4] = {l0, l1, l2, l3};
    const uint32_t tk[4] = {t0, t1, t2, t3};
    const SmemExpTable tab{exptab};
    uint64_t key[4];
    int np = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        key[e] = 0ull;   // sorts after every candidate
        if (4 * lane + e < n_c) {
            const float p = row_prob(lv[e], M, inv_temp, tab);
            np += p > 0.0f;
            key[e] = make_key(p, (int)tk[e]);
        }
    }
    const int n_pos = __reduce_add_sync(kFull, np);
    {
        const uint64_t nx = __shfl_down_sync(kFull, key[0], 1);
        const int i0 = 4 * lane;   // pairs (i, i + 1) with i + 1 < n_c
        const bool ok = (i0 + 1 >= n_c || key[0] > key[1]) && (i0 + 2 >= n_c || key[1] > key[2]) &&
                        (i0 + 3 >= n_c || key[2] > key[3]) && (i0 + 4 >= n_c || key[3] > nx);
        if (!__all_sync(kFull, ok) && !oets_desc64(key, lane, 8)) sort_keys_exact(key, lane);
    }
    uint64_t *keys = reinterpret_cast<uint64_t *>(region + kKeysOffset);
    float *ps = reinterpret_cast<float *>(region + kPsOffset);
    reinterpret_cast<ulonglong2 *>(keys)[2 * lane] = make_ulonglong2(key[0], key[1]);
    reinterpret_cast<ulonglong2 *>(keys)[2 * lane + 1] = make_ulonglong2(key[2], key[3]);
    reinterpret_cast<float4 *>(ps)[lane] =
        make_float4(key_p(key[0]), key_p(key[1]), key_p(key[2]), key_p(key[3]));
    __syncwarp();

    // The list is keys[0..m) (positive probabilities, sorted) followed by
    // zero-probability tokens in token order, n entries in all.
    const int m = min(n_pos, K);
    int n = K;
    int hit = -1;   // 1 + the walk's position; -1 when it runs past the positives
    bool fast = true;
    double P[4];
    prefix_f64(key, m, lane, P);
    if (top_p < 1.0f) {
        const double tpS = (double)top_p * prefix_at(P, m - 1);
        const double eta = (double)sum_eta(m) + 0x1p-40;
        uint32_t nb = 0u;   // positions not certainly below top_p
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (4 * lane + e < m && !(P[e] * (1.0 + eta) < tpS)) nb |= 1u << e;
        const int jj = first_flagged(nb);
        if (jj < 128) {   // 128: the sum never reaches top_p, no cut
            if (prefix_at(P, jj) * (1.0 - eta) >= tpS) n = jj + 1;
            else fast = false;
        }
    }
    if (fast && min_p > 0.0f) {
        if (!(min_p >= 0x1p-100f)) {   // thresholds near the f32 range's end
            fast = false;
        } else {   // keep while p_i >= p_0 * min_p
            const int mm = min(n, m);
            const double thr = (double)__shfl_sync(kFull, key_p(key[0]), 0) * (double)min_p;
            uint32_t nk = 0u;   // positions not certainly kept
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (4 * lane + e < mm && !((double)key_p(key[e]) >= thr * (1.0 + kMinpEta)))
                    nk |= 1u << e;
            const int jj = first_flagged(nk);
            if (jj == 128)
                n = mm;   // every positive kept; the zero tail is not (thresh > 0)
            else if ((double)key_p_at(key, jj) < thr * (1.0 - kMinpEta))
                n = jj;
            else
                fast = false;
        }
    }
    // one uniform, CDF walk (src/zonos2_generate.cpp:86-92): the first position
    // whose partial sum reaches u
    if (fast) {
        const int len = min(n, m);
        const double uS = (double)u * prefix_at(P, max(len, 1) - 1);
        const double eta = (double)sum_eta(len) + 0x1p-40;
        uint32_t nb = 0u;   // positions not certainly below u
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (4 * lane + e < len && !(uS > P[e] * (1.0 + eta))) nb |= 1u << e;
        const int jj = first_flagged(nb);
        if (jj < 128) {
            if (uS <= prefix_at(P, jj) * (1.0 - eta)) hit = jj + 1;
            else fast = false;
        }
    }
    if (!fast) {   // term by term, as the reference
        float *pf = reinterpret_cast<float *>(region + kPfOffset);
        float *q = reinterpret_cast<float *>(region + kQOffset);
        n = K;
        if (lane == 0) prefix_sums(ps, pf, m);
        __syncwarp();
        float S = pf[m - 1];
        if (top_p < 1.0f) {
            const int c = walk_cdf(ps, q, m, S, top_p, lane);
            if (c > 0) n = c;  // never inside the zero tail: the sum stops growing
            S = pf[min(n, m) - 1];
        }
        if (min_p > 0.0f) {
            const float thresh = (ps[0] / S) * min_p;
            const int mm = min(n, m);
            int jn = minp_cut(ps, mm, S, thresh, lane);
            if (jn == mm && n > mm) jn = (0.0f >= thresh) ? n : mm;
            n = jn;
            S = pf[min(n, m) - 1];
        }
        hit = walk_cdf(ps, q, min(n, m), S, u, lane);
    }
    return pick_token(keys, hit > 0 ? hit - 1 : -1, n, m, n_pos, V, pad, lane);
}

// Persistent: CTA b owns work items b + k * gridDim.x, k = 0, 1, ...; warp w starts
// on k = w and then takes the CTA's next free k from a shared counter, so a warp
// held up by a slow row (the exact form, a general-path row) leaves the rest of
// its CTA's rows to its siblings.  Items run codebook-major (item cb * n_streams + s
// is row s * n_cb + cb), so every CTA sees every codebook and a row's cost
// (delay-forced codebooks are cheap) does not stick to one CTA.  While a row is
// sorted and decided, the bulk copy of the warp's next row lands.
template <bool kCtx>
__global__ void __launch_bounds__(32 * kWarps, kCtasPerSm) sample_rows_kernel(const SampleArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    double *exptab = reinterpret_cast<double *>(smem);
    const int lane = threadIdx.x & 31;
    const int w = threadIdx.x >> 5;
    unsigned char *region = smem + kCtaHeader + w * kWarpStride;
    float *rowf = reinterpret_cast<float *>(region + kRowOffset);
    uint32_t *hist = reinterpret_cast<uint32_t *>(region + kHistOffset);
    uint32_t *bkt = reinterpret_cast<uint32_t *>(region + kBktOffset);
    const uint32_t bar = smem_u32(region + kBarOffset);
    unsigned *next_k = reinterpret_cast<unsigned *>(smem + kCtrOffset);
    if (threadIdx.x < 64) exptab[threadIdx.x] = exp2_64th(threadIdx.x);
    if (threadIdx.x == 0) *next_k = (unsigned)kWarps;
    if (lane == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const int V = a.vocab;
    const int NCB = a.n_cb;
    const int S_ = a.n_streams;
    const int K = a.top_k;
    const bool topk_on = K > 0 && K < V;
    const bool pen = a.hist_len > 0 && a.rho != 1.0f;
    // kCtx: compiled for the decode context's launches (rows 16-byte aligned,
    // uniforms drawn ahead, the history index, an allow mask, if any, lane-major),
    // where these tests are constants: the branches on them and the paths they
    // rule out (the ring scan, the shuffled allow unpacking, the scalar row load,
    // the draw kernel's parked uniforms) leave the row loop (0.0668 -> 0.0646 ms
    // on the constrained 4096-stream step)
    const bool inc = kCtx || a.presence != nullptr;
    const bool vec = kCtx || a.vec_logits;
    const bool ahead = kCtx || a.u_cur != nullptr;
    const bool lm_allow = kCtx || a.allow_lane_major;
    const bool hst = kCtx || (a.hist && a.hist_len > 0);
    const uint32_t row_bytes = 4u * (uint32_t)V;
    const uint32_t *slots = reinterpret_cast<const uint32_t *>(a.codes);

    // work item it -> (s, cb), codebook-major: the quotient by an f64 reciprocal,
    // corrected by one either way
    const long long n_items = (long long)S_ * NCB;
    const double inv_S = 1.0 / (double)S_;
    auto item_at = [&](long long it, int &s2, int &cb2) {
        if (it >= n_items) {
            s2 = 0;
            cb2 = NCB;   // no item
            return;
        }
        long long q = (long long)((double)it * inv_S);
        long long rem = it - q * S_;
        if (rem < 0) {
            q--;
            rem += S_;
        } else if (rem >= S_) {
            q++;
            rem -= S_;
        }
        cb2 = (int)q;
        s2 = (int)rem;
    };
    int s, cb;
    item_at(blockIdx.x + (long long)gridDim.x * w, s, cb);

    uint32_t phase = 0u;
    // The warp's first row towards L2 while the kernel before this one finishes: a
    // prefetch reads nothing into the CTA, and L2 holds every write that kernel
    // makes, so it is safe whatever that kernel writes.
    if (vec && lane == 0 && cb < NCB)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                         a.logits + ((long long)s * NCB + cb) * a.row_stride),
                     "r"(row_bytes)
                     : "memory");
    // With uniforms drawn ahead the kernel before this one may be the previous
    // step's sampler (history index, generators) or the head (logits): wait for it
    // before any global read.  Either way the next launch may be scheduled now.
    grid_dep_launch();
    if (ahead) grid_dep_wait();
    bool drawn = ahead;   // the grid before this one has been waited for
    bool pending = false;   // the copy of the current row is in flight
    uint32_t seen_next = 0u, allow_next = ~0u;   // lane-major masks of the next row
    int ev_next = -1;   // lane 0: the token the next row's append evicts

    // Starts the bulk copy of row (s2, cb2) and loads its lane-major masks.
    auto issue = [&](int s2, int cb2) {
        const long long r2 = (long long)s2 * NCB + cb2;
        if (vec && lane == 0) {
            fence_proxy_async();
            mbar_expect_tx(bar, row_bytes);
            bulk_g2s(smem_u32(rowf), a.logits + r2 * a.row_stride, row_bytes, bar);
        }
        if (pen && inc) seen_next = __ldcg(a.presence + (size_t)r2 * 32 + lane);
        if (a.allow && lm_allow) allow_next = __ldg(a.allow + (size_t)s2 * 32 + lane);
        if (inc && lane == 0) ev_next = __ldcg(a.hist + (size_t)r2 * a.hist_len + a.hist_pos);
        pending = true;
    };
    if (cb < NCB) issue(s, cb);
    if (ahead && w == 0) draw_ahead_slice(a.rng, a.rng_ahead, a.u_next, S_, NCB, lane);

    while (cb < NCB) {
        const long long r = (long long)s * NCB + cb;
        const float *lrow = a.logits + r * a.row_stride;
        int s_nx, cb_nx;
        {
            unsigned k = 0u;
            if (lane == 0) k = atomicAdd(next_k, 1u);
            k = __shfl_sync(kFull, k, 0);
            item_at(blockIdx.x + (long long)gridDim.x * k, s_nx, cb_nx);
        }
        if (!pending) issue(s, cb);

        // ---- 1. the history's token set and the allow bits
        uint32_t seenm = seen_next, allowm = ~0u;
        const int ev = ev_next;
        if (pen && !inc) {   // scan the ring into seen-bytes
            unsigned char *seen = region + kBktOffset;
            uint4 *seen4 = reinterpret_cast<uint4 *>(seen);
            seen4[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
            seen4[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
            __syncwarp();
            const int32_t *hrow = a.hist + (size_t)r * a.hist_len;
            const int H = a.hist_len;
            if (a.vec_hist) {
                for (int q0 = 0; q0 < H; q0 += 512) {
                    int4 t[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int q = q0 + 4 * lane + 128 * u;
                        t[u] = q < H ? __ldcg(reinterpret_cast<const int4 *>(hrow + q))
                                     : make_int4(-1, -1, -1, -1);
                    }
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        mark_seen(seen, t[u].x, V);
                        mark_seen(seen, t[u].y, V);
                        mark_seen(seen, t[u].z, V);
                        mark_seen(seen, t[u].w, V);
                    }
                }
            } else {
                for (int q = lane; q < H; q += 32) mark_seen(seen, __ldcg(hrow + q), V);
            }
            __syncwarp();
            seenm = 0u;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t wd = *reinterpret_cast<const uint32_t *>(seen + 4 * (lane + 32 * j));
                seenm |= ((wd * 0x10204080u) >> 28) << (4 * j);   // four 0/1 bytes -> 4 bits
            }
        }
        if (a.allow) {
            if (lm_allow) {
                allowm = allow_next;
            } else {
                const uint32_t aw = lane < a.allow_words
                                        ? __ldg(a.allow + (size_t)s * a.allow_words + lane)
                                        : ~0u;
                allowm = 0u;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const uint32_t wv = __shfl_sync(kFull, aw, (lane + 32 * j) >> 3);
                    allowm |= ((wv >> (4 * (lane & 7))) & 0xfu) << (4 * j);
                }
            }
        }
        const bool forced = a.delay_step >= 0 && a.delay_step < cb;
        if (forced) {   // delay pattern: only the pad token
            const int p = a.pad_id;
            allowm &= lane == ((p >> 2) & 31) ? lm_bit(p) : 0u;
        }

        // ---- 2. wait for the row; slots -> registers
        if (vec) {
            if (!mbar_wait_warp(bar, phase, lane)) return;   // the error word is set
            phase ^= 1u;
        } else {
            for (int t = lane; t < ((V + 3) & ~3); t += 32)
                rowf[t] = t < V ? __ldg(lrow + t) : -INFINITY;
            __syncwarp();
        }
        pending = false;
        // slots at or past the vocabulary never enter a row
        const uint32_t validm = V >= 1024 ? ~0u : valid_slots(lane, V);
        float v[32];
        if (V >= 1024) {
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float4 f = *reinterpret_cast<const float4 *>(rowf + 4 * (lane + 32 * j));
                v[4 * j + 0] = f.x;
                v[4 * j + 1] = f.y;
                v[4 * j + 2] = f.z;
                v[4 * j + 3] = f.w;
            }
        } else {
            load_row_partial(rowf, lane, V, v);
        }

        // ---- 3. prologue and row max; the row is rewritten in place.  Fast form
        // for a penalty >= 1 and finite logits: the penalized logit is
        // min(l * RN(1/rho), l * rho), which is the reference's pick of the two,
        // and one fma per logit (l * 0 + acc) leaves acc nonzero if any logit is
        // NaN or infinite; such rows (and a penalty < 1) take the careful form.
        float mx = -INFINITY;
        uint32_t km = allowm & validm;   // slots that keep their logit
        bool nonfin = false;
        float w;   // the row max, or NaN: the careful form
        {
            float acc = __int_as_float(0x7fc00000);   // NaN: a penalty below 1 takes the careful form
            if (a.rho >= 1.0f) {   // slots in pairs: the products and the fma packed (f32x2)
                float2 acc2 = make_float2(0.0f, 0.0f);
                const float2 ir2 = make_float2(a.inv_rho, a.inv_rho);
                const float2 r2 = make_float2(a.rho, a.rho);
                const float2 zero2 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float2 x = make_float2(v[i], v[i + 1]);
                    acc2 = __ffma2_rn(x, zero2, acc2);
                    const float2 pa = __fmul2_rn(x, ir2), pb = __fmul2_rn(x, r2);
                    const float z0 = ((seenm >> i) & 1u) ? fminf(pa.x, pb.x) : x.x;
                    const float z1 = ((seenm >> (i + 1)) & 1u) ? fminf(pa.y, pb.y) : x.y;
                    v[i] = ((km >> i) & 1u) ? z0 : -INFINITY;
                    v[i + 1] = ((km >> (i + 1)) & 1u) ? z1 : -INFINITY;
                    mx = fmax3(mx, v[i], v[i + 1]);
                }
                acc = __fadd_rn(acc2.x, acc2.y);
            }
            // acc is 0, or NaN if a slot of this lane is non-finite, so mx + acc is the
            // lane's max or NaN, and the warp's NaN-propagating max (one instruction,
            // sm_100a; a max, so exact) is the row max or NaN.  The test needs no vote
            // of its own (0.0678 against 0.0682 ms); -0 + 0 = +0 changes no logit
            // difference, so no token.
            asm("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;" : "=f"(w) : "f"(__fadd_rn(mx, acc)));
        }
        int nf_flag = 0;
        if (isnan(w)) {   // the careful form, and the non-finite flag only it can raise
            mx = careful_prologue(rowf, lane, V, seenm, allowm, validm, a.rho, a.inv_rho, v, &km,
                                  &nonfin);
            asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(mx) : "f"(mx));
            nf_flag = __any_sync(kFull, nonfin) ? 2 : 0;
        } else {
            mx = w;
        }
        const bool live = mx >= -1e9f;  // running max starts at -1e9: :41-42
        const int flag = nf_flag | (live ? 0 : 1);
        // The evicted token leaves the history index now that the row's set has been
        // read: its count drops (two u16 counts per word); the old count comes back
        // by the end of the row.
        uint32_t ev_old = 0u;
        if (inc && lane == 0 && (unsigned)ev < (unsigned)V)
            ev_old = atomicSub(reinterpret_cast<uint32_t *>(a.counts + (size_t)r * kSamplerVocabMax) +
                                   (ev >> 1),
                               1u << (16 * (ev & 1)));

        int tok = a.pad_id;
        if (live && !forced) {
#pragma unroll
            for (int j = 0; j < 8; j++)
                *reinterpret_cast<float4 *>(rowf + 4 * (lane + 32 * j)) =
                    make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            const float M = mx;
            const float T = a.temperature;
            // ---- 4. gap histogram and the bucket of the k-th largest logit.  The
            // open-ended last bucket holds most of a row: it is not counted, its
            // count follows from the number of kept logits.
            const float bw = fmaxf(T * 0.125f, fabsf(M) * 0x1p-18f + T * 0x1p-14f);
            float sc;   // any positive scale will do: every bucket below is computed from it
            asm("rcp.approx.f32 %0, %1;" : "=f"(sc) : "f"(bw));
            const float Msc = M * sc;
            const float s126 = sc * (1.0f / (float)(kBuckets - 2));
            const float Ms126 = M * s126;
            reinterpret_cast<uint4 *>(hist)[lane] = make_uint4(0u, 0u, 0u, 0u);
            __syncwarp();
            // bucket_bits = 0x4B000000 + b, so (bits * 4 + hbase) mod 2^32 is the
            // shared address of counter b
            const uint32_t hbase = smem_u32(hist) - 0x2C000000u;
            // Slots in the open-ended bucket 126 add to a counter of their own lane,
            // 126 + lane (126 and 127 here, the rest in the stage, unused until the
            // scatter), so the red needs no branch and lanes do not collide.  The
            // address is the signed max of hist + 4b and
            // hist + 4 (126 + lane) - 640 (126 - b): the first for b <= 125, the
            // second for b = 126.  Two multiply-adds (fma pipe) and a max, where a
            // compare and a select would both take the ALU pipe, the kernel's
            // busiest (0.0698 against 0.0706 ms).
            const uint32_t k_sp =
                smem_u32(hist) + 504u + 4u * (uint32_t)lane - 80640u - 640u * 0x4B000000u;
            const float2 ns2 = make_float2(-s126, -s126), ms2 = make_float2(Ms126, Ms126);
            const float2 k2 = make_float2((float)(kBuckets - 2), (float)(kBuckets - 2));
            const float2 mag2 = make_float2(0x1p23f, 0x1p23f);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                uint32_t bb[4];
#pragma unroll
                for (int e = 0; e < 4; e += 2) {   // bucket_bits of two slots at once
                    const float2 u =
                        ffma2_sat(make_float2(v[4 * j + e], v[4 * j + e + 1]), ns2, ms2);
                    const float2 t = __ffma2_rn(u, k2, mag2);
                    bb[e] = __float_as_uint(t.x);
                    bb[e + 1] = __float_as_uint(t.y);
                }
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const uint32_t ad =
                        (uint32_t)max((int)(bb[e] * 4u + hbase), (int)(bb[e] * 640u + k_sp));
                    asm volatile("red.shared.add.u32 [%0], 1;" ::"r"(ad) : "memory");
                }
                bkt[lane + 32 * j] = __byte_perm(__byte_perm(bb[0], bb[1], 0x0040u),
                                                 __byte_perm(bb[2], bb[3], 0x0040u), 0x5410u);
            }
            const int n_fin = __reduce_add_sync(kFull, __popc(km));
            __syncwarp();
            const uint4 h4 = reinterpret_cast<const uint4 *>(hist)[lane];
            int h[4] = {(int)h4.x, (int)h4.y, (int)h4.z, (int)h4.w};
            int tot = h[0] + h[1] + h[2] + h[3];
            int incl = warp_incl_scan(tot, lane);
            if (lane == 31) {   // bucket 126 = 4*31 + 2; counters 126, 127 held spare counts
                tot -= h[2] + h[3];
                incl -= h[2] + h[3];
                h[2] = 0;
                h[3] = 0;
                const int rest = n_fin - incl;
                h[2] += rest;
                tot += rest;
                incl += rest;
            }
            int bc = kBuckets - 2;   // every finite logit
            if (topk_on && n_fin > K) {
                const int fl = __ffs(__ballot_sync(kFull, incl >= K)) - 1;
                // in lane fl: the first of its four buckets whose running count reaches K
                const int c1 = incl - tot + h[0], c2 = c1 + h[1], c3 = c2 + h[2];
                const int bstar = 4 * lane + (c1 < K) + (c2 < K) + (c3 < K);
                bc = min(__shfl_sync(kFull, bstar, fl) + 1, kBuckets - 2);
            }
            int n_c;   // candidates: finite logits in buckets 0..bc
            {
                int c = incl - tot, upto = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (4 * lane + i == bc) upto = c + h[i];
                    c += h[i];
                }
                n_c = __shfl_sync(kFull, upto, bc >> 2);
            }
            const uint32_t bc4 = 0x80808080u | ((uint32_t)bc * 0x01010101u);
            uint32_t selm = 0u;   // this lane's candidate slots
#pragma unroll
            for (int j = 0; j < 8; j++) selm |= bytes_le(bkt[lane + 32 * j], bc4) << (4 * j);
            selm &= km;
            {   // counters -> each bucket's first position in bucket order
                const int c0 = incl - tot;
                reinterpret_cast<uint4 *>(hist)[lane] =
                    make_uint4(c0, c0 + h[0], c0 + h[0] + h[1], c0 + h[0] + h[1] + h[2]);
            }

            // the uniform: its producer has finished once waited for
            if (!drawn) {
                grid_dep_wait();
                drawn = true;
            }
            const float u = ahead ? __ldg(a.u_cur + r) : __uint_as_float(__ldcg(slots + r));

            if (!topk_on || n_c > kRegSortMax) {
                RowKnobs kn;
                kn.V = V;
                kn.K = K;
                kn.topk_on = topk_on;
                kn.top_p = a.top_p;
                kn.min_p = a.min_p;
                kn.rho = a.rho;
                kn.inv_rho = a.inv_rho;
                kn.inv_temp = a.inv_temp;
                kn.pad = a.pad_id;
                tok = general_path(kn, region, lrow, selm, n_c, M, seenm, allowm, lane, u);
                __syncwarp();
                if (cb_nx < NCB) issue(s_nx, cb_nx);
            } else {
                // ---- 5. candidates -> four per lane, as 32-bit sort keys, scattered in
                // bucket order (the histogram's prefix gives each bucket's first slot).
                // p is a non-increasing function of the gap, so the keys order the
                // candidates by the gap's bucket coordinate (max - l) / width, monotone
                // in l like the bucket and kept to 15 fractional bits, then by token.
                // That is the exact (p desc, token asc) order unless two gaps share a
                // quantum or two gaps give one p; the order of the exact keys is
                // checked below and, if broken, sorted outright.
                uint32_t *stage = reinterpret_cast<uint32_t *>(region + kStageOffset);
                __syncwarp();   // bucket offsets in place
                {   // as many rounds as the fullest lane needs: a lane with nothing left
                    // writes a spare entry past the stage
                    const int cnt = __popc(selm);
                    const int rounds = __reduce_max_sync(kFull, (unsigned)cnt);
                    uint32_t sm = selm;
                    for (int k = 0; k < rounds; k++) {
                        const bool has = sm != 0u;
                        const int i = __ffs(sm | 0x80000000u) - 1;
                        sm &= sm - 1u;
                        const int t = slot_token(lane, i);
                        // the gap coordinate on the raw float bits: the bucket bits
                        // 0x4B000000 + b (as the histogram's) address the counter as
                        // bits * 4 + hbase, and q = qbits - 0x4B000000 enters the key
                        // ~(q << 10 | t) = q * -1024 + ~t (t < 1024) as qbits, since
                        // 0x4B000000 * 1024 = 0 mod 2^32: one multiply-add each
                        float gu;
                        asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(gu) : "f"(-rowf[t]), "f"(s126), "f"(Ms126));
                        const uint32_t bbits = __float_as_uint(__fmaf_rn(gu, 126.0f, 0x1p23f));
                        const uint32_t qbits =
                            __float_as_uint(__fmaf_rn(gu, 126.0f * 32768.0f, 16384.0f + 0x1p23f));
                        int pos = kRegSortMax;
                        if (has) {
                            uint32_t old;
                            asm volatile("atom.shared.add.u32 %0, [%1], 1;"
                                         : "=r"(old)
                                         : "r"(bbits * 4u + hbase)
                                         : "memory");
                            pos = (int)old;
                        }
                        stage[pos] = qbits * (uint32_t)-1024 + ~(uint32_t)t;
                    }
                }
                __syncwarp();
                uint32_t ck[4];
                {
                    const uint4 k4 = reinterpret_cast<const uint4 *>(stage)[lane];
                    ck[0] = 4 * lane + 0 < n_c ? k4.x : 0u;
                    ck[1] = 4 * lane + 1 < n_c ? k4.y : 0u;
                    ck[2] = 4 * lane + 2 < n_c ? k4.z : 0u;
                    ck[3] = 4 * lane + 3 < n_c ? k4.w : 0u;
                }
                // Bucket order leaves the keys unsorted only inside buckets of a few
                // candidates: odd-even transposition rounds finish them; a bitonic
                // network takes over if 16 rounds do not.
                if (!oets_desc(ck, lane, 16)) bitonic128_desc(ck, lane);
                // ---- 6. probabilities to certify decisions with: p~ = 2^(fl(l - M) * c2),
                // c2 = RN(log2(e) / T), by the hardware exp2.  Against the reference's
                // p = RN(exp(fl(l - M) / T)): the argument differs by at most three f32
                // roundings, a relative 3.02 * 2^-24 of |x| = |l - M| / T (so p~ / p by
                // |x| * 3.02 * 2^-24 relative), the exp2 by less than 2^-21 (its largest
                // error over every f32 argument in [-126, 0], measured on this part, is
                // 2^-22.7) and the reference's rounding by 2^-24.  Every candidate lies in
                // a bucket <= bc, so |x| * log2(e) <= argmax below.
                const float c2 = (float)(a.inv_temp * 1.4426950408889634);
                const float argmax =
                    ((float)bc + 0.52f + fabsf(Msc) * 0x1p-22f) * bw * c2 * 1.0001f;
                const float eps_p = argmax * (2.2f * 0x1p-24f) + (0x1p-21f + 0x1p-23f);
                float lv[4], pv[4];
                uint32_t tk[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    tk[e] = ~ck[e] & 1023u;
                    lv[e] = rowf[tk[e]];
                    // positions past n_c hold key 0 (token 1023: a logit <= M or -inf, so
                    // pv in [0, 1]); every use of pv is limited to n_c, m or mm positions
                    pv[e] = ex2_approx(__fmul_rn(__fsub_rn(lv[e], M), c2));
                }
                __syncwarp();   // the row and the stage are free
                if (cb_nx < NCB) issue(s_nx, cb_nx);

                // The quantized order is the exact (p desc, token asc) order if every
                // adjacent pair (a, b) has l_a > l_b with t_a < t_b or p_a > p_b for
                // certain (p is non-decreasing in l), or l_a == l_b (then t_a < t_b: a
                // shared quantum sorts by token).
                const float sep = 1.0f + 2.2f * eps_p + 0x1p-22f;
                bool ok;
                {
                    const float ln = __shfl_down_sync(kFull, lv[0], 1);
                    const float pn = __shfl_down_sync(kFull, pv[0], 1);
                    const uint32_t tn = __shfl_down_sync(kFull, tk[0], 1);
                    const int i0 = 4 * lane;
                    auto pair_ok = [&](float la, uint32_t ta, float pa, float lb, uint32_t tb,
                                       float pb) {
                        return (la > lb && (ta < tb || pa > __fmul_rn(pb, sep))) || la == lb;
                    };
                    ok = (i0 + 1 >= n_c || pair_ok(lv[0], tk[0], pv[0], lv[1], tk[1], pv[1])) &&
                         (i0 + 2 >= n_c || pair_ok(lv[1], tk[1], pv[1], lv[2], tk[2], pv[2])) &&
                         (i0 + 3 >= n_c || pair_ok(lv[2], tk[2], pv[2], lv[3], tk[3], pv[3])) &&
                         (i0 + 4 >= n_c || pair_ok(lv[3], tk[3], pv[3], ln, tn, pn));
                }
                bool fast = __all_sync(kFull, ok) && argmax <= 110.0f;

                // ---- 7. top-k / top-p / min-p (src/zonos2_generate.cpp:55-84) on
                // prefix sums in 2^-24 fixed point: each term rounded to nearest (within
                // 2^-25; p_0 = 1, so every sum is >= 1), the sums themselves exact.  A
                // decision is taken where it clears the threshold by the reference's own
                // margin plus these errors; any other row goes to the exact form.  Every
                // candidate has p > 0 here (argmax <= 110), so the list is the first
                // m = min(n_c, K) candidates.
                const int m = min(n_c, K);
                int n = K;
                int hit = -1;   // 1 + the walk's position
                uint32_t P[4];
                {
                    uint32_t run = 0u;
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        run += 4 * lane + e < m ? __float2uint_rn(pv[e] * 0x1p24f) : 0u;
                        P[e] = run;
                    }
                    uint32_t incl = run;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const uint32_t y = __shfl_up_sync(kFull, incl, o);
                        if (lane >= o) incl += y;
                    }
                    const uint32_t excl = incl - run;
#pragma unroll
                    for (int e = 0; e < 4; e++) P[e] += excl;
                }
                // |sum~ / sum - 1| <= es.  The reference's running quotient sum over a
                // list of len terms is P_i / S * (1 + d), |d| <= (2 len - 1) * 2^-24 * 1.001
                // (sum_eta), against the exact sums; the f32 thresholds below take at
                // most four roundings (2^-22).
                const float es = eps_p + (float)n_c * 0x1p-25f;
                const float eta_c = 2.2f * es + (0x1p-22f + 0x1p-30f);
                // Each decision counts the positions certainly below / not certainly
                // above its threshold (P is non-decreasing along the list, p~ the same up
                // to its error): equal counts settle it, and the count is the position.
                auto P_at = [&](int i) { return __shfl_sync(kFull, sel4u(P, i & 3), i >> 2); };
                if (a.top_p < 1.0f) {
                    const float tpS = a.top_p * (float)P_at(m - 1);
                    const float eta = sum_eta(m) + eta_c;
                    const uint32_t lo = __float2uint_ru(tpS * (1.0f - eta));   // P < lo: below
                    const uint32_t hi = __float2uint_ru(tpS * (1.0f + 1.01f * eta));   // P >= hi: reached
                    int c = 0;
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        if (4 * lane + e < m) c += (P[e] < lo ? 1 : 0) + (P[e] < hi ? 0x10000 : 0);
                    c = __reduce_add_sync(kFull, c);
                    const int c_lo = c & 0xffff, c_hi = c >> 16;
                    if (c_lo < m) {   // else the sum never reaches top_p: no cut
                        n = c_lo + 1;
                        fast = fast && c_lo == c_hi;
                    }
                }
                if (a.min_p > 0.0f) {   // keep while p_i >= p_0 * min_p, p_0 = 1
                    const int mm = min(n, m);
                    const float em = (float)(kMinpEta * 1.01) + 2.2f * eps_p + 0x1p-22f;
                    const float keep = __fmul_rn(a.min_p, 1.0f + em);
                    const float drop = __fmul_rn(a.min_p, 1.0f - em);
                    int c = 0;
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        if (4 * lane + e < mm) c += (pv[e] >= keep ? 1 : 0) + (pv[e] >= drop ? 0x10000 : 0);
                    c = __reduce_add_sync(kFull, c);
                    n = c & 0xffff;   // the first position dropped (mm: none)
                    fast = fast && n == (c >> 16) && a.min_p >= 0x1p-100f;
                }
                // ---- 8. one uniform, CDF walk (src/zonos2_generate.cpp:86-92): the
                // first position whose partial sum reaches u
                {
                    const int len = min(n, m);
                    const float uS = u * (float)P_at(max(len, 1) - 1);
                    const float eta = sum_eta(len) + eta_c;
                    const uint32_t lo = __float2uint_ru(uS * (1.0f - eta));
                    const uint32_t hi = __float2uint_ru(uS * (1.0f + 1.01f * eta));
                    int c = 0;
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        if (4 * lane + e < len) c += (P[e] < lo ? 1 : 0) + (P[e] < hi ? 0x10000 : 0);
                    c = __reduce_add_sync(kFull, c);
                    hit = (c & 0xffff) + 1;
                    fast = fast && len > 0 && hit <= len && (c & 0xffff) == (c >> 16);
                }
                if (fast) {
                    const int pos = hit - 1;
                    tok = (int)__shfl_sync(kFull, sel4u(tk, pos & 3), pos >> 2);
                } else {
                    tok = exact_decide(region, exptab, n_c, K, V, a.pad_id, a.top_p, a.min_p,
                                       a.inv_temp, M, u, lane, lv[0], lv[1], lv[2], lv[3], tk[0],
                                       tk[1], tk[2], tk[3]);
                }
            }
        } else {
            __syncwarp();   // the row is free
            if (cb_nx < NCB) issue(s_nx, cb_nx);
        }

        // ---- 9. the code (over its parked uniform), flag and history
        if (!drawn) {
            grid_dep_wait();
            drawn = true;
        }
        if (lane == 0) {
            a.codes[r] = tok;
            if (a.flags) a.flags[r] = flag;
            if (hst) {
                int32_t *ring = a.hist + (size_t)r * a.hist_len;
                if (inc) {   // no waits: reductions, in this order on shared words
                    uint32_t *pm = a.presence + (size_t)r * 32;
                    uint32_t *cnt32 =
                        reinterpret_cast<uint32_t *>(a.counts + (size_t)r * kSamplerVocabMax);
                    if ((unsigned)ev < (unsigned)V && ((ev_old >> (16 * (ev & 1))) & 0xffffu) == 1u)
                        atomicAnd(pm + lm_word(ev), ~lm_bit(ev));   // its last occurrence left
                    if ((unsigned)tok < (unsigned)V) {
                        atomicAdd(cnt32 + (tok >> 1), 1u << (16 * (tok & 1)));
                        atomicOr(pm + lm_word(tok), lm_bit(tok));
                    }
                }
                ring[a.hist_pos] = tok;
            }
        }
        __syncwarp();
        s = s_nx;
        cb = cb_nx;
    }
}

// One warp per history ring: token counts in shared memory, then the u16
// counts and the lane-major presence bitmap (word l, bit 4*j + e: token
// 4*(l + 32*j) + e).
__global__ void __launch_bounds__(256) history_index_kernel(const int32_t *hist, long long rows,
                                                            int H, int V, uint16_t *counts,
                                                            uint32_t *presence)
{
    __shared__ uint32_t c[8][kSamplerVocabMax];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long long row = (long long)blockIdx.x * 8 + w;
    if (row >= rows) return;
    uint32_t *cw = c[w];
    for (int t = lane; t < kSamplerVocabMax; t += 32) cw[t] = 0u;
    __syncwarp();
    const int32_t *ring = hist + row * (size_t)H;
    for (int q = lane; q < H; q += 32) {
        const int t = ring[q];
        if ((unsigned)t < (unsigned)V) atomicAdd(cw + t, 1u);
    }
    __syncwarp();
    for (int t = lane; t < kSamplerVocabMax; t += 32)
        counts[row * (size_t)kSamplerVocabMax + t] = (uint16_t)cw[t];
    uint32_t bits = 0u;
#pragma unroll
    for (int i = 0; i < 32; i++) bits |= (cw[slot_token(lane, i)] > 0u ? 1u : 0u) << i;
    presence[row * 32 + lane] = bits;
}

cudaError_t launch_history_index(const int32_t *hist, long long rows, int hist_len, int vocab,
                                 uint16_t *counts, uint32_t *presence, cudaStream_t stream)
{
    if (rows == 0) return cudaSuccess;
    history_index_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(hist, rows, hist_len,
                                                                         vocab, counts, presence);
    return cudaGetLastError();
}

cudaError_t launch_draw_ahead(const uint64_t *rng_in, uint64_t *rng_out, int n_streams, int n_cb,
                              float *u, cudaStream_t stream)
{
    if (n_streams == 0) return cudaSuccess;
    draw_ahead_kernel<<<(unsigned)((n_streams + 127) / 128), 128, 0, stream>>>(rng_in, rng_out,
                                                                              n_streams, n_cb, u);
    return cudaGetLastError();
}

size_t sample_smem_bytes() { return (size_t)kCtaHeader + (size_t)kWarps * kWarpStride; }

namespace {

struct DeviceLaunchInfo {
    bool ready = false;
    int grid_cap = 0;   // resident CTAs of the sampler on this device
};
std::mutex g_launch_mu;
DeviceLaunchInfo g_launch_info[64];

cudaError_t launch_info(int dev, int *grid_cap)
{
    std::lock_guard<std::mutex> lk(g_launch_mu);
    DeviceLaunchInfo &d = g_launch_info[dev];
    if (!d.ready) {
        cudaError_t e = cudaFuncSetAttribute(sample_rows_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sample_smem_bytes());
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(sample_rows_kernel<true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)sample_smem_bytes());
        if (e != cudaSuccess) return e;
        int sms = 0, per_sm = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sample_rows_kernel<false>,
                                                          32 * kWarps, sample_smem_bytes());
        if (e != cudaSuccess) return e;
        d.grid_cap = sms * (per_sm > 0 ? per_sm : 1);
        d.ready = true;
    }
    *grid_cap = d.grid_cap;
    return cudaSuccess;
}

}  // namespace

cudaError_t launch_sample(const SampleArgs &a, cudaStream_t stream)
{
    if (a.n_streams == 0) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    int cap = 0;
    e = launch_info(dev, &cap);
    if (e != cudaSuccess) return e;

    if (!a.u_cur) {
        draw_uniforms_kernel<<<(unsigned)((a.n_streams + 127) / 128), 128, 0, stream>>>(
            a.rng, a.n_streams, a.n_cb, reinterpret_cast<uint32_t *>(a.codes));
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }

    // One CTA per SM, or per row when there are fewer rows than SMs: a small batch
    // spreads over as many SMs as it has rows.
    const long long rows = (long long)a.n_streams * a.n_cb;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows < cap ? rows : cap));
    cfg.blockDim = dim3(32 * kWarps);
    cfg.dynamicSmemBytes = sample_smem_bytes();
    cfg.stream = stream;
    // Programmatic dependent launch: behind the draw kernel the rows' copies start
    // before griddepcontrol.wait (the draw writes only the code slots); with
    // uniforms drawn ahead the kernel waits before its first global read, and only
    // its launch and set-up overlap the kernel before it.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // the decode context's launches take the instantiation specialised for them
    const bool ctx = a.vec_logits && a.u_cur && a.presence && a.hist && a.hist_len > 0 &&
                     (!a.allow || a.allow_lane_major);
    return ctx ? cudaLaunchKernelEx(&cfg, sample_rows_kernel<true>, a)
               : cudaLaunchKernelEx(&cfg, sample_rows_kernel<false>, a);
}

}  // namespace z2
