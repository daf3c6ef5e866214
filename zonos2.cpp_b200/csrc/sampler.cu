// sampler.cu -- fused per-row sampler for the zonos2 decode step (sm_100a).
//
// Restates, per (stream, codebook) row, the reference's sample_token
// (src/zonos2_generate.cpp:36-93) fed through the build-defined prologue
// (repetition penalty over the history window, allow bitmask, delay-pattern
// forcing, non-finite guard), with the row's uniform drawn from a per-stream
// Xoshiro256** in codebook order (src/zonos2_generate.cpp:259-267).
//
// Layout: one CTA per stream, one warp per codebook row.  A row of <= 1024
// logits lives in 32 registers per lane (lane l, slot 4*j + e holds token
// 4*(l + 32*j) + e, so every warp load is a coalesced 128-bit access).
//
// Each warp handles its own row.  After the prologue and the running max, a
// 128-bucket histogram of the gap (max - l), in buckets T/8 wide (the last one
// open-ended), finds the bucket B* holding the k-th largest logit.  Buckets
// <= B*+1 are the candidates: a superset of the top-k that also holds every
// logit whose probability could round equal to the k-th one's (equal
// probabilities need logits far closer than a bucket).  In the common case
// (<= 256 candidates) they are scattered into shared memory in bucket order,
// get an exact probability, and are put in (p desc, token asc) order by
// ranking each one inside its bucket; an adjacency check falls back to a
// bitonic sort if a probability tie straddles a bucket edge.  One running
// prefix sum of the sorted probabilities serves every sum the reference
// recomputes from zero, and lane 0 walks the CDFs over quotients p / sum that
// the warp divides out 32 at a time.  Other rows (top-k off, > 256
// candidates, degenerate distributions) take a slower general path.  Warp 0
// draws the stream's uniforms first and hands each codebook's warp its own
// through a per-warp named barrier.
//
// Exactness: every f32 operation that decides the token is the reference's
// own operation in the reference's order -- (l - max) / T, exp rounded
// correctly to f32, sums accumulated one term at a time in sorted order,
// p / sum divisions, the CDF walk -- so for equal inputs the token equals the
// reference's up to (a) equal-probability ties, taken in ascending token
// order, and (b) the reference's expf being misrounded by one ulp (glibc, on
// about 1e-4 of its inputs).  (l - max) / T is computed as an f64 product
// with RN(1/T) rounded to f32: the f64 error (< 2^-52 relative) cannot reach
// an f32 rounding boundary, which a quotient of two f32 values never comes
// closer to than 2^-48 relative, nor hits exactly.  Compiled with -fmad=false:
// no multiply-add is contracted.
#include <math.h>

#include "common.cuh"
#include "cr_exp.h"
#include "sampler.cuh"

namespace z2 {

namespace {

// Per-warp shared-memory region (bytes).  Common path:
//   [0, 2048)      candidates (logit, token), then sorted keys (<= 256 x u64)
//   [2048, 6144)   the row after the prologue, in token order; then, while
//                  ranking: unsorted keys [2048, 4096), sorted probabilities
//                  [4096, 5120), candidate buckets [5120, 5376); while
//                  deciding: p / sum [2048, 3072), prefix sums [3072, 4096)
//   [6144, 6656)   2^(j/64), j < 64, for the exp
//   [6656, 7680)   the bucket byte of every slot
//   [7680, 8192)   128 bucket counters, then bucket offsets
//   [8192, 8320)   1024-bit map of positive tokens (zero-tail fall-through)
// General path: up to 1024 keys over [0, 8192).  Scan-mode history: the
// 1024 seen-bytes in [0, 1024) during the prologue.
constexpr int kRegion = 8192;
constexpr int kWarpStride = kRegion + 144;  // + positive map; 16-byte skew between warps
constexpr int kValOffset = 2048;
constexpr int kKeyOffset = 2048;
constexpr int kPsOffset = 4096;
constexpr int kBucketOffset = 5120;
constexpr int kQOffset = 2048;
constexpr int kPfOffset = 3072;
constexpr int kExpTabOffset = 6144;
constexpr int kBktOffset = 6656;
constexpr int kHistOffset = 7680;
constexpr int kPosmapOffset = kRegion;
constexpr int kBuckets = 128;   // gap buckets: 0..126 finite, 127 marks a masked slot
constexpr int kRankMax = 256;   // candidates handled by the common path
constexpr int kHeader = 64;     // one uniform per codebook

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
// guard, repetition penalty, allow / delay mask.
__device__ __forceinline__ float prologue(float x, int i, uint32_t seenm, uint32_t allowm,
                                          float rho, float inv_rho)
{
    const bool fin = x < INFINITY;  // false for NaN and +inf
    if ((seenm >> i) & 1u) x = x * (x > 0.0f ? inv_rho : rho);
    return (fin && ((allowm >> i) & 1u)) ? x : -INFINITY;
}

// Gap bucket of a finite logit, 0..126 (the last one open-ended).  Buckets stay
// below 128 so that four of them compare against a bound in one subtraction.
__device__ __forceinline__ int bucket_of(float v, float M, float sc)
{
    return (int)fminf((M - v) * sc, (float)(kBuckets - 2));
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

__device__ __forceinline__ void named_arrive(int id, int n)
{
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
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
// (keys[0..n_pos)); one lane.
__device__ __noinline__ int zero_tail_token(const uint64_t *keys, int n_pos, uint32_t *posmap,
                                            int V, int want)
{
    for (int w = 0; w < 32; w++) posmap[w] = 0u;
    for (int i = 0; i < n_pos; i++) {
        const int t = key_tok(keys[i]);
        posmap[t >> 5] |= 1u << (t & 31);
    }
    for (int w = 0; w < 32; w++) {
        const int lo = 32 * w;
        if (lo >= V) break;
        const uint32_t valid = V - lo >= 32 ? ~0u : ((1u << (V - lo)) - 1u);
        uint32_t z = ~posmap[w] & valid;
        const int c = __popc(z);
        if (want < c) {
            for (; want > 0; want--) z &= z - 1;
            return lo + __ffs(z) - 1;
        }
        want -= c;
    }
    return -1;
}

// The token once the list is settled: position pos, or the last of n entries
// (a zero-probability token when the walk fell past the m positive ones).
__device__ __forceinline__ int pick_token(const uint64_t *keys, int pos, int n, int m, int n_pos,
                                          uint32_t *posmap, int V, int pad)
{
    const int m3 = min(n, m);
    if (pos >= 0) return key_tok(keys[pos]);
    if (n > m3) return zero_tail_token(keys, n_pos, posmap, V, n - 1 - m3);
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
// than 256 candidates): candidates compacted from a fresh read of the logits,
// bitonic sort, sums recomputed from the sorted keys.  Returns the token in
// lane 0.
__device__ __noinline__ int general_path(const RowKnobs &kn, unsigned char *region,
                                         const float *lrow, uint32_t selm, int n_c, float M,
                                         uint32_t seenm, uint32_t allowm, int lane, int cb,
                                         const float *uni)
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
    if (cb > 0) named_sync(cb, 64);
    int tok = kn.pad;
    if (lane == 0) {
        const float u = uni[cb];
        float cum = 0.0f;
        int pos = -1;
        for (int i = 0; i < min(n, m); i++) {
            cum += key_p(ent[i]) / S;
            if (u <= cum) {
                pos = i;
                break;
            }
        }
        tok = pick_token(ent, pos, n, m, n_pos,
                         reinterpret_cast<uint32_t *>(region + kPosmapOffset), kn.V, kn.pad);
    }
    return tok;
}

}  // namespace

// MAX_THREADS / MIN_BLOCKS: the 9-codebook model uses <288, 3> (three CTAs,
// 27 warps per SM at <= 72 registers); wider frames use <512, 1>.
template <int MAX_THREADS, int MIN_BLOCKS>
__global__ void __launch_bounds__(MAX_THREADS, MIN_BLOCKS) sample_kernel(const SampleArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int cb = threadIdx.x >> 5;
    const int s = blockIdx.x;
    const int V = a.vocab;
    float *uni = reinterpret_cast<float *>(smem);
    unsigned char *region = smem + kHeader + cb * kWarpStride;
    uint64_t *ent = reinterpret_cast<uint64_t *>(region);
    uint32_t *hist = reinterpret_cast<uint32_t *>(region + kHistOffset);
    uint32_t *bkt = reinterpret_cast<uint32_t *>(region + kBktOffset);
    double *exptab = reinterpret_cast<double *>(region + kExpTabOffset);
    const size_t row = (size_t)s * (size_t)a.n_cb + (size_t)cb;
    const int K = a.top_k;
    const bool topk_on = K > 0 && K < V;

    // ---- 1. the logits row -> registers; the exp table -> shared memory
    float v[32];
    const float *lrow = a.logits + row * (size_t)a.row_stride;
    if (a.vec_logits) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int t0 = 4 * (lane + 32 * j);
            float4 f = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            if (t0 < V) f = __ldg(reinterpret_cast<const float4 *>(lrow + t0));
            v[4 * j + 0] = f.x;
            v[4 * j + 1] = f.y;
            v[4 * j + 2] = f.z;
            v[4 * j + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int t = 4 * (lane + 32 * j) + e;
                v[4 * j + e] = t < V ? __ldg(lrow + t) : -INFINITY;
            }
    }
    exptab[lane] = exp2_64th(lane);
    exptab[lane + 32] = exp2_64th(lane + 32);

    // ---- 2. the stream's uniforms: warp 0 draws one per codebook, in codebook
    // order, and releases codebook c's warp through named barrier c
    if (cb == 0) {
        if (lane == 0) {
            ulonglong2 *sp = reinterpret_cast<ulonglong2 *>(a.rng + 4 * (size_t)s);
            const ulonglong2 st01 = sp[0], st23 = sp[1];
            Xo256 g{st01.x, st01.y, st23.x, st23.y};
            for (int c = 0; c < a.n_cb; c++) uni[c] = g.randf();
            sp[0] = make_ulonglong2(g.s0, g.s1);
            sp[1] = make_ulonglong2(g.s2, g.s3);
            __threadfence_block();
        }
        __syncwarp();
        for (int c = 1; c < a.n_cb; c++) named_arrive(c, 64);
    }

    // ---- 3. the history's token set: the context keeps it as a bitmap;
    // otherwise the ring is scanned into seen-bytes
    const bool pen = a.hist_len > 0 && a.rho != 1.0f;
    const bool inc = a.presence != nullptr;
    uint32_t seenm = 0u, allowm = ~0u;
    if (pen && inc) {
        const uint32_t pw = lane < a.allow_words
                                ? __ldcg(a.presence + row * (size_t)a.allow_words + lane)
                                : 0u;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t w = __shfl_sync(kFull, pw, (lane + 32 * j) >> 3);
            seenm |= ((w >> (4 * (lane & 7))) & 0xfu) << (4 * j);
        }
    } else if (pen) {
        uint4 *seen4 = reinterpret_cast<uint4 *>(region);
        seen4[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
        seen4[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
        const int32_t *hrow = a.hist + row * (size_t)a.hist_len;
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
                    mark_seen(region, t[u].x, V);
                    mark_seen(region, t[u].y, V);
                    mark_seen(region, t[u].z, V);
                    mark_seen(region, t[u].w, V);
                }
            }
        } else {
            for (int q = lane; q < H; q += 32) mark_seen(region, __ldcg(hrow + q), V);
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t wd = *reinterpret_cast<const uint32_t *>(region + 4 * (lane + 32 * j));
            seenm |= ((wd * 0x10204080u) >> 28) << (4 * j);   // four 0/1 bytes -> 4 bits
        }
    }

    // ---- 4. prologue: penalty, allow bits, delay forcing, non-finite guard
    if (a.allow) {
        const uint32_t aw = lane < a.allow_words ? __ldg(a.allow + (size_t)s * a.allow_words + lane)
                                                 : ~0u;
        allowm = 0u;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t w = __shfl_sync(kFull, aw, (lane + 32 * j) >> 3);
            allowm |= ((w >> (4 * (lane & 7))) & 0xfu) << (4 * j);
        }
    }
    if (a.delay_step >= 0 && a.delay_step < cb) {  // delay pattern: only the pad token
        const int p = a.pad_id;
        allowm &= lane == ((p >> 2) & 31) ? (1u << (4 * (p >> 7) + (p & 3))) : 0u;
    }
    bool nonfin = false;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        nonfin |= !(v[i] < INFINITY);
        v[i] = prologue(v[i], i, seenm, allowm, a.rho, a.inv_rho);
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    const bool live = mx >= -1e9f;  // running max starts at -1e9: :41-42
    const int flag = (__any_sync(kFull, nonfin) ? 2 : 0) | (live ? 0 : 1);
    {   // keep the row for the candidate scatter (the registers die after the histogram)
        float4 *vs = reinterpret_cast<float4 *>(region + kValOffset);
#pragma unroll
        for (int j = 0; j < 8; j++)
            vs[lane + 32 * j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }

    int tok = a.pad_id;
    if (live) {
        const float M = mx;
        const float T = a.temperature;
        // ---- 5. gap histogram and the bucket of the k-th largest logit.  The
        // open-ended last bucket holds most of a row: it is not counted with
        // atomics, its count follows from the number of finite logits.
        const float bw = fmaxf(T * 0.125f, fabsf(M) * 0x1p-18f + T * 0x1p-14f);
        const float sc = 1.0f / bw;
        reinterpret_cast<uint4 *>(hist)[lane] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
        int nf = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t pk = 0u;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float x = v[4 * j + e];
                const bool fin = x > -INFINITY;
                const int b = bucket_of(x, M, sc);
                if (fin && b < kBuckets - 2) atomicAdd(hist + b, 1u);
                nf += fin;
                pk |= (uint32_t)(fin ? b : kBuckets - 1) << (8 * e);
            }
            bkt[lane + 32 * j] = pk;
        }
        const int n_fin = __reduce_add_sync(kFull, nf);
        __syncwarp();
        const uint4 h4 = reinterpret_cast<const uint4 *>(hist)[lane];
        int h[4] = {(int)h4.x, (int)h4.y, (int)h4.z, (int)h4.w};
        int tot = h[0] + h[1] + h[2] + h[3];
        int incl = warp_incl_scan(tot, lane);
        if (lane == 31) {   // bucket 126 = 4*31 + 2
            const int rest = n_fin - incl;
            h[2] += rest;
            tot += rest;
            incl += rest;
        }
        int bc = kBuckets - 2;   // every finite logit
        if (topk_on && n_fin > K) {
            const int fl = __ffs(__ballot_sync(kFull, incl >= K)) - 1;
            int bstar = 0;
            if (lane == fl) {
                int c = incl - tot;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    c += h[i];
                    if (c >= K) {
                        bstar = 4 * lane + i;
                        break;
                    }
                }
            }
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
        if (!topk_on || n_c > kRankMax) {
            tok = general_path(kn, region, lrow, selm, n_c, M, seenm, allowm, lane, cb, uni);
        } else {
            // ---- 6. candidates -> shared memory in bucket order, from the row copy
            {
                const int c0 = incl - tot;
                reinterpret_cast<uint4 *>(hist)[lane] =
                    make_uint4(c0, c0 + h[0], c0 + h[0] + h[1], c0 + h[0] + h[1] + h[2]);
                __syncwarp();
            }
            const float *vs = reinterpret_cast<const float *>(region + kValOffset);
            uint32_t sm = selm;
            while (sm) {
                const int i = __ffs(sm) - 1;
                sm &= sm - 1;
                const int t = slot_token(lane, i);
                const int b = (bkt[lane + 32 * (i >> 2)] >> (8 * (i & 3))) & 0xff;
                const int pos = atomicAdd(hist + b, 1u);
                ent[pos] = make_ent(vs[t], t);
            }
            __syncwarp();

            // ---- 7. exact probabilities (src/zonos2_generate.cpp:44-49), keys
            // ranked inside their buckets
            const SmemExpTable tab{exptab};
            uint64_t *k2 = reinterpret_cast<uint64_t *>(region + kKeyOffset);
            unsigned char *kb = region + kBucketOffset;
            float *ps = reinterpret_cast<float *>(region + kPsOffset);
            int np = 0;
#pragma unroll 2
            for (int q = lane; q < n_c; q += 32) {
                const uint64_t en = ent[q];
                const float x = ent_v(en);
                const float p = row_prob(x, M, a.inv_temp, tab);
                np += p > 0.0f;
                k2[q] = make_key(p, (int)(uint32_t)en);
                kb[q] = (unsigned char)bucket_of(x, M, sc);
            }
            const int n_pos = __reduce_add_sync(kFull, np);
            __syncwarp();
#pragma unroll 2
            for (int q = lane; q < n_c; q += 32) {
                const uint64_t key = k2[q];
                const int b = kb[q];
                const int lo = b ? (int)hist[b - 1] : 0;
                const int hi = (int)hist[b];
                int rank = 0, i = lo;
                for (; i + 2 <= hi; i += 2) rank += (k2[i] > key) + (k2[i + 1] > key);
                if (i < hi) rank += k2[i] > key;
                ent[lo + rank] = key;
                ps[lo + rank] = key_p(key);
            }
            __syncwarp();
            bool bad = false;
            for (int q = lane; q + 1 < n_c; q += 32) bad |= ent[q] < ent[q + 1];
            if (__any_sync(kFull, bad)) {   // a probability tie across a bucket edge
                int N = 32;
                while (N < n_c) N <<= 1;
                for (int i = n_c + lane; i < N; i += 32) ent[i] = 0ull;
                __syncwarp();
                bitonic_smem_desc(ent, N, lane);
                for (int q = lane; q < n_c; q += 32) ps[q] = key_p(ent[q]);
                __syncwarp();
            }

            // ---- 8. top-k / top-p / min-p (src/zonos2_generate.cpp:55-84).  The
            // list is ent[0..m) (positive probabilities, sorted) followed by
            // zero-probability tokens in token order, n entries in all; every sum
            // the reference recomputes from zero over a sorted prefix is one of
            // the running prefix sums.
            const int m = min(n_pos, K);
            int n = K;
            float *pf = reinterpret_cast<float *>(region + kPfOffset);
            float *q = reinterpret_cast<float *>(region + kQOffset);
            if (lane == 0) prefix_sums(ps, pf, m);
            __syncwarp();
            float S = pf[m - 1];
            if (a.top_p < 1.0f) {
                const int cut = walk_cdf(ps, q, m, S, a.top_p, lane);
                if (cut > 0) n = cut;  // never inside the zero tail: the sum stops growing
                S = pf[min(n, m) - 1];
            }
            if (a.min_p > 0.0f) {
                const float thresh = (ps[0] / S) * a.min_p;
                const int mm = min(n, m);
                int j = minp_cut(ps, mm, S, thresh, lane);
                if (j == mm && n > mm) j = (0.0f >= thresh) ? n : mm;
                n = j;
                S = pf[min(n, m) - 1];
            }
            if (cb > 0) named_sync(cb, 64);   // this codebook's uniform is in shared memory
            // ---- 9. one uniform, CDF walk (src/zonos2_generate.cpp:86-92)
            const int hit = walk_cdf(ps, q, min(n, m), S, uni[cb], lane);
            if (lane == 0)
                tok = pick_token(ent, hit > 0 ? hit - 1 : -1, n, m, n_pos,
                                 reinterpret_cast<uint32_t *>(region + kPosmapOffset), V,
                                 a.pad_id);
        }
    } else if (cb > 0) {
        named_sync(cb, 64);
    }

    if (lane == 0) {
        a.codes[row] = tok;
        if (a.flags) a.flags[row] = flag;
        if (a.hist && a.hist_len > 0) {
            int32_t *ring = a.hist + row * (size_t)a.hist_len;
            if (inc) {   // the evicted token leaves the index, the new one enters
                const int ev = __ldcg(ring + a.hist_pos);
                uint16_t *cnt = a.counts + row * (size_t)V;
                uint32_t *pm = a.presence + row * (size_t)a.allow_words;
                if ((unsigned)ev < (unsigned)V) {
                    const unsigned c = cnt[ev] - 1u;
                    cnt[ev] = (uint16_t)c;
                    if (c == 0u) pm[ev >> 5] &= ~(1u << (ev & 31));
                }
                if ((unsigned)tok < (unsigned)V) {
                    const unsigned c = cnt[tok];
                    cnt[tok] = (uint16_t)(c + 1u);
                    if (c == 0u) pm[tok >> 5] |= 1u << (tok & 31);
                }
            }
            ring[a.hist_pos] = tok;
        }
    }
}

// One warp per history ring: token counts in shared memory, then the u16
// counts and the presence bitmap.
__global__ void __launch_bounds__(256) history_index_kernel(const int32_t *hist, long long rows,
                                                            int H, int V, int words,
                                                            uint16_t *counts, uint32_t *presence)
{
    __shared__ uint32_t c[8][kSamplerVocabMax];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long long row = (long long)blockIdx.x * 8 + w;
    if (row >= rows) return;
    uint32_t *cw = c[w];
    for (int t = lane; t < V; t += 32) cw[t] = 0u;
    __syncwarp();
    const int32_t *ring = hist + row * (size_t)H;
    for (int q = lane; q < H; q += 32) {
        const int t = ring[q];
        if ((unsigned)t < (unsigned)V) atomicAdd(cw + t, 1u);
    }
    __syncwarp();
    for (int t = lane; t < V; t += 32) counts[row * (size_t)V + t] = (uint16_t)cw[t];
    for (int wd = 0; wd < words; wd++) {
        const int t = 32 * wd + lane;
        const uint32_t bits = __ballot_sync(kFull, t < V && cw[t] > 0u);
        if (lane == 0) presence[row * (size_t)words + wd] = bits;
    }
}

cudaError_t launch_history_index(const int32_t *hist, long long rows, int hist_len, int vocab,
                                 uint16_t *counts, uint32_t *presence, cudaStream_t stream)
{
    if (rows == 0) return cudaSuccess;
    const int words = (vocab + 31) / 32;
    history_index_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(
        hist, rows, hist_len, vocab, words, counts, presence);
    return cudaGetLastError();
}

size_t sample_smem_bytes(int n_cb) { return (size_t)kHeader + (size_t)n_cb * kWarpStride; }

template <int MAX_THREADS, int MIN_BLOCKS>
static cudaError_t launch_variant(const SampleArgs &a, cudaStream_t stream, bool *attr_done)
{
    const int max_cb = MAX_THREADS / 32;
    if (!*attr_done) {
        const cudaError_t e =
            cudaFuncSetAttribute(sample_kernel<MAX_THREADS, MIN_BLOCKS>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sample_smem_bytes(max_cb));
        if (e != cudaSuccess) return e;
        *attr_done = true;
    }
    sample_kernel<MAX_THREADS, MIN_BLOCKS>
        <<<a.n_streams, 32 * a.n_cb, sample_smem_bytes(a.n_cb), stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_sample(const SampleArgs &a, cudaStream_t stream)
{
    if (a.n_streams == 0) return cudaSuccess;
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    static bool attr_narrow[64] = {false};
    static bool attr_wide[64] = {false};
    if (a.n_cb <= 9) return launch_variant<288, 3>(a, stream, &attr_narrow[dev]);
    return launch_variant<32 * kSamplerCbMax, 1>(a, stream, &attr_wide[dev]);
}

}  // namespace z2
