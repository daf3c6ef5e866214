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
// Every warp handles its own row: prologue, running max, a 256-bucket
// histogram of the gap (max - l) in buckets T/8 wide (the last one open), the bucket B* holding
// the k-th largest logit.  Buckets <= B*+1 are the candidates: a superset of
// the top-k that also holds every logit whose probability could round equal
// to the k-th one's (equal probabilities need logits far closer than a
// bucket).  Candidates are scattered into shared memory in bucket order, get
// an exact probability, and are put in (p desc, token asc) order by ranking
// each one inside its bucket; a final adjacency check falls back to a bitonic
// sort if a probability tie straddles a bucket edge.
// Then one lane runs the reference's sequential top-k / top-p / min-p sums and
// CDF walk in its exact order, over quotients p / sum that the whole warp
// divides out beforehand.  Warp 0 draws the stream's uniforms first and hands
// each codebook's warp its own through a per-warp named barrier.
//
// Exactness: every f32 operation that decides the token is the reference's
// own operation in the reference's order -- (l - max) / T, exp rounded
// correctly to f32, sums accumulated one term at a time in sorted order,
// p / sum divisions, the CDF walk -- so for equal inputs the token equals the
// reference's up to (a) equal-probability ties, taken in ascending token
// order, and (b) the reference's expf being misrounded by one ulp (glibc, on
// about 1e-4 of its inputs).  Compiled with -fmad=false: no multiply-add is
// contracted.
#include <math.h>

#include "common.cuh"
#include "sampler.cuh"

namespace z2 {

namespace {

constexpr int kRegion = 8192;              // per-warp union region (1024 x u64)
constexpr int kWarpStride = kRegion + 144; // + positive map; 16-byte skew between warps
constexpr int kPosmapOffset = kRegion;     // 1024-bit map for the zero-probability tail
constexpr int kBuckets = 128;              // gap buckets: 0..126 finite, 127 masked
constexpr int kHistOffset = 7680;          // 128 bucket counters at the region's end
constexpr int kBktOffset = 6656;           // the bucket byte of every slot (1024 bytes)
constexpr int kScatterMax = 832;           // candidates that fit below the bucket bytes
constexpr int kRankMax = 256;              // candidates ranked inside their buckets
// while ranking (<= 256 candidates):
constexpr int kKeyOffset = 2048;           //   unsorted keys                 [2048, 4096)
constexpr int kPsOffset = 4096;            //   sorted probabilities          [4096, 5120)
constexpr int kBucketOffset = 5120;        //   candidate buckets             [5120, 5376)
// while deciding (<= 256 candidates, keys sorted in [0, 2048)):
constexpr int kQOffset = 2048;             //   p / sum                       [2048, 3072)
constexpr int kPfOffset = 3072;            //   prefix sums of the sorted p   [3072, 4096)
constexpr int kHeader = 64;                // one uniform per codebook

__device__ __forceinline__ float cr_exp(float x)
{
    // exp correctly rounded to f32: the f64 result is within one f64 ulp and
    // no f32 rounding boundary of an input in [-104, 0] lies that close.
    return __double2float_rn(exp((double)x));
}

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

__device__ __forceinline__ int warp_incl_scan(int x, int lane)
{
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    return x;
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
__device__ __forceinline__ float seq_sum(const uint64_t *keys, int m)
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

__device__ __forceinline__ void mark_seen(unsigned char *seen, int t, int vocab)
{
    if ((unsigned)t < (unsigned)vocab) seen[t] = 1;
}

// Gap bucket of a finite logit, 0..126 (the last one open-ended); 127 marks a
// masked slot.  Buckets stay below 128 so four of them compare against a
// bound in one 32-bit subtraction.
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

// Running f32 prefix sums pf[i] = ps[0] + ... + ps[i], one term at a time (one lane).
__device__ __forceinline__ void prefix_sums(const float *ps, float *pf, int m)
{
    float P = 0.0f;
    int i = 0;
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
__device__ int walk_cdf(const float *ps, float *q, int len, float S, float thr, int lane)
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

// The (want)-th token, in token order, outside the positive set of a row
// (keys[0..n_pos)); one lane.
__device__ int zero_tail_token(const uint64_t *keys, int n_pos, uint32_t *posmap, int V,
                               int want)
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

}  // namespace

// The build-defined prologue of one logit (slot i of this lane): non-finite
// guard, repetition penalty, allow / delay mask.
__device__ __forceinline__ float prologue(float x, int i, uint32_t seenm, uint32_t allowm,
                                          float rho, float inv_rho)
{
    const bool fin = x < INFINITY;  // false for NaN and +inf
    if ((seenm >> i) & 1u) x = x * (x > 0.0f ? inv_rho : rho);
    return (fin && ((allowm >> i) & 1u)) ? x : -INFINITY;
}

__device__ __forceinline__ void named_arrive(int id, int n)
{
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

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
    const size_t row = (size_t)s * (size_t)a.n_cb + (size_t)cb;
    const float T = a.temperature;
    const int K = a.top_k;
    const bool topk_on = K > 0 && K < V;

    // ---- 1. the logits row -> registers
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

    // ---- 3. repetition set: seen[t] = 1 for every token of the history window
    const bool pen = a.hist_len > 0 && a.rho != 1.0f;
    if (pen) {
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
    }

    // ---- 4. prologue: penalty, allow bits, delay forcing, non-finite guard
    uint32_t seenm = 0u, allowm = ~0u;
    if (pen) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t wd = *reinterpret_cast<const uint32_t *>(region + 4 * (lane + 32 * j));
            seenm |= ((wd * 0x10204080u) >> 28) << (4 * j);   // four 0/1 bytes -> 4 bits
        }
    }
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

    int tok = a.pad_id;
    if (live) {
        const float M = mx;
        // ---- 5. gap histogram and the bucket of the k-th largest logit
        const float bw = fmaxf(T * 0.125f, fabsf(M) * 0x1p-18f + T * 0x1p-14f);
        const float sc = 1.0f / bw;
        reinterpret_cast<uint4 *>(hist)[lane] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t pk = 0u;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float x = v[4 * j + e];
                const bool fin = x > -INFINITY;
                const int b = bucket_of(x, M, sc);
                if (fin) atomicAdd(hist + b, 1u);
                pk |= (uint32_t)(fin ? b : kBuckets - 1) << (8 * e);
            }
            bkt[lane + 32 * j] = pk;
        }
        __syncwarp();
        const uint4 h4 = reinterpret_cast<const uint4 *>(hist)[lane];
        const int h[4] = {(int)h4.x, (int)h4.y, (int)h4.z, (int)h4.w};
        const int tot = h[0] + h[1] + h[2] + h[3];
        const int incl = warp_incl_scan(tot, lane);
        const int n_fin = __shfl_sync(kFull, incl, 31);
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
        const bool fast = topk_on && n_c <= kScatterMax;
        const uint32_t bc4 = 0x80808080u | ((uint32_t)bc * 0x01010101u);
        uint32_t selm = 0u;   // this lane's candidate slots
#pragma unroll
        for (int j = 0; j < 8; j++) selm |= bytes_le(bkt[lane + 32 * j], bc4) << (4 * j);

        // ---- 6. candidates -> shared memory as (logit, token).  The row's
        // registers are gone by now: the few candidates are read again (L1
        // hits) and pass through the same prologue.
        if (fast) {
            {   // exclusive bucket offsets become scatter cursors (bucket order)
                const int c0 = incl - tot;
                reinterpret_cast<uint4 *>(hist)[lane] =
                    make_uint4(c0, c0 + h[0], c0 + h[0] + h[1], c0 + h[0] + h[1] + h[2]);
                __syncwarp();
            }
            uint32_t sm = selm;
            while (sm) {
                const int i = __ffs(sm) - 1;
                sm &= sm - 1;
                const int t = 4 * (lane + 32 * (i >> 2)) + (i & 3);
                const float x = prologue(__ldg(lrow + t), i, seenm, allowm, a.rho, a.inv_rho);
                const int b = (bkt[lane + 32 * (i >> 2)] >> (8 * (i & 3))) & 0xff;
                const int pos = atomicAdd(hist + b, 1u);
                ent[pos] = make_ent(x, t);
            }
        } else if (topk_on) {
            // lane-major compaction (the entries may grow over the bucket bytes)
            const int cnt = __popc(selm);
            int off = warp_incl_scan(cnt, lane) - cnt;
            __syncwarp();
            uint32_t sm = selm;
            while (sm) {
                const int i = __ffs(sm) - 1;
                sm &= sm - 1;
                const int t = 4 * (lane + 32 * (i >> 2)) + (i & 3);
                ent[off++] = make_ent(prologue(__ldg(lrow + t), i, seenm, allowm, a.rho, a.inv_rho), t);
            }
        } else {
            // top-k off: every finite logit, in token order (the token-order sum)
            __syncwarp();
            int base = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const uint32_t nib = (selm >> (4 * j)) & 0xfu;
                const int cnt = __popc(nib);
                const int inc = warp_incl_scan(cnt, lane);
                int off = base + inc - cnt;
#pragma unroll
                for (int e = 0; e < 4; e++)
                    if ((nib >> e) & 1u) {
                        const int t = 4 * (lane + 32 * j) + e;
                        ent[off++] = make_ent(prologue(__ldg(lrow + t), 4 * j + e, seenm, allowm,
                                                       a.rho, a.inv_rho), t);
                    }
                base += __shfl_sync(kFull, inc, 31);
            }
        }
        __syncwarp();

        // ---- 7. exact probabilities (src/zonos2_generate.cpp:44-49) and order
        int np = 0;
        float s0 = 0.0f;
        const bool small = fast && n_c <= kRankMax;
        float *ps = reinterpret_cast<float *>(region + kPsOffset);
        if (small) {
            // unsorted keys and their buckets beside the (logit, token) entries,
            // then every key is ranked inside its bucket and stored in place
            uint64_t *k2 = reinterpret_cast<uint64_t *>(region + kKeyOffset);
            unsigned char *kb = region + kBucketOffset;
            for (int q = lane; q < n_c; q += 32) {
                const uint64_t en = ent[q];
                const float x = __uint_as_float((uint32_t)(en >> 32));
                const float p = cr_exp(__fdiv_rn(__fsub_rn(x, M), T));
                np += p > 0.0f;
                k2[q] = make_key(p, (int)(uint32_t)en);
                kb[q] = (unsigned char)bucket_of(x, M, sc);
            }
            __syncwarp();
            for (int q = lane; q < n_c; q += 32) {
                const uint64_t key = k2[q];
                const int b = kb[q];
                const int lo = b ? (int)hist[b - 1] : 0;
                const int hi = (int)hist[b];
                int rank = 0;
                for (int i = lo; i < hi; i++) rank += k2[i] > key;
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
        } else {
            for (int q = lane; q < n_c; q += 32) {
                const uint64_t en = ent[q];
                const float x = __uint_as_float((uint32_t)(en >> 32));
                const float p = cr_exp(__fdiv_rn(__fsub_rn(x, M), T));
                np += p > 0.0f;
                ent[q] = make_key(p, (int)(uint32_t)en);
            }
            __syncwarp();
            if (!topk_on && lane == 0) s0 = seq_sum(ent, n_c);  // token-order sum
            int N = 32;
            while (N < n_c) N <<= 1;
            for (int i = n_c + lane; i < N; i += 32) ent[i] = 0ull;
            __syncwarp();
            bitonic_smem_desc(ent, N, lane);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) np += __shfl_xor_sync(kFull, np, o);
        const int n_pos = np;
        s0 = __shfl_sync(kFull, s0, 0);

        // ---- 8. top-k / top-p / min-p (src/zonos2_generate.cpp:55-84).  The
        // list is ent[0..m) (positive probabilities, sorted) followed by
        // zero-probability tokens in token order, n entries in all.  Every
        // sum the reference recomputes from zero over a sorted prefix is one
        // entry of the running prefix sums.
        const int n_list = topk_on ? K : V;
        const int m = min(n_pos, n_list);
        int n = n_list;
        int pos = -1;
        if (small) {
            float *pf = reinterpret_cast<float *>(region + kPfOffset);
            float *q = reinterpret_cast<float *>(region + kQOffset);
            if (lane == 0) prefix_sums(ps, pf, m);
            __syncwarp();
            float S = topk_on ? pf[m - 1] : s0;
            if (a.top_p < 1.0f) {
                const int cut = walk_cdf(ps, q, m, S, a.top_p, lane);
                if (cut > 0) n = cut;  // never inside the zero tail: the sum stops growing
                S = pf[min(n, m) - 1];
            }
            if (a.min_p > 0.0f && n > 0) {
                const float thresh = (ps[0] / S) * a.min_p;
                const int mm = min(n, m);
                int j = mm;
                for (int base = 0; base < mm; base += 32) {
                    const int i = base + lane;
                    const uint32_t fails = __ballot_sync(kFull, i < mm && !(ps[i] / S >= thresh));
                    if (fails) {
                        j = base + __ffs(fails) - 1;
                        break;
                    }
                }
                if (j == mm && n > mm) j = (0.0f >= thresh) ? n : mm;
                n = j;
                S = pf[min(n, m) - 1];
            }
            if (cb > 0) named_sync(cb, 64);   // this codebook's uniform is in shared memory
            // ---- 9. one uniform, CDF walk (src/zonos2_generate.cpp:86-92)
            const int hit = walk_cdf(ps, q, min(n, m), S, uni[cb], lane);
            pos = hit > 0 ? hit - 1 : -1;
        } else {
            float S = topk_on ? (lane == 0 ? seq_sum(ent, m) : 0.0f) : s0;
            S = __shfl_sync(kFull, S, 0);
            if (a.top_p < 1.0f) {
                int cut = -1;
                if (lane == 0) {
                    float cum = 0.0f;
                    for (int i = 0; i < m; i++) {
                        cum += key_p(ent[i]) / S;
                        if (cum >= a.top_p) {
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
            if (a.min_p > 0.0f && n > 0) {
                const float thresh = (key_p(ent[0]) / S) * a.min_p;
                const int mm = min(n, m);
                int j = mm;
                for (int base = 0; base < mm; base += 32) {
                    const int i = base + lane;
                    const uint32_t fails =
                        __ballot_sync(kFull, i < mm && !(key_p(ent[i]) / S >= thresh));
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
            if (lane == 0) {
                const float u = uni[cb];
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
        }
        if (lane == 0) {
            const int m3 = min(n, m);
            if (pos >= 0) tok = key_tok(ent[pos]);
            else if (n > m3)   // the last entry is a zero-probability token
                tok = zero_tail_token(ent, n_pos,
                                      reinterpret_cast<uint32_t *>(region + kPosmapOffset), V,
                                      n - 1 - m3);
            else if (n > 0) tok = key_tok(ent[n - 1]);
        }
    } else if (cb > 0) {
        named_sync(cb, 64);
    }
    if (lane == 0) {
        a.codes[row] = tok;
        if (a.flags) a.flags[row] = flag;
        if (a.hist && a.hist_len > 0) a.hist[row * (size_t)a.hist_len + a.hist_pos] = tok;
    }
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
