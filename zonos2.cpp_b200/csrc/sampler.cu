// sampler.cu -- fused per-row sampler for the zonos2 decode step (sm_100a).
//
// Restates, per (stream, codebook) row, the reference's sample_token
// (src/zonos2_generate.cpp:36-93) fed through the build-defined prologue
// (repetition penalty over the history window, allow bitmask, delay-pattern
// forcing, non-finite guard), with the row's uniform drawn from a per-stream
// Xoshiro256** in codebook order (src/zonos2_generate.cpp:259-267).
//
// Layout: one CTA per stream, one warp per codebook row; a row of <= 1024
// logits lives in 32 registers per lane (lane l, slot (j, e) holds token
// 4*(l + 32*j) + e, so every warp load is a coalesced 128-bit access).
//
// Exactness: every f32 operation that decides the token is the reference's
// own operation in the reference's order -- (l - max) / T, exp rounded
// correctly to f32, the top-k / top-p / min-p sums accumulated sequentially in
// sorted order by one lane, p / sum divisions, the CDF walk -- so for equal
// inputs the token equals the reference's up to (a) equal-probability ties,
// which are taken in ascending token order, and (b) the reference's expf
// being misrounded by one ulp (glibc, about 1e-4 of inputs).  The file is
// compiled with -fmad=false so no multiply-add is contracted.
//
// Work per row: the full row only passes through cheap per-element steps
// (prologue, max, a 256-bucket histogram of (max - l) scaled to T/4-wide
// buckets).  The bucket holding the k-th largest logit plus one bucket of
// slack bounds the candidate set (a superset of the top-k, including any
// logit whose probability could round equal to the k-th), and only those
// candidates get an exact exp, a bitonic sort on (p desc, token asc) keys and
// the sequential sums.
#include <math.h>

#include "common.cuh"
#include "sampler.cuh"

namespace z2 {

namespace {

constexpr int kHeader = 128;           // per-CTA uniforms, one per codebook
constexpr int kRegion = 8192;          // per-warp union region (1024 x u64)
constexpr int kWarpStride = kRegion + 128;  // + 1024-bit positive map
constexpr int kHistOffset = 1024;      // bucket histogram after the seen bytes
constexpr int kQOffset = 2048;         // q = p / sum, when <= 256 keys are sorted
constexpr int kQCap = 256;

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

__device__ __forceinline__ int warp_sum(int x)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
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

// Descending bitonic sort of 32*E keys held E per lane (element lane*E + r).
template <int E>
__device__ __forceinline__ void bitonic_regs_desc(uint64_t (&k)[E], int lane)
{
#pragma unroll
    for (int size = 2; size <= 32 * E; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= E) {
                const int ls = stride / E;
                const bool desc = ((lane * E) & size) == 0;
                const bool lower = ((lane * E) & stride) == 0;
                const bool keep_max = desc == lower;
#pragma unroll
                for (int r = 0; r < E; r++) {
                    const uint64_t o = __shfl_xor_sync(kFull, k[r], ls);
                    k[r] = keep_max ? (k[r] > o ? k[r] : o) : (k[r] < o ? k[r] : o);
                }
            } else {
#pragma unroll
                for (int r = 0; r < E; r++) {
                    if ((r & stride) == 0) {
                        const bool desc = ((lane * E + r) & size) == 0;
                        const uint64_t x = k[r], y = k[r + stride];
                        const bool sw = desc ? (x < y) : (x > y);
                        k[r] = sw ? y : x;
                        k[r + stride] = sw ? x : y;
                    }
                }
            }
        }
    }
}

template <int E>
__device__ __forceinline__ void sort_keys_regs(uint64_t *ent, int n_c, int lane)
{
    uint64_t k[E];
#pragma unroll
    for (int r = 0; r < E; r++) {
        const int i = lane * E + r;
        k[r] = i < n_c ? ent[i] : 0ull;
    }
    __syncwarp();
    bitonic_regs_desc<E>(k, lane);
#pragma unroll
    for (int r = 0; r < E; r++) ent[lane * E + r] = k[r];
    __syncwarp();
}

// Descending bitonic sort of n (power of two, <= 1024) keys in shared memory.
__device__ void bitonic_smem_desc(uint64_t *keys, int n, int lane)
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

// Sequential f32 sum of the probabilities of keys[0..m), in order.
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

__device__ __forceinline__ void finish_row(const SampleArgs &a, size_t row, int tok, int flag)
{
    a.codes[row] = tok;
    if (a.flags) a.flags[row] = flag;
    if (a.hist && a.hist_len > 0) a.hist[row * (size_t)a.hist_len + a.hist_pos] = tok;
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
    uint32_t *posmap = reinterpret_cast<uint32_t *>(region + kRegion);
    const size_t row = (size_t)s * (size_t)a.n_cb + (size_t)cb;

    // ---- 1. the logits row -> registers (issued first, consumed in step 4)
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

    // ---- 2. repetition set: seen[t] = 1 for every token of the history window
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
    }

    // ---- 3. the stream's uniforms: one draw per codebook, in codebook order
    if (threadIdx.x == 0) {
        uint64_t *st = a.rng + 4 * (size_t)s;
        Xo256 g{st[0], st[1], st[2], st[3]};
        for (int c = 0; c < a.n_cb; c++) uni[c] = g.randf();
        st[0] = g.s0;
        st[1] = g.s1;
        st[2] = g.s2;
        st[3] = g.s3;
    }
    __syncthreads();

    // ---- 4. prologue: non-finite guard, penalty, allow bits, delay forcing
    const bool force = a.delay_step >= 0 && a.delay_step < cb;
    uint32_t aw = ~0u;
    if (a.allow && lane < a.allow_words) aw = __ldg(a.allow + (size_t)s * a.allow_words + lane);
    bool nonfin = false;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int t0 = 4 * (lane + 32 * j);
        const uint32_t sn = pen ? *reinterpret_cast<const uint32_t *>(region + t0) : 0u;
        const uint32_t w = __shfl_sync(kFull, aw, (lane + 32 * j) >> 3);
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int t = t0 + e;
            float x = v[4 * j + e];
            if (!(x < INFINITY)) {
                nonfin |= t < V;
                x = -INFINITY;
            }
            if ((sn >> (8 * e)) & 0xffu) x = x > 0.0f ? x * a.inv_rho : x * a.rho;
            if (!((w >> (t & 31)) & 1u)) x = -INFINITY;
            if (force && t != a.pad_id) x = -INFINITY;
            v[4 * j + e] = x;
        }
    }

    // ---- 5. running max from -1e9 (src/zonos2_generate.cpp:41-42), liveness
    float mx = v[0];
#pragma unroll
    for (int i = 1; i < 32; i++) mx = fmaxf(mx, v[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    const bool live = mx >= -1e9f;
    const int flag = (__any_sync(kFull, nonfin) ? 2 : 0) | (live ? 0 : 1);
    if (!live) {
        if (lane == 0) finish_row(a, row, a.pad_id, flag);
        return;
    }
    const float M = mx;
    const float T = a.temperature;
    const int K = a.top_k;
    const bool topk_on = K > 0 && K < V;

    // ---- 6. candidate bound: bucket of the k-th largest logit, plus one
    int nf = 0;
#pragma unroll
    for (int i = 0; i < 32; i++) nf += v[i] > -INFINITY;
    const int n_fin = warp_sum(nf);
    const float bw = fmaxf(T * 0.25f, fabsf(M) * 0x1p-18f + T * 0x1p-14f);
    const float sc = 1.0f / bw;
    float sel_lim = INFINITY;  // selected iff finite and (M - v) * sc < sel_lim
    if (topk_on && n_fin > K) {
        uint32_t *hist = reinterpret_cast<uint32_t *>(region + kHistOffset);
        reinterpret_cast<uint4 *>(hist)[2 * lane] = make_uint4(0u, 0u, 0u, 0u);
        reinterpret_cast<uint4 *>(hist)[2 * lane + 1] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (v[i] > -INFINITY) {
                const int b = (int)fminf((M - v[i]) * sc, 255.0f);
                atomicAdd(hist + b, 1u);
            }
        __syncwarp();
        const uint4 h0 = reinterpret_cast<const uint4 *>(hist)[2 * lane];
        const uint4 h1 = reinterpret_cast<const uint4 *>(hist)[2 * lane + 1];
        const int hb[8] = {(int)h0.x, (int)h0.y, (int)h0.z, (int)h0.w,
                           (int)h1.x, (int)h1.y, (int)h1.z, (int)h1.w};
        int tot = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) tot += hb[i];
        const int incl = warp_incl_scan(tot, lane);
        const int fl = __ffs(__ballot_sync(kFull, incl >= K)) - 1;  // exists: total > K
        int bstar = 0;
        if (lane == fl) {
            int c = incl - tot;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                c += hb[i];
                if (c >= K) {
                    bstar = 8 * lane + i;
                    break;
                }
            }
        }
        bstar = __shfl_sync(kFull, bstar, fl);
        const int bc = min(bstar + 1, 255);
        if (bc < 255) sel_lim = (float)(bc + 1);
        __syncwarp();
    }

    // ---- 7. compaction of candidates as (logit bits, token)
    uint64_t *ent = reinterpret_cast<uint64_t *>(region);
    int n_c;
    if (topk_on) {
        // lane-major order: the sort key carries the token, order is irrelevant
        uint32_t selm = 0;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const bool sl = v[i] > -INFINITY && (sel_lim == INFINITY || (M - v[i]) * sc < sel_lim);
            selm |= (uint32_t)sl << i;
        }
        const int cnt = __popc(selm);
        const int incl = warp_incl_scan(cnt, lane);
        n_c = __shfl_sync(kFull, incl, 31);
        int off = incl - cnt;
#pragma unroll
        for (int i = 0; i < 32; i++)
            if ((selm >> i) & 1u) {
                const int t = 4 * (lane + 32 * (i >> 2)) + (i & 3);
                ent[off++] = ((uint64_t)__float_as_uint(v[i]) << 32) | (uint32_t)t;
            }
    } else {
        // token order: the top-k-off sum runs over the row in token order
        int base = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int cnt = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) cnt += v[4 * j + e] > -INFINITY;
            const int incl = warp_incl_scan(cnt, lane);
            int off = base + incl - cnt;
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (v[4 * j + e] > -INFINITY) {
                    const int t = 4 * (lane + 32 * j) + e;
                    ent[off++] = ((uint64_t)__float_as_uint(v[4 * j + e]) << 32) | (uint32_t)t;
                }
            base += __shfl_sync(kFull, incl, 31);
        }
        n_c = base;
    }
    __syncwarp();

    // ---- 8. exact probabilities (src/zonos2_generate.cpp:44-49) as sort keys
    int np = 0;
    for (int q = lane; q < n_c; q += 32) {
        const uint64_t en = ent[q];
        const float x = __uint_as_float((uint32_t)(en >> 32));
        const int t = (int)(uint32_t)en;
        const float p = cr_exp(__fdiv_rn(__fsub_rn(x, M), T));
        np += p > 0.0f;
        ent[q] = make_key(p, t);
    }
    const int n_pos = warp_sum(np);
    __syncwarp();
    float S = 0.0f;
    if (!topk_on && lane == 0) S = seq_sum(ent, n_c);  // token-order sum

    int N = 32;
    while (N < n_c) N <<= 1;
    if (N <= 256) {
        if (N == 32) sort_keys_regs<1>(ent, n_c, lane);
        else if (N == 64) sort_keys_regs<2>(ent, n_c, lane);
        else if (N == 128) sort_keys_regs<4>(ent, n_c, lane);
        else sort_keys_regs<8>(ent, n_c, lane);
    } else {
        for (int i = n_c + lane; i < N; i += 32) ent[i] = 0ull;
        __syncwarp();
        bitonic_smem_desc(ent, N, lane);
    }

    // ---- 9. top-k / top-p / min-p / draw (src/zonos2_generate.cpp:55-92)
    // The list is ent[0..m) (positive probabilities, sorted) followed by a
    // tail of zero-probability tokens in token order, n entries in all.
    const int n_list = topk_on ? K : V;
    const int m = min(n_pos, n_list);
    float *q = reinterpret_cast<float *>(region + kQOffset);
    const bool use_q = N <= kQCap;
    if (topk_on && lane == 0) S = seq_sum(ent, m);
    S = __shfl_sync(kFull, S, 0);
    int n = n_list;

    if (a.top_p < 1.0f) {
        if (use_q) {
            for (int i = lane; i < m; i += 32) q[i] = key_p(ent[i]) / S;
            __syncwarp();
        }
        int cut = -1;
        if (lane == 0) {
            float cum = 0.0f;
            for (int i = 0; i < m; i++) {
                cum += use_q ? q[i] : key_p(ent[i]) / S;
                if (cum >= a.top_p) {
                    cut = i + 1;
                    break;
                }
            }
        }
        cut = __shfl_sync(kFull, cut, 0);
        if (cut > 0) n = cut;  // never reached inside the zero tail: cum stops growing
        if (lane == 0) S = seq_sum(ent, min(n, m));
        S = __shfl_sync(kFull, S, 0);
        __syncwarp();
    }

    if (a.min_p > 0.0f && n > 0) {
        const float thresh = (key_p(ent[0]) / S) * a.min_p;
        const int mm = min(n, m);
        int j = mm;
        for (int base = 0; base < mm; base += 32) {
            const int i = base + lane;
            const bool fail = i < mm && !(key_p(ent[i]) / S >= thresh);
            const uint32_t b = __ballot_sync(kFull, fail);
            if (b) {
                j = base + __ffs(b) - 1;
                break;
            }
        }
        if (j == mm && n > mm) j = (0.0f >= thresh) ? n : mm;
        n = j;
        if (lane == 0) S = seq_sum(ent, min(n, m));
        S = __shfl_sync(kFull, S, 0);
    }

    const float r = uni[cb];
    const int m3 = min(n, m);
    if (use_q) {
        for (int i = lane; i < m3; i += 32) q[i] = key_p(ent[i]) / S;
        __syncwarp();
    }
    int pos = -1;
    if (lane == 0) {
        float cum = 0.0f;
        for (int i = 0; i < m3; i++) {
            cum += use_q ? q[i] : key_p(ent[i]) / S;
            if (r <= cum) {
                pos = i;
                break;
            }
        }
    }
    pos = __shfl_sync(kFull, pos, 0);

    int tok;
    if (pos >= 0) {
        tok = key_tok(ent[pos]);
    } else if (n > m3) {
        // fell through to the last list entry, a zero-probability token: the
        // (n-1-m3)-th token, in token order, outside the positive set
        posmap[lane] = 0u;
        __syncwarp();
        for (int i = lane; i < n_pos; i += 32) {
            const int t = key_tok(ent[i]);
            atomicOr(posmap + (t >> 5), 1u << (t & 31));
        }
        __syncwarp();
        const int lo = lane * 32;
        const uint32_t valid = lo >= V ? 0u : (V - lo >= 32 ? ~0u : ((1u << (V - lo)) - 1u));
        const uint32_t zw = ~posmap[lane] & valid;
        const int zc = __popc(zw);
        const int incl = warp_incl_scan(zc, lane);
        const int want = n - 1 - m3;
        const int fl = __ffs(__ballot_sync(kFull, incl > want)) - 1;
        int t = -1;
        if (lane == fl) {
            int kth = want - (incl - zc);
            for (int b = 0; b < 32; b++)
                if ((zw >> b) & 1u) {
                    if (kth == 0) {
                        t = lo + b;
                        break;
                    }
                    kth--;
                }
        }
        tok = __shfl_sync(kFull, t, fl);
    } else {
        tok = n > 0 ? key_tok(ent[n - 1]) : a.pad_id;  // n >= 1 whenever min_p <= 1
    }
    if (lane == 0) finish_row(a, row, tok, flag);
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
