// head_tc.cu -- bf16 output head + softcap on the tcgen05 tensor cores (sm_100a).
//
// Restates the multi_output head of the reference -- linear_forward
// (src/zonos2_model.cpp:200-216, :687-690) followed by l = 15*tanh(l/15)
// (:692-703) -- for the sampled rows of each codebook, as one GEMM
//     logits[b, c*V + v] = softcap(sum_k hidden[b, k] * W[c*rpc + v, k])
// with bf16 operands and f32 accumulation.
//
// Persistent kernel, one CTA per SM, three warp roles:
//   warp 0      TMA producer: 128 x 64 tiles of hidden (A) and BN x 64 tiles of
//               W (B), 128-byte swizzled, into a ring of shared-memory stages;
//   warp 1      allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16) from
//               one elected lane, accumulating a 128 x BN f32 tile in TMEM;
//               two accumulators alternate so the epilogue of one tile
//               overlaps the MMAs of the next;
//   warps 2..9  epilogue: tcgen05.ld of their 32 TMEM lanes (two warps per lane
//               quarter, each half of the columns), softcap, then each 32 x 32
//               f32 chunk staged in the warp's 4 KB of shared memory and
//               stored by a tensor copy (whole 128-byte row pieces).
// Stages hand over through mbarriers: TMA completes `full`, tcgen05.commit
// releases `empty` and signals `tfull`, the epilogue releases `tempty`.
// Every wait is bounded: after ~2 s it records an error in g_device_error and
// the kernel winds down (in-flight copies waited for, TMEM freed).
// No TMA load here uses cluster multicast.
#include <cuda.h>
#include <math.h>
#include <stdio.h>

#include <mutex>

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

namespace {

constexpr int kBM = 128;            // rows of hidden per tile (TMEM lanes)
constexpr int kBK = 64;             // bf16 elements per 128-byte swizzled row
constexpr int kThreads = 320;       // 10 warps: producer, MMA, 8 epilogue
constexpr int kEpiThreads = 256;
constexpr unsigned long long kWaitNs = 2000000000ull;

enum : int { kErrTimeout = 1 };

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

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

// Waits for the phase with this parity to complete; false after ~2 s (the
// error word is set, the caller winds down).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0u && globaltimer_ns() - t0 > kWaitNs) {
            atomicCAS(&g_device_error, 0, kErrTimeout);
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                            uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// One tile of shared memory -> global through the tensor map (rows past the
// tensor's end are not written); completes in this thread's bulk group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap *map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row groups of
// 128-byte rows, 1024 bytes apart (SBO); version 1 (sm_100); base offset 0
// (stages are 1024-byte aligned).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr)
{
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// cap * tanh(l / cap) as cap - 2 cap / (2^(l k2) + 1), k2 = 2 log2(e) / cap, with
// the hardware exp2 and reciprocal approximations (relative errors of about
// 2^-22 and 2^-23): the reciprocal r <= 1 is off by about 2^-21 relative, so
// the result is within 2 cap 2^-21 (1.5e-5 for cap = 15) of the exact softcap,
// far inside the bf16 path's tolerance; it saturates to +-cap.
__device__ __forceinline__ float softcap_fast(float l, float cap, float k2)
{
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(l * k2));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(e + 1.0f));
    return __fmaf_rn(-2.0f * cap, r, cap);
}

struct TcArgs {
    int batch, n_cb, vocab, rows_per_cb, dim;
    int tiles_m, tiles_n, n_tiles;
    float softcap;
    float *out;  // [batch][n_cb * vocab], or [batch / 2][..] with cfg
    int cfg;     // rows 2s, 2s+1 (conditional, unconditional) blend into out row s
    float cfg_scale;
    int out_rows;   // rows of out: batch, or batch / 2 with cfg
    const float *row_scale;   // [batch] factor per hidden row before the softcap, or nullptr
};

// The factor of hidden row `row` (1 when there is none or the row is past the batch).
__device__ __forceinline__ float row_factor(const TcArgs &args, int row)
{
    return args.row_scale && row < args.batch ? __ldg(args.row_scale + row) : 1.0f;
}

// The epilogue's 32 output values of one 32-column chunk of this lane's row
// (rows 2s and 2s+1 sit in neighbouring lanes of one warp): the softcap, and
// with classifier-free guidance the blend u + s * (c - u) of the pair, taken
// from the neighbouring lane; the even lane's values are output row s
// (src/zonos2_generate.cpp:178-183).  Every lane takes part.
__device__ __forceinline__ void finish_chunk(const TcArgs &args, const uint32_t (&r)[32], float k2,
                                             float rsc, float (&o)[32])
{
    const float cap = args.softcap;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        const float l = args.row_scale ? __uint_as_float(r[i]) * rsc : __uint_as_float(r[i]);
        o[i] = cap > 0.0f ? softcap_fast(l, cap, k2) : l;
        if (args.cfg) {
            const float u = __shfl_xor_sync(kFull, o[i], 1);
            o[i] = __fadd_rn(u, __fmul_rn(args.cfg_scale, __fsub_rn(o[i], u)));
        }
    }
}

template <int BN, int STAGES, int KSUB>
__global__ void __launch_bounds__(kThreads, 1)
    head_tc_kernel(const __grid_constant__ CUtensorMap map_a,
                   const __grid_constant__ CUtensorMap map_b,
                   const __grid_constant__ CUtensorMap map_o, const TcArgs args)
{
    constexpr uint32_t kABytes = kBM * kBK * 2;
    constexpr uint32_t kBBytes = BN * kBK * 2;
    constexpr uint32_t kSubBytes = kABytes + kBBytes;   // one 64-deep K slice of A and B
    constexpr uint32_t kStageBytes = KSUB * kSubBytes;    // KSUB slices per stage
    constexpr uint32_t kTmemCols = 2 * BN;
    // tcgen05 kind::f16 instruction descriptor: D f32, A and B bf16, both
    // K-major, N = BN, M = 128.
    constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                ((uint32_t)(kBM >> 4) << 24);

    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    // stages, then 4 KB of output staging per epilogue warp, then the barriers
    uint64_t *bars =
        reinterpret_cast<uint64_t *>(smem + STAGES * kStageBytes + (kEpiThreads / 32) * 4096);
    // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2]; then the TMEM slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
    __shared__ int s_abort;

    // the next kernel (the sampler) may be scheduled as SMs free up; it waits for
    // this grid before it reads anything
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = args.dim / (kBK * KSUB);
    auto full = [&](int s) { return smem_u32(bars + s); };
    auto empty = [&](int s) { return smem_u32(bars + STAGES + s); };
    auto tfull = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
    auto tempty = [&](int a) { return smem_u32(bars + 2 * STAGES + 2 + a); };

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), kEpiThreads);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        prefetch_map(&map_a);
        prefetch_map(&map_b);
        prefetch_map(&map_o);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched under programmatic dependent launch: the set-up above overlaps the
    // kernel before this one; nothing global is read or written before it ends.
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == 0) {
        // ---- TMA producer
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < args.n_tiles && ok; tile += gridDim.x) {
                const int mt = tile % args.tiles_m, nt = tile / args.tiles_m;
                const int per_cb = args.vocab / BN;
                const int c = nt / per_cb, t = nt % per_cb;
                const int a_row = mt * kBM;
                const int b_row = c * args.rows_per_cb + t * BN;
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(empty(s), ph ^ 1u) || *(volatile int *)&s_abort) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = smem_u32(smem + s * kStageBytes);
                    mbar_expect_tx(full(s), kStageBytes);
#pragma unroll
                    for (int j = 0; j < KSUB; j++) {
                        const int kx = (kb * KSUB + j) * kBK;
                        tma_load_2d(sa + j * kSubBytes, &map_a, kx, a_row, full(s));
                        tma_load_2d(sa + j * kSubBytes + kABytes, &map_b, kx, b_row, full(s));
                    }
                }
            }
            if (!ok) {
                s_abort = 1;
                // copies still in flight land before the CTA leaves
                for (int k = 0; k < STAGES && k < it; k++) {
                    const int j = it - 1 - k;
                    mbar_wait(full(j % STAGES), (uint32_t)(j / STAGES) & 1u);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            int it = 0, local = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < args.n_tiles && ok; tile += gridDim.x, local++) {
                const int acc = local & 1;
                const uint32_t aph = (uint32_t)(local >> 1) & 1u;
                if (!mbar_wait(tempty(acc), aph ^ 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(full(s), ph) || *(volatile int *)&s_abort) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * kStageBytes);
#pragma unroll
                    for (int j = 0; j < KSUB; j++) {
                        const uint64_t ad = sw128_desc(sa + j * kSubBytes);
                        const uint64_t bd = sw128_desc(sa + j * kSubBytes + kABytes);
#pragma unroll
                        for (int k = 0; k < kBK / 16; k++)   // 32 bytes of K per instruction
                            mma_bf16(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), kIdesc,
                                     (kb | j | k) != 0);
                    }
                    mma_commit(empty(s));
                }
                if (ok) mma_commit(tfull(acc));
            }
            if (!ok) s_abort = 1;
        }
    } else {
        // ---- epilogue: TMEM -> softcap -> global, through the warp's staging
        // buffer and tensor stores as in the two-SM kernel below
        const int q = warp & 3;   // the TMEM lane quarter this warp may read
        const int half = (warp - 2) >> 2;   // which half of the tile's columns
        const uint32_t stage_o = smem_u32(smem + STAGES * kStageBytes + (warp - 2) * 4096);
        const int orow = args.cfg ? lane >> 1 : lane;
        const bool owner = !args.cfg || (lane & 1) == 0;
        int local = 0;
        for (int tile = blockIdx.x; tile < args.n_tiles; tile += gridDim.x, local++) {
            const int acc = local & 1;
            const uint32_t aph = (uint32_t)(local >> 1) & 1u;
            if (!mbar_wait(tfull(acc), aph)) {
                s_abort = 1;
                break;
            }
            if (*(volatile int *)&s_abort) break;
            tc_fence_after();
            const int mt = tile % args.tiles_m, nt = tile / args.tiles_m;
            const int row0 = mt * kBM + 32 * q;
            const int y0 = args.cfg ? row0 >> 1 : row0;
            const float rsc = row_factor(args, row0 + lane);   // this lane's hidden row
            const float k2 = 2.0f * 1.4426950408889634f / args.softcap;   // 2 log2(e) / cap
#pragma unroll 1
            for (int ch = half * (BN / 64); ch < (half + 1) * (BN / 64); ch++) {
                uint32_t r[32];
                tmem_ld32(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN + 32 * ch), r);
                float o[32];
                finish_chunk(args, r, k2, rsc, o);
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();
                if (owner) {
#pragma unroll
                    for (int c = 0; c < 8; c++)
                        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(
                                         stage_o + orow * 128 + ((c ^ (orow & 7)) << 4)),
                                     "f"(o[4 * c]), "f"(o[4 * c + 1]), "f"(o[4 * c + 2]),
                                     "f"(o[4 * c + 3])
                                     : "memory");
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0 && y0 < args.out_rows)
                    tma_store_2d(&map_o, stage_o, nt * BN + 32 * ch, y0);
            }
            tc_fence_before();
            mbar_arrive(tempty(acc));
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols)
                     : "memory");
}

// ---- two-SM pairs (cluster of 2, tcgen05 cta_group::2) ----------------------
__device__ __forceinline__ uint32_t cluster_rank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of this CTA's shared variable `addr` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// mbar_wait with cluster-scope acquire: for barriers that the other CTA of the
// pair arrives on.
__device__ __forceinline__ bool mbar_try_wait_cl(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity)
{
    if (mbar_try_wait_cl(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; it++) {
        if (mbar_try_wait_cl(bar, parity)) return true;
        if ((it & 255u) == 0u && globaltimer_ns() - t0 > kWaitNs) {
            atomicCAS(&g_device_error, 0, kErrTimeout);
            return false;
        }
    }
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// TMA load into this CTA's shared memory, completing on the mbarrier at cluster
// address `bar` (in either CTA of the pair).  Not a multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int x, int y,
                                                 uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on the mbarrier at cluster address `bar` once the pair's MMAs issued
// so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// Persistent two-SM version for large batches: the two CTAs of a cluster
// compute a 256 x 256 tile with tcgen05.mma.cta_group::2 (M=256, N=256,
// K=16), each holding half of the A rows and half of the B rows in its own
// shared memory and half of the accumulator rows in its own TMEM.  Per SM and
// 64-deep K step that is 32 KB of operands instead of 48 KB for the same MMA
// work, which is what limits the one-SM kernel (its operands come from L2).
//   warp 0 (both CTAs)   TMA producer of the CTA's halves; both CTAs' copies
//                        complete on rank 0's `full`, which expects both;
//   warp 1, rank 0       issues the pair's MMAs; its commits release `empty`
//                        and signal `tfull` in both CTAs;
//   warps 2..5 (both)    epilogue of the CTA's 128 accumulator rows, then one
//                        arrive per warp on rank 0's `tempty` (8 arrivals).
// No load is multicast: every copy lands in the CTA that issued it.  A CTA that
// gives up waits at the final cluster barrier, so its shared memory outlives
// any copy of its own still in flight while rank 0 drains `full`.
template <int BN, int STAGES, int KSUB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    head_tc2_kernel(const __grid_constant__ CUtensorMap map_a,
                    const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_o, const TcArgs args)
{
    // BN: N of the pair's tile (256 or 128); each CTA holds BN / 2 of its B rows
    constexpr uint32_t kABytes = kBM * kBK * 2;
    constexpr uint32_t kBBytes = (BN / 2) * kBK * 2;
    constexpr uint32_t kSubBytes = kABytes + kBBytes;   // one 64-deep K slice of A and B
    constexpr uint32_t kStageBytes = KSUB * kSubBytes;    // KSUB slices per stage
    constexpr uint32_t kTmemCols = 2 * BN;
    constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                ((uint32_t)((2 * kBM) >> 4) << 24);

    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    // stages, then 4 KB of output staging per epilogue warp, then the barriers
    uint64_t *bars =
        reinterpret_cast<uint64_t *>(smem + STAGES * kStageBytes + (kEpiThreads / 32) * 4096);
    // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2]; the TMEM slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
    __shared__ int s_abort;

    // the next kernel (the sampler) may be scheduled as SMs free up; it waits for
    // this grid before it reads anything
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int KB = args.dim / (kBK * KSUB);
    auto full = [&](int s) { return smem_u32(bars + s); };
    auto empty = [&](int s) { return smem_u32(bars + STAGES + s); };
    auto tfull = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
    auto tempty = [&](int a) { return smem_u32(bars + 2 * STAGES + 2 + a); };

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 2 * kEpiThreads / 32);   // one per epilogue warp, both CTAs
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        prefetch_map(&map_a);
        prefetch_map(&map_b);
        prefetch_map(&map_o);
    }
    if (warp == 1) {   // both CTAs, same warp: one allocation across the pair
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();    // barriers of both CTAs initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Launched under programmatic dependent launch: the set-up above overlaps the
    // kernel before this one; nothing global is read or written before it ends.
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int tiles_m2 = (args.tiles_m + 1) >> 1;   // 256-row blocks
    const int per_cb = args.vocab / BN;
    const int n_tiles = tiles_m2 * args.n_cb * per_cb;

    if (warp == 0) {
        // ---- TMA producer (this CTA's halves)
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int tile = pair; tile < n_tiles && ok; tile += n_pairs) {
                const int mt = tile % tiles_m2, nt = tile / tiles_m2;
                const int c = nt / per_cb, t = nt % per_cb;
                const int a_row = mt * 2 * kBM + (int)rank * kBM;
                const int b_row = c * args.rows_per_cb + t * BN + (int)rank * (BN / 2);
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait(empty(s), ph ^ 1u) || *(volatile int *)&s_abort) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = smem_u32(smem + s * kStageBytes);
                    if (rank == 0) mbar_expect_tx(full(s), 2 * kStageBytes);   // both halves
                    const uint32_t fb = peer_addr(full(s), 0);   // rank 0's, as a cluster address
#pragma unroll
                    for (int j = 0; j < KSUB; j++) {
                        const int kx = (kb * KSUB + j) * kBK;
                        tma_load_2d_pair(sa + j * kSubBytes, &map_a, kx, a_row, fb);
                        tma_load_2d_pair(sa + j * kSubBytes + kABytes, &map_b, kx, b_row, fb);
                    }
                }
            }
            if (!ok) {
                s_abort = 1;
                if (rank == 0)   // the pair's copies still in flight land first
                    for (int k = 0; k < STAGES && k < it; k++) {
                        const int j = it - 1 - k;
                        mbar_wait(full(j % STAGES), (uint32_t)(j / STAGES) & 1u);
                    }
            }
        }
    } else if (warp == 1 && rank == 0) {
        // ---- MMA issuer (rank 0) for the pair
        if (lane == 0) {
            int it = 0, local = 0;
            bool ok = true;
            for (int tile = pair; tile < n_tiles && ok; tile += n_pairs, local++) {
                const int acc = local & 1;
                const uint32_t aph = (uint32_t)(local >> 1) & 1u;
                if (!mbar_wait_cl(tempty(acc), aph ^ 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < KB; kb++, it++) {
                    const int s = it % STAGES;
                    const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
                    if (!mbar_wait_cl(full(s), ph) || *(volatile int *)&s_abort) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * kStageBytes);
#pragma unroll
                    for (int j = 0; j < KSUB; j++) {
                        const uint64_t ad = sw128_desc(sa + j * kSubBytes);
                        const uint64_t bd = sw128_desc(sa + j * kSubBytes + kABytes);
#pragma unroll
                        for (int k = 0; k < kBK / 16; k++)
                            mma_bf16_pair(d_tmem, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k),
                                          kIdesc, (kb | j | k) != 0);
                    }
                    mma_commit_pair(empty(s));
                    mma_commit_pair(peer_addr(empty(s), 1));
                }
                if (ok) {
                    mma_commit_pair(tfull(acc));
                    mma_commit_pair(peer_addr(tfull(acc), 1));
                }
            }
            if (!ok) s_abort = 1;
        }
    } else if (warp >= 2) {
        // ---- epilogue: this CTA's 128 accumulator rows -> softcap -> global.  Each
        // warp stages a 32 x 32 chunk in its own 4 KB of shared memory (128-byte
        // swizzle: 16-byte piece c of row r at r * 128 + (c ^ (r & 7)) * 16) and
        // one lane stores it with a tensor copy, whole 128-byte row pieces at a
        // time, while the warp goes on to the next chunk.
        const int q = warp & 3;             // the TMEM lane quarter this warp may read
        const int half = (warp - 2) >> 2;   // which half of the tile's columns
        const uint32_t tempty0 = peer_addr(tempty(0), 0), tempty1 = peer_addr(tempty(1), 0);
        const uint32_t stage_o = smem_u32(smem + STAGES * kStageBytes + (warp - 2) * 4096);
        const int orow = args.cfg ? lane >> 1 : lane;   // this lane's row in the chunk
        const bool owner = !args.cfg || (lane & 1) == 0;
        int local = 0;
        for (int tile = pair; tile < n_tiles; tile += n_pairs, local++) {
            const int acc = local & 1;
            const uint32_t aph = (uint32_t)(local >> 1) & 1u;
            if (!mbar_wait(tfull(acc), aph)) {
                s_abort = 1;
                break;
            }
            if (*(volatile int *)&s_abort) break;
            tc_fence_after();
            const int mt = tile % tiles_m2, nt = tile / tiles_m2;
            const int row0 = mt * 2 * kBM + (int)rank * kBM + 32 * q;   // the warp's first row
            const int y0 = args.cfg ? row0 >> 1 : row0;                  // its first output row
            const float rsc = row_factor(args, row0 + lane);            // this lane's hidden row
            const float k2 = 2.0f * 1.4426950408889634f / args.softcap;   // 2 log2(e) / cap
#pragma unroll 1
            for (int ch = half * (BN / 64); ch < (half + 1) * (BN / 64); ch++) {
                uint32_t r[32];
                tmem_ld32(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN + 32 * ch), r);
                float o[32];
                finish_chunk(args, r, k2, rsc, o);
                if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                __syncwarp();   // the previous chunk has left the staging buffer
                if (owner) {
#pragma unroll
                    for (int c = 0; c < 8; c++)
                        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(
                                         stage_o + orow * 128 + ((c ^ (orow & 7)) << 4)),
                                     "f"(o[4 * c]), "f"(o[4 * c + 1]), "f"(o[4 * c + 2]),
                                     "f"(o[4 * c + 3])
                                     : "memory");
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0 && y0 < args.out_rows)
                    tma_store_2d(&map_o, stage_o, nt * BN + 32 * ch, y0);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc ? tempty1 : tempty0);
        }
        if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();    // the pair is done with both CTAs' TMEM and barriers
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(kTmemCols)
                     : "memory");
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D bf16 tensor map over rows x cols (cols contiguous), box box_cols x box_rows.
bool make_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// 2-D f32 tensor map over rows x cols (cols contiguous), box 32 cols x box_rows,
// 128-byte swizzle (the epilogue's staging layout).
bool make_map_f32(CUtensorMap *m, void *base, uint64_t rows, uint64_t cols, uint32_t box_rows)
{
    EncodeTiledFn enc = encode_fn();
    if (!enc || rows == 0) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {32, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// Launches a head kernel under programmatic dependent launch (its set-up overlaps
// the previous kernel's tail; it waits for that grid before any global access).
template <class Kernel>
cudaError_t launch_pdl(Kernel kernel, int grid, size_t smem, cudaStream_t stream,
                       const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mo,
                       const TcArgs &t)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, ma, mb, mo, t);
}

template <int BN, int STAGES, int KSUB>
cudaError_t launch_pair(const HeadArgs &a, const CUtensorMap &ma, int tiles_m, int sms,
                        cudaStream_t stream)
{
    static std::mutex mu;
    static int pairs_cap[64] = {0};   // clusters of two that fit at once; 0 until queried
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    // stages, 4 KB of output staging per epilogue warp, barriers, alignment
    const size_t smem =
        (size_t)STAGES * KSUB * (kBM + BN / 2) * kBK * 2 + (kEpiThreads / 32) * 4096 + 1024 + 512;
    int pairs = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (pairs_cap[dev] == 0) {
            e = cudaFuncSetAttribute(head_tc2_kernel<BN, STAGES, KSUB>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(2 * (sms / 2));
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = smem;
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, head_tc2_kernel<BN, STAGES, KSUB>, &cfg);
            if (e != cudaSuccess) return e;
            pairs_cap[dev] = n > 0 ? n : 1;
        }
        pairs = pairs_cap[dev];
    }
    CUtensorMap mb;   // each CTA of a pair loads half of the tile's BN weight rows
    if (!make_map(&mb, a.W, (uint64_t)a.n_cb * a.rows_per_cb, (uint64_t)a.dim, BN / 2))
        return cudaErrorInvalidValue;
    TcArgs t;
    t.batch = a.batch;
    t.n_cb = a.n_cb;
    t.vocab = a.vocab;
    t.rows_per_cb = a.rows_per_cb;
    t.dim = a.dim;
    t.tiles_m = tiles_m;
    t.tiles_n = a.n_cb * (a.vocab / BN);
    t.n_tiles = ((tiles_m + 1) / 2) * t.tiles_n;
    t.softcap = a.softcap;
    t.out = a.out;
    t.cfg = a.cfg;
    t.cfg_scale = a.cfg_scale;
    t.out_rows = a.cfg ? a.batch / 2 : a.batch;
    t.row_scale = a.row_scale;
    CUtensorMap mo;   // the logits, f32, 32 x 32 chunks (16 output rows with guidance)
    if (!make_map_f32(&mo, a.out, (uint64_t)t.out_rows, (uint64_t)a.n_cb * a.vocab,
                      a.cfg ? 16 : 32))
        return cudaErrorInvalidValue;
    const int grid = 2 * (t.n_tiles < pairs ? t.n_tiles : pairs);
    return launch_pdl(head_tc2_kernel<BN, STAGES, KSUB>, grid, smem, stream, ma, mb, mo, t);
}

template <int BN, int STAGES, int KSUB>
cudaError_t launch_bn(const HeadArgs &a, const CUtensorMap &ma, int tiles_m, int sms,
                      cudaStream_t stream)
{
    static std::mutex mu;
    static bool attr[64] = {false};   // the shared-memory size has been set on the device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    // stages, 4 KB of output staging per epilogue warp, barriers, alignment
    const size_t smem =
        (size_t)STAGES * KSUB * (kBM + BN) * kBK * 2 + (kEpiThreads / 32) * 4096 + 1024 + 512;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!attr[dev]) {
            e = cudaFuncSetAttribute(head_tc_kernel<BN, STAGES, KSUB>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            attr[dev] = true;
        }
    }
    CUtensorMap mb;
    if (!make_map(&mb, a.W, (uint64_t)a.n_cb * a.rows_per_cb, (uint64_t)a.dim, BN))
        return cudaErrorInvalidValue;
    TcArgs t;
    t.batch = a.batch;
    t.n_cb = a.n_cb;
    t.vocab = a.vocab;
    t.rows_per_cb = a.rows_per_cb;
    t.dim = a.dim;
    t.tiles_m = tiles_m;
    t.tiles_n = a.n_cb * (a.vocab / BN);
    t.n_tiles = t.tiles_m * t.tiles_n;
    t.softcap = a.softcap;
    t.out = a.out;
    t.cfg = a.cfg;
    t.cfg_scale = a.cfg_scale;
    t.out_rows = a.cfg ? a.batch / 2 : a.batch;
    t.row_scale = a.row_scale;
    CUtensorMap mo;
    if (!make_map_f32(&mo, a.out, (uint64_t)t.out_rows, (uint64_t)a.n_cb * a.vocab,
                      a.cfg ? 16 : 32))
        return cudaErrorInvalidValue;
    const int grid = t.n_tiles < sms ? t.n_tiles : sms;
    return launch_pdl(head_tc_kernel<BN, STAGES, KSUB>, grid, smem, stream, ma, mb, mo, t);
}

}  // namespace

cudaError_t launch_head_tc_bf16(const HeadArgs &a, cudaStream_t stream)
{
    if (a.batch == 0) return cudaSuccess;
    if (a.dim % kBK != 0 || a.vocab % 64 != 0 || a.rows_per_cb < a.vocab)
        return cudaErrorNotSupported;
    if ((uintptr_t)a.W % 16 != 0 || (uintptr_t)a.hidden % 16 != 0 || (uintptr_t)a.out % 16 != 0)
        return cudaErrorNotSupported;
    int dev = 0, sms = 148;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    CUtensorMap ma;
    if (!make_map(&ma, a.hidden, (uint64_t)a.batch, (uint64_t)a.dim, kBM))
        return cudaErrorInvalidValue;
    const int tiles_m = (a.batch + kBM - 1) / kBM;
    // Tile choice.  Two-SM pairs (stages of two 64-deep K slices: the same bytes in
    // flight as six one-slice stages, half the hand-overs) once half the pairs get
    // a 256 x 256 tile; a pair moves 128 + 128 operand rows per SM per tile.
    // Below that the one-SM kernel, its N tile by a model of operand traffic: a
    // tile rereads its A rows once per N tile and its B rows once per M tile, so a
    // wave costs about (128 + BN) rows per SM and the launch ceil(tiles / SMs)
    // waves; ties go to the wider tile.  Measured on a B200 (ms, 9 x 1024 x 2048;
    // pairs with two slices per stage, the one-SM kernel with BN 256 with one,
    // 128 and 64 with two):
    //   rows   pairs   BN 256  BN 128  BN 64
    //    128     -     0.0185  0.0184  0.0121
    //    256     -     0.0204  0.0133  0.0282
    //    384   0.0186  0.0189    -       -
    //    512   0.0185  0.0188    -       -
    //    768   0.0308  0.0337    -       -
    //   1024   0.0321  0.0354    -       -
    //   1536   0.0466  0.0515    -       -
    //   4096   0.115   0.1305    -       -
    // Pairs with 128-wide tiles (128 + 64 rows per SM) measured slower: 0.0217 ms at
    // 256 rows, 0.0354 at 512, 0.0592 at 1024 (one slice per stage); 0.0151 at 256
    // and 0.0147 at 130 with two slices per stage, three stages or four.
    const int cols = a.n_cb * a.vocab;
    if (a.vocab % 256 == 0 && a.dim % (2 * kBK) == 0 &&
        ((tiles_m + 1) / 2) * (cols / 256) >= sms / 4)
        return launch_pair<256, 3, 2>(a, ma, tiles_m, sms, stream);
    auto waves = [&](long long tiles, int slots) { return (tiles + slots - 1) / slots; };
    long long best = -1;
    int pick = 64;
    const int bns[3] = {256, 128, 64};
    for (int bn : bns) {
        if (a.vocab % bn != 0) continue;
        const long long c = waves((long long)tiles_m * (cols / bn), sms) * (kBM + bn);
        if (best < 0 || c < best) {
            best = c;
            pick = bn;
        }
    }
    // Stages of two 64-deep K slices where three or more such stages fit (BN 128
    // and 64: 0.013 against 0.017 ms at 256 rows, 0.012 against 0.016 at 128);
    // with BN 256 they would leave two stages, and four of one slice measure
    // faster (0.019 against 0.021 ms at 512 rows).
    const bool two = a.dim % (2 * kBK) == 0;
    if (pick == 256) return launch_bn<256, 4, 1>(a, ma, tiles_m, sms, stream);
    if (pick == 128)
        return two ? launch_bn<128, 3, 2>(a, ma, tiles_m, sms, stream)
                   : launch_bn<128, 6, 1>(a, ma, tiles_m, sms, stream);
    return two ? launch_bn<64, 4, 2>(a, ma, tiles_m, sms, stream)
               : launch_bn<64, 8, 1>(a, ma, tiles_m, sms, stream);
}

}  // namespace z2
