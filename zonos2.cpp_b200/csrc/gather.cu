// gather.cu -- several GPUs: the batch-sharded decode job's codes collected on
// one rank over NCCL.
//
// Decode streams are independent, so a job shards its global batch into
// contiguous slices, one per rank (zonos2cu_shard_range), each rank's context
// created with first_stream = its slice's start.  The only data that crosses
// GPUs is the int32 codes, which the writer rank collects: the role of the
// frame collection at src/zonos2_generate.cpp:278, for a batch.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, reusing a copy the
// process already holds, e.g. PyTorch's), so the library loads and runs its
// one-GPU entry points on hosts without NCCL.  The gather is grouped
// point-to-point: every other rank sends its block to the root, the root
// receives them all in one group and copies its own block on the stream.
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <set>
#include <thread>

#include "zonos2_cuda.h"

const char *z2_set_error(const char *fmt, const char *a, const char *b);

namespace {

struct NcclApi {
    bool tried = false;
    bool ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommCount)(const ncclComm_t, int *) = nullptr;
    ncclResult_t (*CommUserRank)(const ncclComm_t, int *) = nullptr;
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t,
                         cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
    // Non-blocking set-up and tear-down (NCCL >= 2.14); the bounded calls need them.
    bool nb_ok = false;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int,
                                       ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
};
std::mutex g_nccl_mu;
NcclApi g_nccl;

template <class F>
bool sym(void *h, const char *name, F *out)
{
    *out = reinterpret_cast<F>(dlsym(h, name));
    return *out != nullptr;
}

// The NCCL entry points, loaded once; null if libnccl.so.2 cannot be found.
const NcclApi *nccl()
{
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.tried) return g_nccl.ok ? &g_nccl : nullptr;
    g_nccl.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        z2_set_error("%s: %s", "dlopen libnccl.so.2", dlerror());
        return nullptr;
    }
    NcclApi &a = g_nccl;
    a.ok = sym(h, "ncclGetUniqueId", &a.GetUniqueId) && sym(h, "ncclCommInitRank", &a.CommInitRank) &&
           sym(h, "ncclCommDestroy", &a.CommDestroy) && sym(h, "ncclCommCount", &a.CommCount) &&
           sym(h, "ncclCommUserRank", &a.CommUserRank) && sym(h, "ncclSend", &a.Send) &&
           sym(h, "ncclRecv", &a.Recv) && sym(h, "ncclGroupStart", &a.GroupStart) &&
           sym(h, "ncclGroupEnd", &a.GroupEnd) && sym(h, "ncclGetErrorString", &a.GetErrorString);
    if (!a.ok) z2_set_error("%s: %s", "libnccl.so.2", "an entry point is missing");
    a.nb_ok = sym(h, "ncclCommInitRankConfig", &a.CommInitRankConfig) &&
              sym(h, "ncclCommGetAsyncError", &a.CommGetAsyncError) &&
              sym(h, "ncclCommAbort", &a.CommAbort) && sym(h, "ncclCommFinalize", &a.CommFinalize);
    return a.ok ? &a : nullptr;
}

int nccl_fail(const NcclApi *a, ncclResult_t r, const char *what)
{
    z2_set_error("%s: %s", what, a->GetErrorString(r));
    return ZONOS2CU_ENCCL;
}

#define Z2_NCCL(api, call)                                          \
    do {                                                            \
        const ncclResult_t r_ = (call);                             \
        if (r_ != ncclSuccess) return nccl_fail(api, r_, #call);    \
    } while (0)

struct DeviceScope {
    int prev = -1;
    explicit DeviceScope(int dev)
    {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceScope()
    {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Communicators made non-blocking by zonos2cu_comm_create_timeout: their groups
// and their tear-down complete in the background and are polled.
std::set<void *> g_nonblocking;

bool is_nonblocking(void *c)
{
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    return g_nonblocking.count(c) != 0;
}

void forget_comm(void *c)
{
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    g_nonblocking.erase(c);
}

// Polls a non-blocking communicator until its pending operation (set-up, a
// group, finalisation) ends or timeout_ms passes.  Returns ncclSuccess, the
// error the operation ended with, or ncclInProgress when the time ran out.
ncclResult_t wait_async(const NcclApi *a, ncclComm_t c, int timeout_ms)
{
    using clk = std::chrono::steady_clock;
    const clk::time_point deadline = clk::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        ncclResult_t st = ncclInProgress;
        const ncclResult_t r = a->CommGetAsyncError(c, &st);
        if (r != ncclSuccess) return r;
        if (st != ncclInProgress) return st;
        if (clk::now() >= deadline) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// A non-blocking communicator's grouped sends and receives may still be
// connecting when ncclGroupEnd returns: how long the gather waits for them.
constexpr int kGroupTimeoutMs = 120000;
// ... and how long zonos2cu_comm_destroy waits for the flush before it aborts.
constexpr int kFinalizeTimeoutMs = 60000;

// The outcome of an enqueueing call (ncclSend, ncclGroupEnd): on a non-blocking
// communicator ncclInProgress means it is still connecting to its peers, and is
// polled up to kGroupTimeoutMs.
int settle(const NcclApi *a, ncclComm_t c, ncclResult_t r, const char *what)
{
    if (r == ncclInProgress && is_nonblocking(c)) r = wait_async(a, c, kGroupTimeoutMs);
    if (r == ncclInProgress) {
        z2_set_error("%s: %s", what, "not enqueued within the timeout");
        return ZONOS2CU_ENCCL;
    }
    return r == ncclSuccess ? ZONOS2CU_OK : nccl_fail(a, r, what);
}

}  // namespace

extern "C" {

int zonos2cu_shard_range(long long n_streams, int n_ranks, int rank, long long *first,
                         long long *count)
{
    if (n_streams < 0 || n_ranks < 1 || rank < 0 || rank >= n_ranks || !first || !count)
        return ZONOS2CU_EINVAL;
    const long long base = n_streams / n_ranks, extra = n_streams % n_ranks;
    *count = base + (rank < extra ? 1 : 0);
    *first = rank * base + (rank < extra ? rank : extra);
    return ZONOS2CU_OK;
}

int zonos2cu_comm_unique_id(unsigned char id[128])
{
    if (!id) return ZONOS2CU_EINVAL;
    const NcclApi *a = nccl();
    if (!a) return ZONOS2CU_ENCCL;
    ncclUniqueId u;
    Z2_NCCL(a, a->GetUniqueId(&u));
    static_assert(sizeof(u.internal) == 128, "NCCL unique id size");
    memcpy(id, u.internal, 128);
    return ZONOS2CU_OK;
}

int zonos2cu_comm_create(int device, int n_ranks, int rank, const unsigned char id[128],
                         void **comm_out)
{
    if (!id || !comm_out || n_ranks < 1 || rank < 0 || rank >= n_ranks) return ZONOS2CU_EINVAL;
    *comm_out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return ZONOS2CU_EINVAL;
    const NcclApi *a = nccl();
    if (!a) return ZONOS2CU_ENCCL;
    DeviceScope g(device);
    ncclUniqueId u;
    memcpy(u.internal, id, 128);
    ncclComm_t c = nullptr;
    Z2_NCCL(a, a->CommInitRank(&c, n_ranks, u, rank));
    *comm_out = c;
    return ZONOS2CU_OK;
}

int zonos2cu_comm_create_timeout(int device, int n_ranks, int rank, const unsigned char id[128],
                                 int timeout_ms, void **comm_out)
{
    if (!id || !comm_out || n_ranks < 1 || rank < 0 || rank >= n_ranks || timeout_ms < 1)
        return ZONOS2CU_EINVAL;
    *comm_out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return ZONOS2CU_EINVAL;
    const NcclApi *a = nccl();
    if (!a) return ZONOS2CU_ENCCL;
    if (!a->nb_ok) {
        z2_set_error("%s: %s", "libnccl.so.2", "no non-blocking communicator set-up");
        return ZONOS2CU_ENCCL;
    }
    DeviceScope g(device);
    ncclUniqueId u;
    memcpy(u.internal, id, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t c = nullptr;
    ncclResult_t r = a->CommInitRankConfig(&c, n_ranks, u, rank, &cfg);
    if ((r == ncclSuccess || r == ncclInProgress) && c) r = wait_async(a, c, timeout_ms);
    if (r != ncclSuccess) {
        if (c) a->CommAbort(c);   // also ends the set-up still waiting for its peers
        if (r == ncclInProgress) {
            z2_set_error("%s: %s", "ncclCommInitRankConfig",
                         "not every rank joined within the timeout; aborted");
            return ZONOS2CU_ENCCL;
        }
        return nccl_fail(a, r, "ncclCommInitRankConfig");
    }
    {
        std::lock_guard<std::mutex> lk(g_nccl_mu);
        g_nonblocking.insert(c);
    }
    *comm_out = c;
    return ZONOS2CU_OK;
}

int zonos2cu_comm_destroy(void *comm)
{
    if (!comm) return ZONOS2CU_OK;
    const NcclApi *a = nccl();
    if (!a) return ZONOS2CU_ENCCL;
    const ncclComm_t c = static_cast<ncclComm_t>(comm);
    if (is_nonblocking(comm)) {
        forget_comm(comm);
        ncclResult_t r = a->CommFinalize(c);
        if (r == ncclSuccess || r == ncclInProgress) r = wait_async(a, c, kFinalizeTimeoutMs);
        if (r != ncclSuccess) {
            a->CommAbort(c);
            if (r == ncclInProgress) {
                z2_set_error("%s: %s", "ncclCommFinalize", "did not flush within the timeout; aborted");
                return ZONOS2CU_ENCCL;
            }
            return nccl_fail(a, r, "ncclCommFinalize");
        }
    }
    Z2_NCCL(a, a->CommDestroy(c));
    return ZONOS2CU_OK;
}

int zonos2cu_comm_abort(void *comm)
{
    if (!comm) return ZONOS2CU_OK;
    const NcclApi *a = nccl();
    if (!a) return ZONOS2CU_ENCCL;
    if (!a->nb_ok) {
        z2_set_error("%s: %s", "libnccl.so.2", "ncclCommAbort is missing");
        return ZONOS2CU_ENCCL;
    }
    forget_comm(comm);
    Z2_NCCL(a, a->CommAbort(static_cast<ncclComm_t>(comm)));
    return ZONOS2CU_OK;
}

int zonos2cu_gather_codes(void *comm, int root, const int32_t *codes_dev, int n_steps,
                          long long n_streams, int n_cb, int32_t *out_dev, void *stream)
{
    if (!comm || n_steps < 0 || n_streams < 0 || n_cb < 1) return ZONOS2CU_EINVAL;
    const NcclApi *a = nccl();
    if (!a) return ZONOS2CU_ENCCL;
    const ncclComm_t c = static_cast<ncclComm_t>(comm);
    int n_ranks = 0, rank = 0;
    Z2_NCCL(a, a->CommCount(c, &n_ranks));
    Z2_NCCL(a, a->CommUserRank(c, &rank));
    if (root < 0 || root >= n_ranks) return ZONOS2CU_EINVAL;
    long long first = 0, count = 0;
    zonos2cu_shard_range(n_streams, n_ranks, rank, &first, &count);
    const size_t my_elems = (size_t)n_steps * (size_t)count * (size_t)n_cb;
    if (my_elems > 0 && !codes_dev) return ZONOS2CU_EINVAL;
    if (rank == root && n_steps > 0 && n_streams > 0 && !out_dev) return ZONOS2CU_EINVAL;
    if (n_steps == 0 || n_streams == 0) return ZONOS2CU_OK;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (rank != root) {
        if (!my_elems) return ZONOS2CU_OK;
        return settle(a, c, a->Send(codes_dev, my_elems, ncclInt32, root, c, st), "ncclSend");
    }
    // the root: every other rank's block in rank order, its own copied in place
    Z2_NCCL(a, a->GroupStart());
    for (int r = 0; r < n_ranks; r++) {
        long long f = 0, n = 0;
        zonos2cu_shard_range(n_streams, n_ranks, r, &f, &n);
        const size_t elems = (size_t)n_steps * (size_t)n * (size_t)n_cb;
        if (r == root || elems == 0) continue;
        const ncclResult_t res =
            a->Recv(out_dev + (size_t)n_steps * (size_t)f * (size_t)n_cb, elems, ncclInt32, r, c, st);
        if (res != ncclSuccess) {
            a->GroupEnd();
            return nccl_fail(a, res, "ncclRecv");
        }
    }
    if (const int rc = settle(a, c, a->GroupEnd(), "ncclGroupEnd")) return rc;
    int32_t *mine = out_dev + (size_t)n_steps * (size_t)first * (size_t)n_cb;
    if (my_elems && mine != codes_dev) {
        const cudaError_t e = cudaMemcpyAsync(mine, codes_dev, sizeof(int32_t) * my_elems,
                                              cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) {
            z2_set_error("%s: %s", "root block copy", cudaGetErrorString(e));
            (void)cudaGetLastError();   // reported here: not left for the next launch
            return ZONOS2CU_ECUDA;
        }
    }
    return ZONOS2CU_OK;
}


// ---- codes pushed to one rank by copy engines ----------------------------------
// The root's output lives in memory of its own (cudaMalloc: an IPC handle names a
// whole allocation); every other rank maps it once (cudaIpcOpenMemHandle, peer
// access enabled lazily) and after each step copies its block into it with
// cudaMemcpyAsync on a stream of its own: the copy engines move it over NVLink
// while the SMs run the next step, and no rank waits for another inside the loop.

int zonos2cu_ipc_alloc(int device, long long bytes, void **dev_ptr_out, unsigned char handle[64])
{
    if (!dev_ptr_out || !handle || bytes <= 0) return ZONOS2CU_EINVAL;
    *dev_ptr_out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        (void)cudaGetLastError();
        return ZONOS2CU_EINVAL;
    }
    DeviceScope g(device);
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e != cudaSuccess) {
        z2_set_error("%s: %s", "ipc buffer", cudaGetErrorString(e));
        (void)cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? ZONOS2CU_ENOMEM : ZONOS2CU_ECUDA;
    }
    cudaIpcMemHandle_t h;
    static_assert(sizeof(h) == 64, "CUDA IPC handle size");
    e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        z2_set_error("%s: %s", "cudaIpcGetMemHandle", cudaGetErrorString(e));
        (void)cudaGetLastError();
        cudaFree(p);
        return ZONOS2CU_ECUDA;
    }
    memcpy(handle, &h, 64);
    *dev_ptr_out = p;
    return ZONOS2CU_OK;
}

int zonos2cu_ipc_free(void *dev_ptr)
{
    if (!dev_ptr) return ZONOS2CU_OK;
    const cudaError_t e = cudaFree(dev_ptr);
    if (e != cudaSuccess) {
        z2_set_error("%s: %s", "ipc buffer free", cudaGetErrorString(e));
        (void)cudaGetLastError();
        return ZONOS2CU_ECUDA;
    }
    return ZONOS2CU_OK;
}

int zonos2cu_ipc_open(int device, const unsigned char handle[64], void **dev_ptr_out)
{
    if (!handle || !dev_ptr_out) return ZONOS2CU_EINVAL;
    *dev_ptr_out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) {
        (void)cudaGetLastError();
        return ZONOS2CU_EINVAL;
    }
    DeviceScope g(device);
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        z2_set_error("%s: %s", "cudaIpcOpenMemHandle", cudaGetErrorString(e));
        (void)cudaGetLastError();
        return ZONOS2CU_ECUDA;
    }
    *dev_ptr_out = p;
    return ZONOS2CU_OK;
}

int zonos2cu_ipc_close(void *dev_ptr)
{
    if (!dev_ptr) return ZONOS2CU_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    if (e != cudaSuccess) {
        z2_set_error("%s: %s", "cudaIpcCloseMemHandle", cudaGetErrorString(e));
        (void)cudaGetLastError();
        return ZONOS2CU_ECUDA;
    }
    return ZONOS2CU_OK;
}

int zonos2cu_push_codes(const int32_t *codes_dev, int n_steps, long long elems_per_step,
                        int32_t *dst_dev, long long dst_stride, void *stream)
{
    if (n_steps < 0 || elems_per_step < 0 || dst_stride < elems_per_step) return ZONOS2CU_EINVAL;
    if (n_steps == 0 || elems_per_step == 0) return ZONOS2CU_OK;
    if (!codes_dev || !dst_dev) return ZONOS2CU_EINVAL;
    // n_steps blocks, contiguous at the source, dst_stride apart at the
    // destination: one strided copy
    const size_t w = sizeof(int32_t) * (size_t)elems_per_step;
    const cudaError_t e = cudaMemcpy2DAsync(dst_dev, sizeof(int32_t) * (size_t)dst_stride, codes_dev,
                                            w, w, (size_t)n_steps, cudaMemcpyDeviceToDevice,
                                            static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        z2_set_error("%s: %s", "push copy", cudaGetErrorString(e));
        (void)cudaGetLastError();
        return ZONOS2CU_ECUDA;
    }
    return ZONOS2CU_OK;
}

}  // extern "C"
