// comm.cu -- column-sharded linear: each GPU owns n/P output rows of W, runs
// the local GEMV/GEMM into its slice and an NCCL all-gather (NVLink/NVSwitch)
// reassembles the full output on every rank.
//
// The reference is single-device; its nearest counterpart is the row split of
// one projection over 8 AIE columns and the host gather of the per-column C
// sections (crates/xnpu-cli/src/main.rs:2186-2191, w4u_read_c :3066-3091).
//
// NCCL is bound at run time (dlopen of libnccl.so.2): in a process that has
// already loaded torch this resolves to torch's NCCL, so both share one
// library, and the rest of libxq4 works on machines without NCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <mutex>
#include <vector>
#include <new>
#include <string.h>

#include "xq4_internal.h"

namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    const char *(*GetErrorString)(ncclResult_t);
    bool ok;
};

NcclApi *nccl_api()
{
    static NcclApi api = [] {
        NcclApi a{};
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
        a.GetUniqueId = (decltype(a.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        a.CommInitRank = (decltype(a.CommInitRank))dlsym(h, "ncclCommInitRank");
        a.CommDestroy = (decltype(a.CommDestroy))dlsym(h, "ncclCommDestroy");
        a.AllGather = (decltype(a.AllGather))dlsym(h, "ncclAllGather");
        a.GetErrorString = (decltype(a.GetErrorString))dlsym(h, "ncclGetErrorString");
        a.ok = a.GetUniqueId && a.CommInitRank && a.CommDestroy && a.AllGather && a.GetErrorString;
        return a;
    }();
    return &api;
}

int nccl_fail(ncclResult_t r, const char *what)
{
    NcclApi *a = nccl_api();
    return xq4_fail(XQ4_ENCCL, "%s: %s", what, a->ok ? a->GetErrorString(r) : "NCCL unavailable");
}

// ws[p][t][j] -> y[t][p*ns + j]  (rank-major all-gather result -> token-major)
template <typename T>
__global__ void shard_permute(const T *__restrict__ ws, T *__restrict__ y, int nranks, int m, int ns)
{
    const size_t total = (size_t)nranks * m * ns;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t j = i % ns;
        const size_t rest = i / ns;
        const size_t t = rest % m, p = rest / m;
        y[t * ((size_t)nranks * ns) + p * ns + j] = ws[i];
    }
}

}  // namespace

// A buffer every rank allocated together and mapped from every peer.
struct shared_buf {
    char *local;
    size_t bytes;
    char *peer[XQ4_MAX_RANKS];  // peer[rank] == local; others opened from IPC handles
};

struct xq4_comm {
    xq4_device *dev;
    ncclComm_t nccl;
    int rank, nranks;
    // fused gather (created by the first xq4_linear_sharded_fused call): CTA
    // count at 0, epoch at 4, poison word at 8, the two inbox halves from
    // kInboxHead
    shared_buf inbox{};
    void *xchg = nullptr;               // device scratch for exchanging IPC handles
    unsigned *poison_host = nullptr;    // host-mapped flag: a kernel gave up waiting for a peer
    unsigned *poison_dev = nullptr;     // its device address
};

static constexpr size_t kInboxHead = 256;
static constexpr size_t kPoisonOff = 8;
static constexpr size_t kInboxHalfBytes = (size_t)XQ4_FUSED_MAX_VALUES * sizeof(unsigned long long);

extern "C" int xq4_comm_unique_id(void *id_out)
{
    xq4_clear_error();
    if (!id_out) return xq4_fail(XQ4_EINVAL, "NULL argument");
    static_assert(sizeof(ncclUniqueId) == XQ4_UNIQUE_ID_BYTES, "unique id size");
    NcclApi *a = nccl_api();
    if (!a->ok) return xq4_fail(XQ4_ENCCL, "libnccl.so.2 could not be loaded: %s", dlerror());
    ncclUniqueId id;
    ncclResult_t r = a->GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id_out, &id, sizeof id);
    return XQ4_OK;
}

extern "C" int xq4_comm_init(xq4_device *dev, int rank, int nranks, const void *unique_id, xq4_comm **out)
{
    xq4_clear_error();
    if (!dev || !unique_id || !out) return xq4_fail(XQ4_EINVAL, "NULL argument");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks)
        return xq4_fail(XQ4_EINVAL, "rank %d / nranks %d invalid", rank, nranks);
    NcclApi *a = nccl_api();
    if (!a->ok) return xq4_fail(XQ4_ENCCL, "libnccl.so.2 could not be loaded");
    cudaError_t e = cudaSetDevice(xq4_device_ordinal(dev));
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof id);
    ncclComm_t c;
    ncclResult_t r = a->CommInitRank(&c, nranks, id, rank);
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommInitRank");
    xq4_comm *cm = new (std::nothrow) xq4_comm{dev, c, rank, nranks};
    if (!cm) {
        a->CommDestroy(c);
        return xq4_fail(XQ4_ENOMEM, "host allocation");
    }
    *out = cm;
    return XQ4_OK;
}

extern "C" int xq4_comm_destroy(xq4_comm *comm)
{
    xq4_clear_error();
    if (!comm) return XQ4_OK;
    NcclApi *a = nccl_api();
    cudaSetDevice(xq4_device_ordinal(comm->dev));
    if (comm->inbox.local) {
        // every rank stops using its peers' memory before any rank frees its own
        cudaDeviceSynchronize();
        int one = 1;
        int *d = (int *)comm->xchg;
        cudaMemcpy(d, &one, sizeof one, cudaMemcpyHostToDevice);
        a->AllGather(d, d + 16, 1, ncclInt32, comm->nccl, 0);
        cudaDeviceSynchronize();
        for (int r = 0; r < comm->nranks; r++)
            if (r != comm->rank && comm->inbox.peer[r]) cudaIpcCloseMemHandle(comm->inbox.peer[r]);
        a->AllGather(d, d + 16, 1, ncclInt32, comm->nccl, 0);
        cudaDeviceSynchronize();
        cudaFree(comm->inbox.local);
    }
    if (comm->xchg) cudaFree(comm->xchg);
    if (comm->poison_host) cudaFreeHost(comm->poison_host);
    ncclResult_t r = a->CommDestroy(comm->nccl);
    delete comm;
    if (r != ncclSuccess) return nccl_fail(r, "ncclCommDestroy");
    return XQ4_OK;
}

extern "C" int xq4_linear_sharded(xq4_comm *comm, const xq4_weight *w, const void *x_dev, void *y_full_dev,
                                  void *ws_dev, int m, int out_dtype, void *stream)
{
    xq4_clear_error();
    if (!comm || !w || !x_dev || !y_full_dev) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (m <= 0) return xq4_fail(XQ4_EINVAL, "m must be >= 1 (got %d)", m);
    if (out_dtype != XQ4_OUT_BF16 && out_dtype != XQ4_OUT_F32)
        return xq4_fail(XQ4_EINVAL, "unknown out_dtype %d", out_dtype);
    if (m > 1 && !ws_dev) return xq4_fail(XQ4_EINVAL, "m > 1 needs a workspace");
    const size_t esz = out_dtype == XQ4_OUT_F32 ? 4 : 2;
    const int ns = w->n;
    if ((ns * esz) % 16)
        return xq4_fail(XQ4_EINVAL, "shard rows (%d) x element size must be a multiple of 16 bytes", ns);
    if (((uintptr_t)x_dev & 15) || ((uintptr_t)y_full_dev & 15) || ((uintptr_t)ws_dev & 15))
        return xq4_fail(XQ4_EINVAL, "x, y and ws must be 16-byte aligned");
    NcclApi *a = nccl_api();
    if (!a->ok) return xq4_fail(XQ4_ENCCL, "libnccl.so.2 could not be loaded");
    cudaError_t e = cudaSetDevice(xq4_device_ordinal(comm->dev));
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    cudaStream_t st = (cudaStream_t)stream;  // NULL = CUDA's default stream
    const int f32 = out_dtype == XQ4_OUT_F32;
    const ncclDataType_t dt = f32 ? ncclFloat32 : ncclBfloat16;
    const size_t slice = (size_t)m * ns;  // elements per rank
    char *gather = (char *)(m == 1 ? y_full_dev : ws_dev);
    void *mine = gather + (size_t)comm->rank * slice * esz;
    e = xq4_use_gemv(m) ? xq4_launch_gemv(w->d_pack, w->n, w->k, x_dev, m, mine, f32, st)
                        : xq4_launch_gemm(w->d_pack, w->n, w->k, x_dev, m, mine, f32, st);
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "shard linear launch: %s", cudaGetErrorString(e));
    ncclResult_t r = a->AllGather(mine, gather, slice, dt, comm->nccl, st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    if (m > 1) {
        const size_t total = slice * comm->nranks;
        const unsigned blocks = (unsigned)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
        if (f32)
            shard_permute<float><<<blocks, 256, 0, st>>>((const float *)ws_dev, (float *)y_full_dev,
                                                         comm->nranks, m, ns);
        else
            shard_permute<uint16_t><<<blocks, 256, 0, st>>>((const uint16_t *)ws_dev, (uint16_t *)y_full_dev,
                                                            comm->nranks, m, ns);
        e = cudaGetLastError();
        if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "shard permute: %s", cudaGetErrorString(e));
    }
    return XQ4_OK;
}

// ------------------------------------------------------------------ no allocation
// xq4_linear_sharded_noalloc: the same sharded linear for callers that cannot
// allocate device memory at the time of the call -- a serving engine that has
// reserved the GPU's memory for weights and KV cache up front and refuses
// later allocations, a decode loop that cannot afford cudaMalloc/cudaFree
// (cudaFree synchronises the whole device), or a foreign-language caller of
// this C ABI with no device allocator of its own.  Instead of the caller's
// workspace, the m > 1 gather stages through the fixed array below (8 MiB,
// which every GPU that loads this library holds until the process exits).
// Nothing in it needs to start at zero: each call writes the whole gather
// region (local slice, then the all-gather) before the permute reads it.
// Every call shares the array, so calls that overlap on the GPU (other
// streams, other threads) race on it.
static __device__ __align__(256) unsigned char g_xq4_noalloc_scratch[XQ4_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on device `ordinal` (current), looked
// up once per device.
static int noalloc_scratch(int ordinal, void **out)
{
    static void *addr[64];
    static bool ready[64];
    static std::mutex mu;
    if (ordinal < 0 || ordinal >= 64) return xq4_fail(XQ4_EINVAL, "device ordinal %d out of range", ordinal);
    std::lock_guard<std::mutex> lock(mu);
    if (!ready[ordinal]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_xq4_noalloc_scratch);
        if (e != cudaSuccess)
            return xq4_fail(XQ4_ECUDA, "cudaGetSymbolAddress(no-allocation scratch): %s", cudaGetErrorString(e));
        addr[ordinal] = p;
        ready[ordinal] = true;
    }
    *out = addr[ordinal];
    return XQ4_OK;
}

extern "C" int xq4_linear_sharded_noalloc(xq4_comm *comm, const xq4_weight *w, const void *x_dev,
                                          void *y_full_dev, int m, int out_dtype, void *stream)
{
    xq4_clear_error();
    if (!comm || !w || !x_dev || !y_full_dev) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (m <= 0) return xq4_fail(XQ4_EINVAL, "m must be >= 1 (got %d)", m);
    if (out_dtype != XQ4_OUT_BF16 && out_dtype != XQ4_OUT_F32)
        return xq4_fail(XQ4_EINVAL, "unknown out_dtype %d", out_dtype);
    const size_t esz = out_dtype == XQ4_OUT_F32 ? 4 : 2;
    const int ns = w->n;
    if ((ns * esz) % 16)
        return xq4_fail(XQ4_EINVAL, "shard rows (%d) x element size must be a multiple of 16 bytes", ns);
    const size_t need = m > 1 ? (size_t)m * ns * comm->nranks * esz : 0;
    if (need > XQ4_NOALLOC_SCRATCH_BYTES)
        return xq4_fail(XQ4_EINVAL,
                        "m x n_total x element size = %zu bytes exceeds the %u-byte scratch of the no-allocation "
                        "entry point (use xq4_linear_sharded with a workspace)",
                        need, (unsigned)XQ4_NOALLOC_SCRATCH_BYTES);
    if (((uintptr_t)x_dev & 15) || ((uintptr_t)y_full_dev & 15))
        return xq4_fail(XQ4_EINVAL, "x and y must be 16-byte aligned");
    NcclApi *a = nccl_api();
    if (!a->ok) return xq4_fail(XQ4_ENCCL, "libnccl.so.2 could not be loaded");
    const int ordinal = xq4_device_ordinal(comm->dev);
    cudaError_t e = cudaSetDevice(ordinal);
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    void *ws = nullptr;
    if (m > 1)
        if (int rc = noalloc_scratch(ordinal, &ws)) return rc;
    cudaStream_t st = (cudaStream_t)stream;  // NULL = CUDA's default stream
    const int f32 = out_dtype == XQ4_OUT_F32;
    const ncclDataType_t dt = f32 ? ncclFloat32 : ncclBfloat16;
    const size_t slice = (size_t)m * ns;  // elements per rank
    char *gather = (char *)(m == 1 ? y_full_dev : ws);
    void *mine = gather + (size_t)comm->rank * slice * esz;
    e = xq4_use_gemv(m) ? xq4_launch_gemv(w->d_pack, w->n, w->k, x_dev, m, mine, f32, st)
                        : xq4_launch_gemm(w->d_pack, w->n, w->k, x_dev, m, mine, f32, st);
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "shard linear launch: %s", cudaGetErrorString(e));
    ncclResult_t r = a->AllGather(mine, gather, slice, dt, comm->nccl, st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    if (m > 1) {
        const size_t total = slice * comm->nranks;
        const unsigned blocks = (unsigned)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
        if (f32)
            shard_permute<float><<<blocks, 256, 0, st>>>((const float *)ws, (float *)y_full_dev, comm->nranks, m, ns);
        else
            shard_permute<uint16_t><<<blocks, 256, 0, st>>>((const uint16_t *)ws, (uint16_t *)y_full_dev,
                                                            comm->nranks, m, ns);
        e = cudaGetLastError();
        if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "shard permute: %s", cudaGetErrorString(e));
    }
    return XQ4_OK;
}

// ------------------------------------------------------------------ peer-memory gather
namespace {

// Allocate `bytes` on every rank and map every peer's allocation (collective).
int alloc_shared(xq4_comm *comm, size_t bytes, shared_buf *out)
{
    NcclApi *a = nccl_api();
    shared_buf b{};
    b.bytes = bytes;
    cudaError_t e = cudaMalloc((void **)&b.local, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return xq4_fail(XQ4_ENOMEM, "cudaMalloc(%zu) for a shared buffer: %s", bytes, cudaGetErrorString(e));
    }
    cudaMemset(b.local, 0, bytes);
    cudaIpcMemHandle_t mine, all[XQ4_MAX_RANKS];
    e = cudaIpcGetMemHandle(&mine, b.local);
    if (e != cudaSuccess) {
        cudaFree(b.local);
        return xq4_fail(XQ4_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    }
    char *x = (char *)comm->xchg;
    cudaMemcpy(x, &mine, sizeof mine, cudaMemcpyHostToDevice);
    ncclResult_t r = a->AllGather(x, x + sizeof mine, sizeof mine, ncclUint8, comm->nccl, 0);
    if (r != ncclSuccess) {
        cudaFree(b.local);
        return nccl_fail(r, "ncclAllGather(IPC handles)");
    }
    e = cudaMemcpy(all, x + sizeof mine, sizeof mine * comm->nranks, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        cudaFree(b.local);
        return xq4_fail(XQ4_ECUDA, "IPC handle exchange: %s", cudaGetErrorString(e));
    }
    for (int q = 0; q < comm->nranks; q++) {
        if (q == comm->rank) {
            b.peer[q] = b.local;
            continue;
        }
        void *p = nullptr;
        e = cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int j = 0; j < q; j++)
                if (j != comm->rank && b.peer[j]) cudaIpcCloseMemHandle(b.peer[j]);
            cudaFree(b.local);
            return xq4_fail(XQ4_ECUDA, "cudaIpcOpenMemHandle(rank %d): %s", q, cudaGetErrorString(e));
        }
        b.peer[q] = (char *)p;
    }
    *out = b;
    return XQ4_OK;
}

}  // namespace

namespace {

// First fused call on a communicator: map every rank's inbox (collective).
// The inbox is zeroed before its handle leaves this rank, so no peer writes
// into it before that.
int setup_inbox(xq4_comm *comm)
{
    if (!comm->poison_host) {
        void *h = nullptr;
        cudaError_t e = cudaHostAlloc(&h, 64, cudaHostAllocMapped);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return xq4_fail(XQ4_ENOMEM, "cudaHostAlloc for the communicator's poison flag: %s", cudaGetErrorString(e));
        }
        memset(h, 0, 64);
        void *d = nullptr;
        e = cudaHostGetDevicePointer(&d, h, 0);
        if (e != cudaSuccess) {
            cudaFreeHost(h);
            return xq4_fail(XQ4_ECUDA, "cudaHostGetDevicePointer: %s", cudaGetErrorString(e));
        }
        comm->poison_host = (unsigned *)h;
        comm->poison_dev = (unsigned *)d;
    }
    cudaError_t e = cudaMalloc(&comm->xchg, 64 * 2 * (XQ4_MAX_RANKS + 1));
    if (e != cudaSuccess) {
        cudaGetLastError();
        comm->xchg = nullptr;
        return xq4_fail(XQ4_ENOMEM, "cudaMalloc for the handle exchange: %s", cudaGetErrorString(e));
    }
    if (int rc = alloc_shared(comm, kInboxHead + 2 * kInboxHalfBytes, &comm->inbox)) {
        cudaFree(comm->xchg);
        comm->xchg = nullptr;
        comm->inbox = shared_buf{};
        return rc;
    }
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "inbox set-up: %s", cudaGetErrorString(e));
    return XQ4_OK;
}

}  // namespace

int xq4_comm_nranks(const xq4_comm *comm) { return comm->nranks; }
int xq4_comm_rank(const xq4_comm *comm) { return comm->rank; }

int xq4_comm_check_usable(const xq4_comm *comm)
{
    if (comm->poison_host && *(volatile const unsigned *)comm->poison_host)
        return xq4_fail(XQ4_ETIMEDOUT,
                        "an earlier call on this communicator gave up waiting for a peer's rows (fault bit 0x8); "
                        "the ranks' call counts are out of step: destroy and re-create the communicator");
    return XQ4_OK;
}

namespace {
void fill_poison(const xq4_comm *comm, xq4_p2p_poison *p)
{
    *p = xq4_p2p_poison{};
    for (int q = 0; q < comm->nranks; q++) p->word[q] = (unsigned *)(comm->inbox.peer[q] + kPoisonOff);
    p->host = comm->poison_dev;
}
}  // namespace

int xq4_comm_chain_p2p(xq4_comm *comm, const xq4_device *dev, xq4_chain_p2p *out)
{
    if (comm->dev != dev) return xq4_fail(XQ4_EINVAL, "communicator of another device");
    if (comm->nranks > XQ4_MAX_RANKS) return xq4_fail(XQ4_ENOTSUP, "more than %d ranks", XQ4_MAX_RANKS);
    *out = xq4_chain_p2p{};
    out->nranks = comm->nranks;
    out->rank = comm->rank;
    if (comm->nranks == 1) return XQ4_OK;
    cudaError_t e = cudaSetDevice(xq4_device_ordinal(comm->dev));
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    if (!comm->inbox.local)
        if (int rc = setup_inbox(comm)) return rc;
    for (int q = 0; q < comm->nranks; q++)
        out->inbox[q] = (unsigned long long *)(comm->inbox.peer[q] + kInboxHead);
    out->half_words = XQ4_FUSED_MAX_VALUES;
    out->epoch = (unsigned *)(comm->inbox.local + 4);
    fill_poison(comm, &out->poison);
    return XQ4_OK;
}

extern "C" int xq4_linear_sharded_fused(xq4_comm *comm, const xq4_weight *w, const void *x_dev, void *y_full_dev,
                                        int m, int out_dtype, void *stream)
{
    xq4_clear_error();
    if (!comm || !w || !x_dev || !y_full_dev) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (m <= 0 || m > 15) return xq4_fail(XQ4_EINVAL, "m must be in 1..15 (got %d)", m);
    if (out_dtype != XQ4_OUT_BF16 && out_dtype != XQ4_OUT_F32)
        return xq4_fail(XQ4_EINVAL, "unknown out_dtype %d", out_dtype);
    if ((uintptr_t)x_dev & 15) return xq4_fail(XQ4_EINVAL, "x must be 16-byte aligned");
    if (((uintptr_t)y_full_dev & 3) && out_dtype == XQ4_OUT_F32) return xq4_fail(XQ4_EINVAL, "y must be 4-byte aligned");
    if ((uintptr_t)y_full_dev & 1) return xq4_fail(XQ4_EINVAL, "y must be 2-byte aligned");
    if (comm->nranks > XQ4_MAX_RANKS) return xq4_fail(XQ4_ENOTSUP, "more than %d ranks", XQ4_MAX_RANKS);
    const int ns = w->n;
    const size_t values = (size_t)m * ns * comm->nranks;
    if (values > XQ4_FUSED_MAX_VALUES)
        return xq4_fail(XQ4_EINVAL, "m x n_total = %zu is above XQ4_FUSED_MAX_VALUES (%u)", values,
                        (unsigned)XQ4_FUSED_MAX_VALUES);
    cudaError_t e = cudaSetDevice(xq4_device_ordinal(comm->dev));
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    if (!comm->inbox.local && comm->nranks > 1)
        if (int rc = setup_inbox(comm)) return rc;
    if (int rc = xq4_comm_check_usable(comm)) return rc;
    xq4_p2p_out p{};
    p.nranks = comm->nranks;
    p.rank = comm->rank;
    p.n_total = ns * comm->nranks;
    p.row_off = ns * comm->rank;
    if (comm->nranks > 1) {
        for (int q = 0; q < comm->nranks; q++)
            p.inbox[q] = (unsigned long long *)(comm->inbox.peer[q] + kInboxHead);
        p.half_words = XQ4_FUSED_MAX_VALUES;
        p.cnt = (unsigned *)comm->inbox.local;
        p.epoch = (unsigned *)(comm->inbox.local + 4);
        fill_poison(comm, &p.poison);
        e = xq4_launch_gemv(w->d_pack, w->n, w->k, x_dev, m, y_full_dev, out_dtype == XQ4_OUT_F32,
                            (cudaStream_t)stream, &p);
    } else {  // one rank: the shard is the whole matrix
        e = xq4_launch_gemv(w->d_pack, w->n, w->k, x_dev, m, y_full_dev, out_dtype == XQ4_OUT_F32,
                            (cudaStream_t)stream);
    }
    if (e == cudaErrorCooperativeLaunchTooLarge)
        return xq4_fail(XQ4_ENOTSUP, "fused sharded launch: its CTAs wait for the peers' matching CTAs, so the whole "
                                     "grid must be resident at once, and this device cannot hold it");
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "fused sharded launch: %s", cudaGetErrorString(e));
    return XQ4_OK;
}
