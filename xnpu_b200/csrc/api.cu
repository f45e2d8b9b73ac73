// api.cu -- the C ABI (include/xq4.h): devices, buffers, weights, the linear
// op and the timeline wait.  Mirrors the reference HAL's operator surface
// (crates/xnpu-hal/src/{accel,bo,hwctx,ert}.rs) over CUDA.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <limits.h>
#include <string.h>
#include <time.h>
#include <unistd.h>
#include <map>
#include <new>
#include <tuple>
#include <vector>

#include "xq4_internal.h"
#include "xq4_layout.h"

// ------------------------------------------------------------------ errors
static thread_local char g_err[512];

int xq4_fail(int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

void xq4_clear_error(void) { g_err[0] = 0; }

static int cuda_fail(cudaError_t e, const char *what)
{
    return xq4_fail(XQ4_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define CK(call, what)                                \
    do {                                              \
        cudaError_t e_ = (call);                      \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

extern "C" const char *xq4_last_error_string(void) { return g_err; }
extern "C" const char *xq4_version(void) { return "xq4 0.1 (sm_100a)"; }

// ------------------------------------------------------------------ device
namespace {
constexpr int kRing = 256;  // timeline points kept as live events
}

struct xq4_device {
    int ordinal;
    cudaStream_t stream;
    cudaEvent_t ring[kRing];
    uint64_t last_seq;      // newest submitted point (0 = none)
    uint64_t done_seq;      // newest point known complete
    cudaDeviceProp prop;
};

cudaStream_t xq4_device_cuda_stream(xq4_device *dev) { return dev->stream; }
int xq4_device_ordinal(const xq4_device *dev) { return dev->ordinal; }

extern "C" int xq4_device_open(int ordinal, xq4_device **out)
{
    xq4_clear_error();
    if (!out) return xq4_fail(XQ4_EINVAL, "out is NULL");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return xq4_fail(XQ4_ENODEV, "no CUDA device (%s)", e == cudaSuccess ? "count 0" : cudaGetErrorString(e));
    if (ordinal < 0 || ordinal >= count)
        return xq4_fail(XQ4_ENODEV, "device ordinal %d out of range [0, %d)", ordinal, count);
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, ordinal), "cudaGetDeviceProperties");
    if (prop.major != 10)
        return xq4_fail(XQ4_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a only", ordinal,
                        prop.major, prop.minor);
    CK(cudaSetDevice(ordinal), "cudaSetDevice");
    xq4_device *d = new (std::nothrow) xq4_device();
    if (!d) return xq4_fail(XQ4_ENOMEM, "host allocation");
    d->ordinal = ordinal;
    d->prop = prop;
    cudaError_t ce = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
    if (ce != cudaSuccess) {
        delete d;
        return cuda_fail(ce, "cudaStreamCreate");
    }
    for (int i = 0; i < kRing; i++) {
        ce = cudaEventCreateWithFlags(&d->ring[i], cudaEventDisableTiming);
        if (ce != cudaSuccess) {
            for (int j = 0; j < i; j++) cudaEventDestroy(d->ring[j]);
            cudaStreamDestroy(d->stream);
            delete d;
            return cuda_fail(ce, "cudaEventCreate");
        }
    }
    *out = d;
    return XQ4_OK;
}

extern "C" int xq4_device_close(xq4_device *dev)
{
    xq4_clear_error();
    if (!dev) return XQ4_OK;
    cudaSetDevice(dev->ordinal);
    cudaError_t e = cudaStreamSynchronize(dev->stream);
    for (int i = 0; i < kRing; i++) cudaEventDestroy(dev->ring[i]);
    cudaStreamDestroy(dev->stream);
    delete dev;
    if (e != cudaSuccess) return cuda_fail(e, "draining the device queue at close");
    return XQ4_OK;
}

extern "C" int xq4_device_query(const xq4_device *dev, xq4_device_info *info)
{
    xq4_clear_error();
    if (!dev || !info) return xq4_fail(XQ4_EINVAL, "NULL argument");
    memset(info, 0, sizeof *info);
    info->ordinal = dev->ordinal;
    info->sm_count = dev->prop.multiProcessorCount;
    info->cc_major = dev->prop.major;
    info->cc_minor = dev->prop.minor;
    info->hbm_bytes = dev->prop.totalGlobalMem;
    info->l2_bytes = (size_t)dev->prop.l2CacheSize;
    snprintf(info->name, sizeof info->name, "%.95s", dev->prop.name);
    return XQ4_OK;
}

extern "C" void *xq4_device_stream(xq4_device *dev) { return dev ? (void *)dev->stream : nullptr; }

// ------------------------------------------------------------------ buffers
struct xq4_buffer {
    xq4_device *dev;
    int ordinal;  // destroy does not touch `dev`, which may be closed already
    void *ptr;
    size_t bytes;
};

extern "C" int xq4_buffer_create(xq4_device *dev, size_t bytes, xq4_buffer **out)
{
    xq4_clear_error();
    if (!dev || !out) return xq4_fail(XQ4_EINVAL, "NULL argument");
    *out = nullptr;
    if (bytes == 0) return xq4_fail(XQ4_EINVAL, "zero-size buffer");
    CK(cudaSetDevice(dev->ordinal), "cudaSetDevice");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return xq4_fail(XQ4_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    xq4_buffer *b = new (std::nothrow) xq4_buffer{dev, dev->ordinal, p, bytes};
    if (!b) {
        cudaFree(p);
        return xq4_fail(XQ4_ENOMEM, "host allocation");
    }
    *out = b;
    return XQ4_OK;
}

static int check_range(const xq4_buffer *buf, size_t off, size_t len)
{
    if (off > buf->bytes || len > buf->bytes - off)
        return xq4_fail(XQ4_EINVAL, "range [%zu, %zu) outside buffer of %zu bytes", off, off + len, buf->bytes);
    return XQ4_OK;
}

extern "C" int xq4_buffer_upload(xq4_buffer *buf, const void *host, size_t offset, size_t len)
{
    xq4_clear_error();
    if (!buf || (!host && len)) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (int rc = check_range(buf, offset, len)) return rc;
    if (!len) return XQ4_OK;
    CK(cudaSetDevice(buf->dev->ordinal), "cudaSetDevice");
    CK(cudaMemcpyAsync((char *)buf->ptr + offset, host, len, cudaMemcpyHostToDevice, buf->dev->stream),
       "upload");
    CK(cudaStreamSynchronize(buf->dev->stream), "upload sync");
    return XQ4_OK;
}

extern "C" int xq4_buffer_download(xq4_buffer *buf, void *host, size_t offset, size_t len)
{
    xq4_clear_error();
    if (!buf || (!host && len)) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (int rc = check_range(buf, offset, len)) return rc;
    if (!len) return XQ4_OK;
    CK(cudaSetDevice(buf->dev->ordinal), "cudaSetDevice");
    CK(cudaMemcpyAsync(host, (const char *)buf->ptr + offset, len, cudaMemcpyDeviceToHost, buf->dev->stream),
       "download");
    CK(cudaStreamSynchronize(buf->dev->stream), "download sync");
    return XQ4_OK;
}

extern "C" int xq4_buffer_destroy(xq4_buffer *buf)
{
    xq4_clear_error();
    if (!buf) return XQ4_OK;
    cudaSetDevice(buf->ordinal);
    cudaDeviceSynchronize();  // no queued op may still use it
    cudaError_t e = cudaFree(buf->ptr);
    delete buf;
    if (e != cudaSuccess) return cuda_fail(e, "cudaFree");
    return XQ4_OK;
}

extern "C" void *xq4_buffer_device_ptr(const xq4_buffer *buf) { return buf ? buf->ptr : nullptr; }
extern "C" size_t xq4_buffer_size(const xq4_buffer *buf) { return buf ? buf->bytes : 0; }

// ------------------------------------------------------------------ weights
extern "C" int xq4_weight_import(xq4_device *dev, const void *src, size_t src_len,
                                 const xq4_layout_desc *desc, xq4_weight **out)
{
    xq4_clear_error();
    if (!dev || !src || !out) return xq4_fail(XQ4_EINVAL, "NULL argument");
    *out = nullptr;
    int r0, r1;
    if (int rc = xq4_check_desc(desc, src_len, &r0, &r1)) return rc;
    const int n = r1 - r0, k = desc->k;
    const size_t bytes = xq4g_bytes(n, k);
    std::vector<uint8_t> host;
    try {
        host.resize(bytes);
    } catch (...) {
        return xq4_fail(XQ4_ENOMEM, "host staging of %zu bytes", bytes);
    }
    if (int rc = xq4_repack_rows(src, src_len, desc, r0, r1, host.data())) return rc;
    CK(cudaSetDevice(dev->ordinal), "cudaSetDevice");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return xq4_fail(XQ4_ENOMEM, "cudaMalloc(%zu) for weight: %s", bytes, cudaGetErrorString(e));
    }
    e = cudaMemcpyAsync(p, host.data(), bytes, cudaMemcpyHostToDevice, dev->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(dev->stream);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "weight upload");
    }
    xq4_weight *w = new (std::nothrow) xq4_weight();
    if (!w) {
        cudaFree(p);
        return xq4_fail(XQ4_ENOMEM, "host allocation");
    }
    w->dev = dev;
    w->ordinal = dev->ordinal;
    w->n = n;
    w->k = k;
    w->nb = xq4g_nb(n);
    w->kc = xq4g_kc(k);
    w->d_pack = (uint8_t *)p;
    w->bytes = bytes;
    *out = w;
    return XQ4_OK;
}

extern "C" int xq4_weight_destroy(xq4_weight *w)
{
    xq4_clear_error();
    if (!w) return XQ4_OK;
    cudaSetDevice(w->ordinal);
    cudaDeviceSynchronize();  // no queued op may still use it
    cudaError_t e = cudaFree(w->d_pack);
    delete w;
    if (e != cudaSuccess) return cuda_fail(e, "cudaFree(weight)");
    return XQ4_OK;
}

extern "C" int xq4_weight_shape(const xq4_weight *w, int *n, int *k, size_t *device_bytes)
{
    xq4_clear_error();
    if (!w) return xq4_fail(XQ4_EINVAL, "NULL weight");
    if (n) *n = w->n;
    if (k) *k = w->k;
    if (device_bytes) *device_bytes = w->bytes;
    return XQ4_OK;
}

extern "C" int xq4_dequant(const xq4_weight *w, void *out_dev, void *stream)
{
    xq4_clear_error();
    if (!w || !out_dev) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if ((uintptr_t)out_dev & 15) return xq4_fail(XQ4_EINVAL, "output must be 16-byte aligned");
    CK(cudaSetDevice(w->ordinal), "cudaSetDevice");
    // NULL is CUDA's default stream, as everywhere in the CUDA API
    cudaStream_t st = (cudaStream_t)stream;
    CK(xq4_launch_dequant(w->d_pack, w->n, w->k, out_dev, st), "dequant launch");
    return XQ4_OK;
}

// ------------------------------------------------------------------ W4A8 parity mode
extern "C" int xq4_quantize_x(const void *x_dev, int m, int k, void *q_dev, void *d_dev, int device, void *stream)
{
    xq4_clear_error();
    if (!x_dev || !q_dev || !d_dev) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (m <= 0 || k <= 0 || k % 32) return xq4_fail(XQ4_EINVAL, "m >= 1 and k a positive multiple of 32 (got m=%d k=%d)", m, k);
    CK(cudaSetDevice(device), "cudaSetDevice");
    CK(xq4_launch_quantize_x(x_dev, m, k, q_dev, d_dev, (cudaStream_t)stream), "quantize launch");
    return XQ4_OK;
}

extern "C" int xq4_linear_w4a8(const xq4_weight *w, const void *q_dev, const void *d_dev, void *y_dev, int m,
                               int out_dtype, void *stream)
{
    xq4_clear_error();
    if (!w || !q_dev || !d_dev || !y_dev) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (m <= 0) return xq4_fail(XQ4_EINVAL, "m must be >= 1 (got %d)", m);
    if (out_dtype != XQ4_OUT_BF16 && out_dtype != XQ4_OUT_F32)
        return xq4_fail(XQ4_EINVAL, "unknown out_dtype %d", out_dtype);
    if (((uintptr_t)q_dev & 15) || (w->k % 16))
        return xq4_fail(XQ4_EINVAL, "q must be 16-byte aligned");
    CK(cudaSetDevice(w->ordinal), "cudaSetDevice");
    cudaError_t e = xq4_launch_w4a8(w->d_pack, w->n, w->k, q_dev, d_dev, m, y_dev, out_dtype == XQ4_OUT_F32,
                                    (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "w4a8 launch");
    return XQ4_OK;
}

// ------------------------------------------------------------------ linear
static int launch_linear(const xq4_weight *w, const void *x, void *y, int m, int out_dtype, cudaStream_t st)
{
    if (m <= 0) return xq4_fail(XQ4_EINVAL, "m must be >= 1 (got %d)", m);
    if (out_dtype != XQ4_OUT_BF16 && out_dtype != XQ4_OUT_F32)
        return xq4_fail(XQ4_EINVAL, "unknown out_dtype %d", out_dtype);
    if (((uintptr_t)x & 15) || ((uintptr_t)y & 15))
        return xq4_fail(XQ4_EINVAL, "x and y must be 16-byte aligned");
    const int f32 = out_dtype == XQ4_OUT_F32;
    const bool gemv = xq4_use_gemv(m);
    cudaError_t e = gemv ? xq4_launch_gemv(w->d_pack, w->n, w->k, x, m, y, f32, st)
                         : xq4_launch_gemm(w->d_pack, w->n, w->k, x, m, y, f32, st);
    if (e != cudaSuccess) return cuda_fail(e, gemv ? "gemv launch" : "gemm launch");
    return XQ4_OK;
}

extern "C" int xq4_linear(xq4_device *dev, const xq4_weight *w, const xq4_buffer *x_buf, size_t x_off,
                          xq4_buffer *y_buf, size_t y_off, int m, int out_dtype, uint64_t *seq)
{
    xq4_clear_error();
    if (!dev || !w || !x_buf || !y_buf) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (w->dev != dev || x_buf->dev != dev || y_buf->dev != dev)
        return xq4_fail(XQ4_EINVAL, "weight and buffers must belong to this device");
    if (m <= 0) return xq4_fail(XQ4_EINVAL, "m must be >= 1 (got %d)", m);
    const size_t xb = (size_t)m * w->k * 2, yb = (size_t)m * w->n * (out_dtype == XQ4_OUT_F32 ? 4 : 2);
    if (int rc = check_range(x_buf, x_off, xb)) return rc;
    if (int rc = check_range(y_buf, y_off, yb)) return rc;
    CK(cudaSetDevice(dev->ordinal), "cudaSetDevice");
    int rc = launch_linear(w, (const char *)x_buf->ptr + x_off, (char *)y_buf->ptr + y_off, m, out_dtype,
                           dev->stream);
    if (rc) return rc;
    const uint64_t s = dev->last_seq + 1;
    CK(cudaEventRecord(dev->ring[s % kRing], dev->stream), "cudaEventRecord");
    dev->last_seq = s;
    if (seq) *seq = s;
    return XQ4_OK;
}

extern "C" int xq4_linear_raw(const xq4_weight *w, const void *x_dev, void *y_dev, int m, int out_dtype,
                              void *stream)
{
    xq4_clear_error();
    if (!w || !x_dev || !y_dev) return xq4_fail(XQ4_EINVAL, "NULL argument");
    // NULL is CUDA's default stream (not the device queue): a caller on the
    // default stream gets its own stream order.
    CK(cudaSetDevice(w->ordinal), "cudaSetDevice");
    return launch_linear(w, x_dev, y_dev, m, out_dtype, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ op chains
struct xq4_chain {
    xq4_device *dev;
    int ordinal;
    int n_ops, n_preps;
    xq4_chain_op_dev *d_ops;  // one allocation: op table, segment counters, prep table,
    xq4_chain_prep_dev *d_preps;  // plan (segment CTA counts, visit lists), fp16 images
    xq4_chain_plan plan;
    int grid;                 // CTAs per launch (the plan's)
    bool has_w4a8;            // some op runs in the W4A8 mode
    xq4_chain_p2p p2p;        // sharded ops' communicator (nranks 1: none)
    xq4_comm *comm;           // that communicator, or NULL
};

extern "C" int xq4_chain_create(xq4_device *dev, const xq4_chain_op *ops, int n_ops, xq4_chain **out)
{
    xq4_clear_error();
    if (!dev || !ops || !out) return xq4_fail(XQ4_EINVAL, "NULL argument");
    *out = nullptr;
    if (n_ops <= 0 || n_ops > (1 << 20)) return xq4_fail(XQ4_EINVAL, "n_ops %d out of range", n_ops);
    std::vector<xq4_chain_op_dev> tab((size_t)n_ops);
    xq4_comm *comm = nullptr;
    for (int i = 0; i < n_ops; i++) {
        if (!ops[i].comm) continue;
        if (comm && ops[i].comm != comm) return xq4_fail(XQ4_EINVAL, "op %d: a second communicator in one chain", i);
        comm = ops[i].comm;
    }
    xq4_chain_p2p p2p{};
    p2p.nranks = 1;
    CK(cudaSetDevice(dev->ordinal), "cudaSetDevice");
    {
        const cudaError_t e = xq4_gemv_chain_prepare();
        if (e == cudaErrorCooperativeLaunchTooLarge)
            return xq4_fail(XQ4_ENOTSUP, "chain: its ops wait for one another across CTAs, so all of its CTAs (2 per "
                                         "SM) must be resident at once, and this device cannot hold them");
        if (e != cudaSuccess) return cuda_fail(e, "chain kernel set-up");
    }
    if (comm) {
        if (int rc = xq4_comm_chain_p2p(comm, dev, &p2p)) return rc;
        if (int rc = xq4_comm_check_usable(comm)) return rc;
    }
    long long inbox_words = 0;
    for (int i = 0; i < n_ops; i++) {
        const xq4_chain_op &o = ops[i];
        if (!o.w || !o.x_dev || !o.y_dev) return xq4_fail(XQ4_EINVAL, "op %d: NULL weight or pointer", i);
        if (o.w->dev != dev) return xq4_fail(XQ4_EINVAL, "op %d: weight of another device", i);
        if (o.m < 1 || o.m > 8) return xq4_fail(XQ4_EINVAL, "op %d: m must be in 1..8 (got %d)", i, o.m);
        if (o.out_dtype != XQ4_OUT_BF16 && o.out_dtype != XQ4_OUT_F32)
            return xq4_fail(XQ4_EINVAL, "op %d: unknown out_dtype %d", i, o.out_dtype);
        const uintptr_t ya = o.out_dtype == XQ4_OUT_F32 ? 3 : 1;
        if (((uintptr_t)o.x_dev & 15) || ((uintptr_t)o.y_dev & ya))
            return xq4_fail(XQ4_EINVAL, "op %d: x must be 16-byte aligned and y aligned to its element", i);
        xq4_chain_op_dev &d = tab[(size_t)i];
        d.pack = o.w->d_pack;
        d.x = o.x_dev;
        d.y = o.y_dev;
        d.n = o.w->n;
        d.k = o.w->k;
        d.nb = o.w->nb;
        d.kc = o.w->kc;
        d.m = o.m;
        d.out_f32 = o.out_dtype == XQ4_OUT_F32;
        d.wait_prev = o.wait_prev != 0;
        d.xh = 0;
        d.xh_img = nullptr;
        d.xh_tbl = nullptr;
        d.xh_tbl1 = nullptr;
        d.w4a8 = 0;
        d.qx_img = nullptr;
        d.qx_tbl = nullptr;
        d.xh_max = nullptr;
        d.spr = (d.kc + XQ4_GEMV_STAGE_CHUNKS_ABI - 1) / XQ4_GEMV_STAGE_CHUNKS_ABI;
        d.shard = o.comm && p2p.nranks > 1;
        d.residual = (const uint16_t *)o.residual_dev;
        d.res_ext = 0;
        d.swiglu = o.swiglu != 0;
        if (o.residual_dev || o.swiglu || o.norm_w_dev) {
            if (o.comm && o.residual_dev) return xq4_fail(XQ4_EINVAL, "op %d: a residual epilogue on a sharded op", i);
            if ((o.residual_dev || o.swiglu) && o.out_dtype != XQ4_OUT_BF16)
                return xq4_fail(XQ4_EINVAL, "op %d: a residual or SwiGLU epilogue writes bf16 only", i);
            if (o.residual_dev && o.swiglu) return xq4_fail(XQ4_EINVAL, "op %d: residual and SwiGLU together", i);
            if (o.swiglu && (o.w->n & 1)) return xq4_fail(XQ4_EINVAL, "op %d: SwiGLU needs an even row count", i);
            if ((uintptr_t)o.residual_dev & 1) return xq4_fail(XQ4_EINVAL, "op %d: residual not 2-byte aligned", i);
            if ((uintptr_t)o.norm_w_dev & 15) return xq4_fail(XQ4_EINVAL, "op %d: norm weights not 16-byte aligned", i);
            if (o.norm_w_dev && !(o.norm_eps >= 0.f)) return xq4_fail(XQ4_EINVAL, "op %d: norm_eps must be >= 0", i);
        }
        d.n_total = o.w->n * (d.shard ? p2p.nranks : 1);
        d.row_off = d.shard ? o.w->n * p2p.rank : 0;
        d.inbox_off = 0;
        if (d.shard) {
            d.inbox_off = inbox_words;
            inbox_words += (long long)o.m * (d.swiglu ? d.n_total / 2 : d.n_total);
            if (inbox_words > (long long)XQ4_FUSED_MAX_VALUES)
                return xq4_fail(XQ4_EINVAL, "sharded ops: m x n_total summed to %lld, above XQ4_FUSED_MAX_VALUES",
                                inbox_words);
        }
    }
    // segments: a new one starts at op 0 and at every op that waits
    std::vector<int> op_seg((size_t)n_ops);
    int n_seg = 0;
    for (int i = 0; i < n_ops; n_seg++) {
        int j = i + 1;
        while (j < n_ops && !tab[(size_t)j].wait_prev) j++;
        long long units = 0;
        for (int q = i; q < j; q++) {
            tab[(size_t)q].seg_start = units;
            units += (long long)tab[(size_t)q].nb * tab[(size_t)q].spr;
            op_seg[(size_t)q] = n_seg;
        }
        for (int q = i; q < j; q++) tab[(size_t)q].seg_units = units;
        i = j;
    }
    // fp16 path for every op whose x no op of the chain writes: each distinct
    // such activation is converted once per run by the prep kernel
    struct prep_key {
        const void *x;
        int m, k;
        const void *norm_w;
        float eps;
        int w4a8;
        size_t img_off, tbl_off, tbl1_off, max_off, qx_off, qtbl_off;
    };
    // bytes of op j's output
    const auto y_bytes = [&](int j) {
        const size_t rows = (size_t)tab[(size_t)j].n_total / (tab[(size_t)j].swiglu ? 2 : 1);
        return (size_t)ops[j].m * rows * (ops[j].out_dtype == XQ4_OUT_F32 ? 4 : 2);
    };
    std::vector<prep_key> preps;
    std::vector<int> op_prep((size_t)n_ops, -1);
    const auto align = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t tab_bytes = align(tab.size() * sizeof(xq4_chain_op_dev));
    const size_t done_bytes = align(((size_t)n_seg + 1) * sizeof(unsigned));
    size_t img_bytes = 0;
    // residuals no op of the chain writes (the reducer reads those before the
    // consumers hand over the row block)
    for (int i = 0; i < n_ops; i++) {
        if (!ops[i].residual_dev) continue;
        const char *r0 = (const char *)ops[i].residual_dev, *r1 = r0 + (size_t)ops[i].m * ops[i].w->n * 2;
        bool written = false;
        for (int j = 0; j < n_ops && !written; j++) {
            const char *y0 = (const char *)ops[j].y_dev;
            written = r0 < y0 + y_bytes(j) && y0 < r1;
        }
        tab[(size_t)i].res_ext = written ? 0 : 1;
    }
    // An activation whose readers (ops without RMSNorm or W4A8) stream fewer
    // chunks in all than the single-op GEMV's fp16 threshold keeps the bf16
    // path: its prep launch would cost more than the fp16 path saves
    // (measured: the decode step's o chain, 7.7 -> 6.4 us per layer), and the
    // ops then compute along the same path as the single-op GEMV.
    // A sharded op counts at its full size, so that every rank and the
    // unsharded op take the same path.
    std::map<std::tuple<const void *, int, int>, long long> x_chunks;
    for (int i = 0; i < n_ops; i++)
        if (!ops[i].norm_w_dev && !ops[i].w4a8) {
            const xq4_chain_op_dev &d = tab[(size_t)i];
            const long long rbs = d.shard ? (d.n_total + XQ4G_ROWS - 1) / XQ4G_ROWS : d.nb;
            x_chunks[std::make_tuple(ops[i].x_dev, ops[i].m, ops[i].w->k)] += rbs * d.kc;
        }
    for (int i = 0; i < n_ops; i++) {
        const xq4_chain_op &o = ops[i];
        const char *x0 = (const char *)o.x_dev, *x1 = x0 + (size_t)o.m * o.w->k * 2;
        if (!o.norm_w_dev && !o.w4a8 && x_chunks[std::make_tuple(o.x_dev, o.m, o.w->k)] < XQ4_XH_MIN_CHUNKS)
            continue;  // bf16 path
        bool written = false;
        for (int j = 0; j < n_ops && !written; j++) {
            const char *y0 = (const char *)ops[j].y_dev;
            const char *y1 = y0 + y_bytes(j);
            written = x0 < y1 && y0 < x1;
        }
        if (written) {
            if (o.norm_w_dev)
                return xq4_fail(XQ4_EINVAL, "op %d: RMSNorm needs an activation no op of the chain writes", i);
            if (o.w4a8)
                return xq4_fail(XQ4_EINVAL, "op %d: W4A8 needs an activation no op of the chain writes", i);
            continue;
        }
        const int w8 = o.w4a8 != 0;
        int pi = -1;
        for (size_t q = 0; q < preps.size(); q++)
            if (preps[q].x == o.x_dev && preps[q].m == o.m && preps[q].k == o.w->k && preps[q].w4a8 == w8 &&
                preps[q].norm_w == o.norm_w_dev && (!o.norm_w_dev || preps[q].eps == o.norm_eps))
                pi = (int)q;
        if (pi < 0) {
            prep_key pk{o.x_dev, o.m, o.w->k, o.norm_w_dev, o.norm_eps, w8, 0, 0, 0, 0, 0, 0};
            const size_t kp = (size_t)o.w->kc * XQ4G_KCHUNK;
            if (w8) {  // int8 image and the per-group table
                pk.qx_off = img_bytes;
                img_bytes += align((size_t)o.m * kp);
                pk.qtbl_off = img_bytes;
                img_bytes += align((size_t)o.w->kc * 2 * 8 * sizeof(int2));
            } else {  // fp16 image and its zero-point tables
                pk.img_off = img_bytes;
                img_bytes += align((size_t)o.m * kp * 2);
                pk.tbl_off = img_bytes;
                img_bytes += align((size_t)o.w->kc * 32 * sizeof(float));
                pk.tbl1_off = img_bytes;
                img_bytes += align((size_t)o.w->kc * 2 * sizeof(float4));
            }
            pk.max_off = img_bytes;
            img_bytes += 256;
            pi = (int)preps.size();
            preps.push_back(pk);
        }
        op_prep[(size_t)i] = pi;
    }
    const size_t prep_bytes = align(preps.size() * sizeof(xq4_chain_prep_dev));
    // The plan: CTA c owns the row blocks of op i whose first stage falls in
    // [c*U/G, (c+1)*U/G) of its segment's U stages (shares differ by at most
    // one row block); its visits are the ops where that is not empty.
    const int grid = xq4_gemv_chain_grid();
    std::vector<int4> visits;
    std::vector<int> vstart((size_t)grid + 1);
    std::vector<unsigned> seg_cnt((size_t)n_seg, 0u);
    for (int c = 0; c < grid; c++) {
        vstart[(size_t)c] = (int)visits.size();
        for (int i = 0; i < n_ops; i++) {
            const xq4_chain_op_dev &d = tab[(size_t)i];
            const auto first_at = [&](long long st) -> int {  // first row block starting at stage >= st
                if (st <= 0) return 0;
                const long long r = (st + d.spr - 1) / d.spr;
                return r < d.nb ? (int)r : d.nb;
            };
            const int rb0 = first_at((long long)c * d.seg_units / grid - d.seg_start);
            const int rb1 = first_at((long long)(c + 1) * d.seg_units / grid - d.seg_start);
            if (rb0 >= rb1) continue;
            const int seg = op_seg[(size_t)i];
            const bool first = visits.size() == (size_t)vstart[(size_t)c] || (visits.back().w >> 2) != seg;
            if (first) {
                seg_cnt[(size_t)seg]++;
                if (visits.size() > (size_t)vstart[(size_t)c]) visits.back().w |= 2;  // last of its segment
            }
            visits.push_back(make_int4(i, rb0, rb1, seg << 2 | (first ? 1 : 0)));
        }
        if (visits.size() > (size_t)vstart[(size_t)c]) visits.back().w |= 2;
    }
    vstart[(size_t)grid] = (int)visits.size();
    if (visits.size() > (size_t)INT_MAX / 2 || n_seg >= (1 << 29))
        return xq4_fail(XQ4_EINVAL, "chain too large: %zu visits", visits.size());
    const size_t seg_bytes = align((size_t)n_seg * sizeof(unsigned));
    const size_t vstart_bytes = align(vstart.size() * sizeof(int));
    const size_t visit_bytes = align(visits.size() * sizeof(int4));
    const size_t plan_bytes = seg_bytes + vstart_bytes + visit_bytes;
    const size_t total = tab_bytes + done_bytes + prep_bytes + plan_bytes + img_bytes;
    CK(cudaSetDevice(dev->ordinal), "cudaSetDevice");
    void *mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, total);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return xq4_fail(XQ4_ENOMEM, "cudaMalloc(%zu) for the chain: %s", total, cudaGetErrorString(e));
    }
    char *base = (char *)mem, *plan_d = base + tab_bytes + done_bytes + prep_bytes, *img = plan_d + plan_bytes;
    xq4_chain_plan plan{};
    plan.seg_cnt = (const unsigned *)plan_d;
    plan.vstart = (const int *)(plan_d + seg_bytes);
    plan.visits = (const int4 *)(plan_d + seg_bytes + vstart_bytes);
    plan.done = (unsigned *)(base + tab_bytes);
    plan.n_seg = n_seg;
    std::vector<xq4_chain_prep_dev> ptab(preps.size());
    for (size_t q = 0; q < preps.size(); q++) {
        const prep_key &pk = preps[q];
        xq4_chain_prep_dev &pd = ptab[q];
        pd = xq4_chain_prep_dev{};
        pd.x = pk.x;
        pd.max = (unsigned *)(img + pk.max_off);
        pd.m = pk.m;
        pd.k = pk.k;
        pd.kc = (pk.k + XQ4G_KCHUNK - 1) / XQ4G_KCHUNK;
        pd.norm = pk.norm_w != nullptr;
        pd.norm_w = (const uint16_t *)pk.norm_w;
        pd.eps = pk.eps;
        pd.w4a8 = pk.w4a8;
        if (pk.w4a8) {
            pd.qx = (uint8_t *)(img + pk.qx_off);
            pd.qtbl = (int2 *)(img + pk.qtbl_off);
        } else {
            pd.img = (uint16_t *)(img + pk.img_off);
            pd.tbl = (float *)(img + pk.tbl_off);
            pd.tbl1 = (float4 *)(img + pk.tbl1_off);
        }
    }
    for (int i = 0; i < n_ops; i++) {
        const int pi = op_prep[(size_t)i];
        if (pi < 0) continue;
        xq4_chain_op_dev &d = tab[(size_t)i];
        if (ptab[(size_t)pi].w4a8) {
            d.w4a8 = 1;
            d.qx_img = ptab[(size_t)pi].qx;
            d.qx_tbl = ptab[(size_t)pi].qtbl;
            continue;
        }
        d.xh = 1;
        d.xh_img = ptab[(size_t)pi].img;
        d.xh_tbl = (const float4 *)ptab[(size_t)pi].tbl;
        d.xh_tbl1 = ptab[(size_t)pi].tbl1;
        d.xh_max = ptab[(size_t)pi].max;
    }
    e = cudaMemcpy(base, tab.data(), tab.size() * sizeof(xq4_chain_op_dev), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(base + tab_bytes, 0, done_bytes);
    if (e == cudaSuccess && !ptab.empty())
        e = cudaMemcpy(base + tab_bytes + done_bytes, ptab.data(), ptab.size() * sizeof(xq4_chain_prep_dev),
                       cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy((void *)plan.seg_cnt, seg_cnt.data(), seg_cnt.size() * sizeof(unsigned), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy((void *)plan.vstart, vstart.data(), vstart.size() * sizeof(int), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && !visits.empty())
        e = cudaMemcpy((void *)plan.visits, visits.data(), visits.size() * sizeof(int4), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(mem);
        return cuda_fail(e, "chain upload");
    }
    bool has_w4a8 = false;
    for (const xq4_chain_op_dev &d : tab) has_w4a8 = has_w4a8 || d.w4a8;
    xq4_chain *c = new (std::nothrow) xq4_chain{dev, dev->ordinal, n_ops, (int)preps.size(), (xq4_chain_op_dev *)mem,
                                                (xq4_chain_prep_dev *)(base + tab_bytes + done_bytes),
                                                plan, grid, has_w4a8, p2p,
                                                p2p.nranks > 1 ? comm : nullptr};
    if (!c) {
        cudaFree(mem);
        return xq4_fail(XQ4_ENOMEM, "host allocation");
    }
    *out = c;
    return XQ4_OK;
}

extern "C" int xq4_chain_destroy(xq4_chain *chain)
{
    xq4_clear_error();
    if (!chain) return XQ4_OK;
    cudaSetDevice(chain->ordinal);
    cudaError_t e = cudaDeviceSynchronize();  // no launch of this chain still reads the table
    cudaFree(chain->d_ops);
    delete chain;
    if (e != cudaSuccess) return cuda_fail(e, "chain destroy");
    return XQ4_OK;
}

extern "C" int xq4_chain_run(const xq4_chain *chain, void *stream)
{
    xq4_clear_error();
    if (!chain) return xq4_fail(XQ4_EINVAL, "NULL chain");
    if (chain->comm)
        if (int rc = xq4_comm_check_usable(chain->comm)) return rc;
    CK(cudaSetDevice(chain->ordinal), "cudaSetDevice");
    CK(xq4_launch_gemv_chain(chain->d_ops, chain->plan, chain->grid, chain->d_preps, chain->n_preps, chain->p2p,
                             chain->has_w4a8, (cudaStream_t)stream),
       "chain launch");
    return XQ4_OK;
}

extern "C" int xq4_chain_submit(xq4_device *dev, const xq4_chain *chain, uint64_t *seq)
{
    xq4_clear_error();
    if (!dev || !chain) return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (chain->dev != dev) return xq4_fail(XQ4_EINVAL, "chain of another device");
    if (chain->comm)
        if (int rc = xq4_comm_check_usable(chain->comm)) return rc;
    CK(cudaSetDevice(dev->ordinal), "cudaSetDevice");
    CK(xq4_launch_gemv_chain(chain->d_ops, chain->plan, chain->grid, chain->d_preps, chain->n_preps, chain->p2p,
                             chain->has_w4a8, dev->stream),
       "chain launch");
    const uint64_t s = dev->last_seq + 1;
    CK(cudaEventRecord(dev->ring[s % kRing], dev->stream), "cudaEventRecord");
    dev->last_seq = s;
    if (seq) *seq = s;
    return XQ4_OK;
}

static uint64_t now_ns()
{
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000000000ull + ts.tv_nsec;
}

extern "C" int xq4_wait(xq4_device *dev, uint64_t seq, int64_t timeout_ns)
{
    xq4_clear_error();
    if (!dev) return xq4_fail(XQ4_EINVAL, "NULL device");
    if (seq > dev->last_seq) return xq4_fail(XQ4_EINVAL, "seq %llu was never submitted (last %llu)",
                                             (unsigned long long)seq, (unsigned long long)dev->last_seq);
    if (seq <= dev->done_seq) return XQ4_OK;
    // An evicted point is covered by the oldest live one (in-order queue).
    uint64_t probe = seq;
    if (dev->last_seq >= (uint64_t)kRing && seq <= dev->last_seq - kRing) probe = dev->last_seq - kRing + 1;
    cudaEvent_t ev = dev->ring[probe % kRing];
    // Poll without sleeping for the first 2 ms (a decode step or a chain is
    // shorter: a sleep's timer slack would add tens of microseconds to every
    // wait), then sleep 20 us between polls.
    const uint64_t t0 = now_ns();
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) {
            if (probe > dev->done_seq) dev->done_seq = probe;
            return XQ4_OK;
        }
        if (e != cudaErrorNotReady) return cuda_fail(e, "timeline wait");
        const int64_t waited = (int64_t)(now_ns() - t0);
        if (timeout_ns >= 0 && waited >= timeout_ns)
            return xq4_fail(XQ4_ETIMEDOUT, "seq %llu not complete after %lld ns", (unsigned long long)seq,
                            (long long)timeout_ns);
        if (waited > 2000000) usleep(20);
    }
}

extern "C" uint64_t xq4_last_seq(const xq4_device *dev) { return dev ? dev->last_seq : 0; }

extern "C" int xq4_device_fault(xq4_device *dev, uint32_t *bits)
{
    xq4_clear_error();
    if (!dev || !bits) return xq4_fail(XQ4_EINVAL, "NULL argument");
    CK(cudaSetDevice(dev->ordinal), "cudaSetDevice");
    CK(cudaDeviceSynchronize(), "synchronize before reading the fault word");
    *bits = xq4_take_fault_gemv() | xq4_take_fault_gemm() | xq4_take_fault_w4a8() | xq4_take_fault_attn();
    return XQ4_OK;
}
