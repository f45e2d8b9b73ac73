// gemv.cu -- K1: decode GEMV for m = 1..16 tokens over XQ4G int4 weights.
//
// y[m][n] = sum_k (q[n][k] * s[n][k/32]) * x[m][k], the reference's GEMV
// (crates/xnpu-cli/src/main.rs:2287-2296: w = nibble * scale in f32, no
// intermediate rounding, f32 accumulation, one final rounding).  This is the
// B200 replacement for the reference's w4gemv2 / w4gemvu AIE kernels (invoked
// at main.rs:2171-2448, :3288-3898).
//
// Design (HBM-bound: 0.5625 B of weights per weight, 2*m flops per weight):
//  * Persistent grid, one CTA per SM.  CTA c owns the contiguous row blocks
//    [c*nb/G, (c+1)*nb/G); in the XQ4G layout that is ONE contiguous byte
//    range, streamed front to back.
//  * A producer thread copies the range into an 8-stage shared-memory ring
//    with cp.async.bulk (the bulk-copy engine, no multicast); one stage = 32
//    consecutive 64-K chunks (18 KB) of one row block, completion counted on
//    a per-stage mbarrier.  147 KB in flight per SM keeps HBM busy (measured
//    6.2 TB/s for the copy stream alone).
//  * 16 consumer warps take two chunks each per stage (two independent
//    instruction streams per warp).  A lane's 16 code bytes
//    are exactly its mma.m16n8k16 A fragments for the chunk's 4 K steps, and
//    each K step lies in one 32-K scale group (xq4_layout.h).  The unpack is
//    one lop3 per bf16x2 pair (p = 128 + code, exact) and one fma.rn.bf16x2
//    (q = p - 136, exact).  The tensor core forms T = sum q*x over the
//    group's 32 K (two K steps, f32) and the group adds s * T in f32.  In
//    exact arithmetic that is sum (q*s)*x, the reference's formula with the
//    weight never rounded (the rounded RNE_bf16(q*s) is the dequant op's
//    output, dequant.cu); only the f32 summation order differs.
//  * The activation slice of a chunk is loaded before the stage wait.
//  * At the end of a row block the per-warp partials are summed through
//    shared memory in fixed warp order (deterministic) and written once.
//  * Programmatic dependent launch: the producer starts streaming weights
//    before griddepcontrol.wait; only the consumers (which read x and write
//    y) wait for the preceding kernel.
//  * Every mbarrier wait is bounded; a wait that runs out sets g_xq4_fault and
//    the kernel returns.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

#ifndef XQ4_GEMV_CPW
#define XQ4_GEMV_CPW 2
#endif
#ifndef XQ4_GEMV_STAGES
#define XQ4_GEMV_STAGES 8
#endif
constexpr int kConsumerWarps = 16;
constexpr int kCpw = XQ4_GEMV_CPW;                    // chunks per consumer warp per stage
constexpr int kStageChunks = kConsumerWarps * kCpw;
constexpr int kStages = XQ4_GEMV_STAGES;
constexpr int kStageBytes = kStageChunks * XQ4G_UNIT_BYTES;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kBarBytes = ((2 * kStages + 2) * 8 + 127) & ~127;  // full/empty/reduce mbarriers, padded
static_assert(kBarBytes >= (2 * kStages + 2) * 8, "barrier region too small");
constexpr int kMaxSmem = 227 * 1024;

// Shared-memory plan: [barriers | partials x2 | ring]
template <int NT>
__host__ __device__ constexpr size_t red_bytes() { return 2 * (size_t)kConsumerWarps * NT * 128 * 4; }
template <int NT>
__host__ __device__ constexpr size_t ring_offset() { return (kBarBytes + red_bytes<NT>() + 127) & ~(size_t)127; }
template <int NT>
__host__ __device__ constexpr size_t smem_bytes() { return ring_offset<NT>() + (size_t)kStages * kStageBytes; }

// One ring stage for one consumer warp: its chunks kc0 + warp + c*16.  The
// activation runs are loaded before the stage wait so their latency overlaps
// it.  SAFE handles a partial stage (chunks past kc_n) and a K tail that is
// not a whole chunk (k % 64 == 32); the fast path has no per-chunk tests.
template <int NT, bool SAFE>
__device__ __forceinline__ bool consume_stage(const uint8_t *stage, uint64_t *full, uint32_t phase, int kc0,
                                              int kc_n, int k, const uint16_t *const (&xr)[NT], int warp,
                                              int lane, float (&acc)[NT][4])
{
    const int g = lane >> 2, t = lane & 3;
    uint4 xf[kCpw][NT][2];  // 8 K of group 0 and 8 K of group 1, per chunk
#pragma unroll
    for (int c = 0; c < kCpw; c++) {
        const int kc = kc0 + warp + c * kConsumerWarps;
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int G2 = 0; G2 < 2; G2++) {
                const int kb = kc * XQ4G_KCHUNK + 32 * G2 + 8 * t;
                if (!SAFE || (kc < kc_n && kb < k))
                    xf[c][nt][G2] = xq4d::ldg_v4(xr[nt] + kb);
                else
                    xf[c][nt][G2] = make_uint4(0, 0, 0, 0);
            }
    }
    if (!xq4d::mbar_wait(full, phase)) return false;
    uint4 cw[kCpw];
    uint2 sw[kCpw];
#pragma unroll
    for (int c = 0; c < kCpw; c++) {
        const int cl = warp + c * kConsumerWarps;  // chunk within the stage
        const uint8_t *up = stage + cl * XQ4G_UNIT_BYTES;
        if (!SAFE || kc0 + cl < kc_n) {
            cw[c] = *reinterpret_cast<const uint4 *>(up + lane * 16);
            sw[c] = *reinterpret_cast<const uint2 *>(up + XQ4G_CODE_BYTES + g * 8);
        } else {
            cw[c] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // q = 0
            sw[c] = make_uint2(0, 0);
        }
    }
#pragma unroll
    for (int c = 0; c < kCpw; c++) {
        const uint32_t words[4] = {cw[c].x, cw[c].y, cw[c].z, cw[c].w};
#pragma unroll
        for (int G2 = 0; G2 < 2; G2++) {
            const uint32_t sg = G2 ? sw[c].y : sw[c].x;
            const float s_lo = __uint_as_float(sg << 16);          // row g
            const float s_hi = __uint_as_float(sg & 0xFFFF0000u);  // row g+8
            uint32_t a0[4], a1[4];
            xq4d::unpack_word_q(words[2 * G2], a0);
            xq4d::unpack_word_q(words[2 * G2 + 1], a1);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float tacc[4];
                xq4d::mma_bf16_16816_z(tacc, a0, xf[c][nt][G2].x, xf[c][nt][G2].y);
                xq4d::mma_bf16_16816(tacc, a1, xf[c][nt][G2].z, xf[c][nt][G2].w);
                acc[nt][0] = fmaf(s_lo, tacc[0], acc[nt][0]);
                acc[nt][1] = fmaf(s_lo, tacc[1], acc[nt][1]);
                acc[nt][2] = fmaf(s_hi, tacc[2], acc[nt][2]);
                acc[nt][3] = fmaf(s_hi, tacc[3], acc[nt][3]);
            }
        }
    }
    return true;
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
gemv_kernel(const uint8_t *__restrict__ pack, int n, int k, int nb, int kc_n,
            const uint16_t *__restrict__ x, int m, void *__restrict__ y, int out_f32)
{
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kStages;
    uint64_t *red_full = empty + kStages;  // [2], one per partial buffer
    float *red = reinterpret_cast<float *>(smem + kBarBytes);
    uint8_t *ring = smem + ring_offset<NT>();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int rb0 = (int)((long long)cta * nb / G), rb1 = (int)((long long)(cta + 1) * nb / G);
    const int spr = (kc_n + kStageChunks - 1) / kStageChunks;  // stages per row block
    const int total = (rb1 - rb0) * spr;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            xq4d::mbar_init(&full[s], 1);
            xq4d::mbar_init(&empty[s], kConsumerWarps);
        }
        xq4d::mbar_init(&red_full[0], kConsumerWarps);
        xq4d::mbar_init(&red_full[1], kConsumerWarps);
        xq4d::fence_barrier_init();
    }
    __syncthreads();
    xq4d::grid_dep_launch();

    if (warp == kConsumerWarps) {  // ------------------------------ producer
        if (lane == 0) {
            int slot = 0, rb = rb0, kc0 = 0;
            uint32_t phase = 0;
            for (int i = 0; i < total; i++) {
                if (i >= kStages && !xq4d::mbar_wait(&empty[slot], phase ^ 1)) {
                    atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_EMPTY);
                    break;
                }
                const int cnt = min(kStageChunks, kc_n - kc0);
                const uint32_t bytes = (uint32_t)cnt * XQ4G_UNIT_BYTES;
                xq4d::mbar_arrive_expect_tx(&full[slot], bytes);
                xq4d::bulk_g2s(ring + (size_t)slot * kStageBytes,
                               pack + ((size_t)rb * kc_n + kc0) * XQ4G_UNIT_BYTES, bytes, &full[slot]);
                if (++slot == kStages) {
                    slot = 0;
                    phase ^= 1;
                }
                kc0 += kStageChunks;
                if (kc0 >= kc_n) {
                    kc0 = 0;
                    rb++;
                }
            }
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    xq4d::grid_dep_wait();  // x is written, y may be read, by the neighbouring kernels

    const int g = lane >> 2, t = lane & 3;
    // B column g of the mma is token g (+8*nt).  A column past m only feeds
    // output columns that are never written, so those lanes read token 0's
    // row instead of being predicated off.
    const uint16_t *xr[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int tok = g + 8 * nt;
        xr[nt] = x + (size_t)(tok < m ? tok : 0) * k;
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;

    int slot = 0, rbl = 0, kc0 = 0;
    uint32_t phase = 0;
    const bool k_whole = (k % XQ4G_KCHUNK) == 0;
    for (int i = 0; i < total; i++) {
        const uint8_t *stage = ring + (size_t)slot * kStageBytes;
        const bool ok = (k_whole && kc0 + kStageChunks <= kc_n)
                            ? consume_stage<NT, false>(stage, &full[slot], phase, kc0, kc_n, k, xr, warp, lane, acc)
                            : consume_stage<NT, true>(stage, &full[slot], phase, kc0, kc_n, k, xr, warp, lane, acc);
        if (!ok) {
            atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
            return;
        }
        __syncwarp();
        if (lane == 0) xq4d::mbar_arrive(&empty[slot]);
        if (++slot == kStages) {
            slot = 0;
            phase ^= 1;
        }
        kc0 += kStageChunks;

        if (kc0 >= kc_n) {  // ------------------------------ row block complete
            kc0 = 0;
            const int buf = rbl & 1;
            float *rd = red + (size_t)buf * kConsumerWarps * NT * 128;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float *r = rd + ((size_t)warp * NT + nt) * 128;
                r[g * 8 + 2 * t] = acc[nt][0];
                r[g * 8 + 2 * t + 1] = acc[nt][1];
                r[(g + 8) * 8 + 2 * t] = acc[nt][2];
                r[(g + 8) * 8 + 2 * t + 1] = acc[nt][3];
                acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
            }
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(&red_full[buf]);
            if (!xq4d::mbar_wait(&red_full[buf], (uint32_t)(rbl >> 1) & 1)) {
                atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                return;
            }
            const int rb = rb0 + rbl;
            for (int idx = threadIdx.x; idx < NT * 128; idx += kConsumerThreads) {
                const int nt = idx >> 7, tl = (idx & 127) >> 4, r = idx & 15;
                float s = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; w++) s += rd[((size_t)w * NT + nt) * 128 + r * 8 + tl];
                const int tok = nt * 8 + tl, row = rb * XQ4G_ROWS + r;
                if (tok < m && row < n) {
                    if (out_f32)
                        reinterpret_cast<float *>(y)[(size_t)tok * n + row] = s;
                    else
                        reinterpret_cast<__nv_bfloat16 *>(y)[(size_t)tok * n + row] = __float2bfloat16_rn(s);
                }
            }
            rbl++;
        }
    }
}

int sm_count_of_current_device()
{
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = v > 0 ? v : 148;
    }
    return cache[dev];
}

template <int NT>
cudaError_t launch_one(const uint8_t *pack, int n, int k, const uint16_t *x, int m, void *y, int out_f32,
                       cudaStream_t st)
{
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem_bytes<NT>());
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int nb = xq4g_nb(n), kc = xq4g_kc(k);
    const size_t smem = smem_bytes<NT>();
    static_assert(smem_bytes<2>() <= (size_t)kMaxSmem, "shared memory plan too large");
    const int sms = sm_count_of_current_device();
    const int grid = nb < sms ? nb : sms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
#ifdef XQ4_GEMV_NO_PDL
    cfg.numAttrs = 0;
#else
    cfg.numAttrs = 1;
#endif
    return cudaLaunchKernelEx(&cfg, gemv_kernel<NT>, pack, n, k, nb, kc, x, m, y, out_f32);
}

}  // namespace

// m in 1..16 per launch; larger m is split into 16-token slices.
cudaError_t xq4_launch_gemv(const uint8_t *pack, int n, int k, const void *x, int m, void *y,
                            int out_f32, cudaStream_t st)
{
    const size_t ysz = out_f32 ? 4 : 2;
    for (int t0 = 0; t0 < m; t0 += 16) {
        const int mt = m - t0 < 16 ? m - t0 : 16;
        const uint16_t *xs = reinterpret_cast<const uint16_t *>(x) + (size_t)t0 * k;
        void *ys = reinterpret_cast<char *>(y) + (size_t)t0 * n * ysz;
        cudaError_t e = mt <= 8 ? launch_one<1>(reinterpret_cast<const uint8_t *>(pack), n, k, xs, mt, ys,
                                                out_f32, st)
                                : launch_one<2>(reinterpret_cast<const uint8_t *>(pack), n, k, xs, mt, ys,
                                                out_f32, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Read and clear this unit's fault word on the current device.
unsigned int xq4_take_fault_gemv()
{
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_xq4_fault, sizeof v) != cudaSuccess) return ~0u;
    cudaMemcpyToSymbol(g_xq4_fault, &zero, sizeof zero);
    return v;
}
