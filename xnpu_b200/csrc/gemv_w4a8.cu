// gemv_w4a8.cu -- W4A8 parity mode: the reference's NPU arithmetic on B200.
//
// The reference's w4gemvu kernel does not see bf16 activations: the host
// quantizes each 32-K group of x to int8 with one bf16 scale
// (w4u_quantize_x, crates/xnpu-cli/src/main.rs:2955-2986), the AIE matrix
// unit forms int8 x int4 dot products (mmul<4,16,16,int8,int4>,
// main.rs:2912-2916), every 2048-K chunk's output is written as bf16, and
// the host sums a row's chunk partials in f32 (w4u_read_c, main.rs:3066-3091).
// This file provides both halves on the GPU:
//
//  * quantize_kernel: one warp per (token, group): max |x| by shuffles,
//    d = RNE_bf16(amax / 127) (IEEE division), q = clamp(rne(x / d), +-127);
//    bit-exact with the reference's scalar path.
//  * w4a8_kernel: the decode GEMV's pipeline (persistent CTAs, bulk-copy ring
//    of XQ4G stages, 8 consumer warps, a reducer warp), with the integer
//    tensor-core path: each 32-K group is ONE mma.m16n8k32 u8 x s8 -> s32.
//    The A operand is the raw codes c = q + 8 (two ANDs and a shift per 8
//    codes), and the accumulator input is -8 * sum(q_x) of the group, so the
//    MMA returns sum(q_w * q_x) exactly.  Each group then adds
//    (s_w * d_x) * T in f32 (one fma).  A ring stage is 32 chunks = one
//    2048-K reference chunk: the reducer warp sums the 8 warps' partials,
//    rounds the chunk partial to bf16 and adds it to the row's f32 total.
//
// Operand order: lane (g, t) of the m16n8k32 fragment feeds K slots
// 4t..4t+3 and 16+4t..16+4t+3; XQ4G gives it the 8 codes at K = 8t..8t+7 of
// the group, and masking a code word yields them in the order
// (0, 2, 1, 3) within each 4.  The staged activations are stored with the
// same byte order (one prmt per word), so A and B agree slot by slot.
#include <cuda_runtime.h>
#include <atomic>
#include <cuda_bf16.h>
#include <stdint.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

constexpr int kStages = 3;
constexpr int kConsumerWarps = 8;
constexpr int kStageChunks = 32;  // 32 x 64 K = one 2048-K reference chunk
constexpr int kCpw = kStageChunks / kConsumerWarps;
constexpr int kStageBytes = kStageChunks * XQ4G_UNIT_BYTES;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps, kReducerWarp = kConsumerWarps + 1;
constexpr int kThreads = kConsumerThreads + 64;
constexpr int kRedBufs = 3;
constexpr int kMaxTok = 8;  // tokens per launch (one n8 tile)
constexpr int kMaxSmem = 227 * 1024;
constexpr int kBarBytes = ((2 * kStages + 2 * kRedBufs) * 8 + 127) & ~127;

// Shared-memory plan: [barriers | partials | group table | staged q_x | ring]
// group table: per 32-K group, 8 ints -8*sum(q_x) then 8 floats d_x (tokens 0..7)
__host__ __device__ constexpr size_t red_offset() { return kBarBytes; }
__host__ __device__ constexpr size_t tab_offset() { return red_offset() + (size_t)kRedBufs * kConsumerWarps * 128 * 4; }
__host__ __device__ constexpr size_t xq_offset(int kc_n) { return tab_offset() + (size_t)kc_n * 2 * 64; }
__host__ __device__ constexpr size_t ring_offset(int m, int kc_n)
{
    return (xq_offset(kc_n) + (size_t)m * kc_n * XQ4G_KCHUNK + 127) & ~(size_t)127;
}
__host__ __device__ constexpr size_t smem_bytes(int m, int kc_n)
{
    return ring_offset(m, kc_n) + (size_t)kStages * kStageBytes;
}

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f)
{
    const uint32_t b = __float_as_uint(f);
    return (uint16_t)((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);
}
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// One warp per (token, 32-K group): the reference's per-group quantizer.
__global__ void quantize_kernel(const uint16_t *__restrict__ x, int m, int k, int8_t *__restrict__ q,
                                uint16_t *__restrict__ d)
{
    const int lane = threadIdx.x & 31;
    const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int ng = k / 32;
    if (item >= (long long)m * ng) return;
    const int tok = (int)(item / ng), grp = (int)(item % ng);
    const size_t idx = (size_t)tok * k + (size_t)grp * 32 + lane;
    const float v = bf16_bits_to_f32(x[idx]);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (amax == 0.0f) {  // q stays 0, d stays 0
        q[idx] = 0;
        if (lane == 0) d[(size_t)tok * ng + grp] = 0;
        return;
    }
    const uint16_t db = f32_to_bf16_rne(__fdiv_rn(amax, 127.0f));
    const float r = rintf(__fdiv_rn(v, bf16_bits_to_f32(db)));  // round half to even
    q[idx] = (int8_t)fminf(fmaxf(r, -127.0f), 127.0f);
    if (lane == 0) d[(size_t)tok * ng + grp] = db;
}

__global__ void __launch_bounds__(kThreads, 2)
w4a8_kernel(const uint8_t *__restrict__ pack, int n, int k, int nb, int kc_n, const int8_t *__restrict__ qx,
            const uint16_t *__restrict__ dx, int m, void *__restrict__ y, int out_f32)
{
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kStages;
    uint64_t *red_full = empty + kStages;
    uint64_t *red_free = red_full + kRedBufs;
    float *red = reinterpret_cast<float *>(smem + red_offset());       // [buf][warp][tok][row]
    uint32_t *tab = reinterpret_cast<uint32_t *>(smem + tab_offset());  // [group][16]
    uint8_t *xq = smem + xq_offset(kc_n);                               // [m][kp] permuted
    uint8_t *ring = smem + ring_offset(m, kc_n);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int rb0 = (int)((long long)cta * nb / G), rb1 = (int)((long long)(cta + 1) * nb / G);
    const int spr = (kc_n + kStageChunks - 1) / kStageChunks;  // stages (2048-K chunks) per row block
    const int total = (rb1 - rb0) * spr;
    const int kp = kc_n * XQ4G_KCHUNK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            xq4d::mbar_init(&full[s], 1);
            xq4d::mbar_init(&empty[s], kConsumerWarps);
        }
        for (int b = 0; b < kRedBufs; b++) {
            xq4d::mbar_init(&red_full[b], kConsumerWarps);
            xq4d::mbar_init(&red_free[b], 1);
        }
        xq4d::fence_barrier_init();
    }
    __syncthreads();
    xq4d::grid_dep_launch();

    if (warp == kProducerWarp) {  // ------------------------------ producer
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

    if (warp == kReducerWarp) {  // ------------------------------ reducer
        // Stage i's 8 partials (one 2048-K chunk of one row block): sum in
        // warp order, round the chunk partial to bf16, add it to the row's
        // f32 total; write the row block after its last chunk.
        xq4d::grid_dep_wait();
        float run[4] = {0.f, 0.f, 0.f, 0.f};  // outputs o = lane + 32 j (o = tok * 16 + row)
        int st = 0;
        for (int i = 0; i < total; i++) {
            const int buf = i % kRedBufs;
            const uint32_t use = (uint32_t)(i / kRedBufs);
            if (!xq4d::mbar_wait(&red_full[buf], use & 1)) {
                atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                return;
            }
            const float *rd = red + (size_t)buf * kConsumerWarps * 128;
            const int rb = rb0 + i / spr;
            const bool last = st == spr - 1;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int o = lane + 32 * j;
                if (o < m * 16) {
                    float sum = 0.f;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; w++) sum += rd[(size_t)w * 128 + o];
                    const float part = bf16_bits_to_f32(f32_to_bf16_rne(sum));
                    run[j] = st == 0 ? part : run[j] + part;
                    if (last) {
                        const int tok = o >> 4, row = rb * XQ4G_ROWS + (o & 15);
                        if (row < n) {
                            if (out_f32)
                                reinterpret_cast<float *>(y)[(size_t)tok * n + row] = run[j];
                            else
                                reinterpret_cast<uint16_t *>(y)[(size_t)tok * n + row] = f32_to_bf16_rne(run[j]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(&red_free[buf]);
            st = last ? 0 : st + 1;
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    xq4d::grid_dep_wait();
    {
        // Stage q_x (byte order 0,2,1,3 within each 4) and the group table.
        const int runs = k / 16, kp_runs = kp / 16;
        for (int r = threadIdx.x; r < m * kp_runs; r += kConsumerThreads) {
            const int tok = r / kp_runs, rr = r - tok * kp_runs;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (rr < runs) v = xq4d::ldg_v4(qx + (size_t)tok * k + 16 * rr);
            v.x = __byte_perm(v.x, 0, 0x3120);
            v.y = __byte_perm(v.y, 0, 0x3120);
            v.z = __byte_perm(v.z, 0, 0x3120);
            v.w = __byte_perm(v.w, 0, 0x3120);
            *reinterpret_cast<uint4 *>(xq + (size_t)tok * kp + 16 * rr) = v;
        }
        xq4d::named_bar_sync(1, kConsumerThreads);
        const int ngp = kp / 32, ng = k / 32;
        for (int e = threadIdx.x; e < ngp * kMaxTok; e += kConsumerThreads) {
            const int grp = e / kMaxTok, tok = e - grp * kMaxTok;
            int sum = 0;
            float dv = 0.f;
            if (tok < m && grp < ng) {
                const uint32_t *p = reinterpret_cast<const uint32_t *>(xq + (size_t)tok * kp + 32 * grp);
#pragma unroll
                for (int w = 0; w < 8; w++) sum = __dp4a((int)p[w], 0x01010101, sum);
                dv = bf16_bits_to_f32(dx[(size_t)tok * ng + grp]);
            }
            tab[grp * 16 + tok] = (uint32_t)(-8 * sum);
            tab[grp * 16 + 8 + tok] = __float_as_uint(dv);
        }
        xq4d::named_bar_sync(1, kConsumerThreads);
    }

    const int g = lane >> 2, t = lane & 3;
    const uint32_t xrow = xq4d::smem_u32(xq + (size_t)(g < m ? g : 0) * kp);  // B column g = token g
    const uint32_t tab_s = xq4d::smem_u32(tab), ring_s = xq4d::smem_u32(ring);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int slot = 0, kc0 = 0;
    uint32_t phase = 0;
    for (int i = 0; i < total; i++) {
        const uint32_t stage = ring_s + (uint32_t)slot * kStageBytes;
        if (!xq4d::mbar_wait(&full[slot], phase)) {
            atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
            return;
        }
#pragma unroll
        for (int c = 0; c < kCpw; c++) {
            const int cl = warp + c * kConsumerWarps;  // chunk within the stage
            const int kc = kc0 + cl;
            if (kc < kc_n) {
                const uint32_t up = stage + cl * XQ4G_UNIT_BYTES;
                const uint4 cw = xq4d::lds_v4(up + lane * 16);
                const uint2 sw = xq4d::lds_v2(up + XQ4G_CODE_BYTES + g * 8);
                const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
                for (int G2 = 0; G2 < 2; G2++) {
                    const int grp = kc * 2 + G2;
                    const uint2 b = xq4d::lds_v2(xrow + grp * 32 + 8 * t);
                    const uint2 cxp = xq4d::lds_v2(tab_s + (grp * 16 + 2 * t) * 4);
                    const uint2 ddp = xq4d::lds_v2(tab_s + (grp * 16 + 8 + 2 * t) * 4);
                    const uint32_t w0 = words[2 * G2], w1 = words[2 * G2 + 1];
                    const uint32_t a[4] = {w0 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu,
                                           (w1 >> 4) & 0x0F0F0F0Fu};
                    int T[4];
                    xq4d::mma_u8s8_16832(T, a, b.x, b.y, (int)cxp.x, (int)cxp.y);
                    const uint32_t sg = G2 ? sw.y : sw.x;
                    const float s_lo = __uint_as_float(sg << 16), s_hi = __uint_as_float(sg & 0xFFFF0000u);
                    const float d0 = __uint_as_float(ddp.x), d1 = __uint_as_float(ddp.y);
                    acc[0] = fmaf(s_lo * d0, (float)T[0], acc[0]);
                    acc[1] = fmaf(s_lo * d1, (float)T[1], acc[1]);
                    acc[2] = fmaf(s_hi * d0, (float)T[2], acc[2]);
                    acc[3] = fmaf(s_hi * d1, (float)T[3], acc[3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) xq4d::mbar_arrive(&empty[slot]);
        if (++slot == kStages) {
            slot = 0;
            phase ^= 1;
        }
        // stage done = one 2048-K chunk of the row block: hand the partial on
        const int buf = i % kRedBufs;
        const uint32_t use = (uint32_t)(i / kRedBufs);
        if (use > 0 && !xq4d::mbar_wait(&red_free[buf], (use - 1) & 1)) {
            atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
            return;
        }
        float *r = red + (size_t)buf * kConsumerWarps * 128 + (size_t)warp * 128;  // [tok][row]
        r[(2 * t) * 16 + g] = acc[0];
        r[(2 * t + 1) * 16 + g] = acc[1];
        r[(2 * t) * 16 + g + 8] = acc[2];
        r[(2 * t + 1) * 16 + g + 8] = acc[3];
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        __syncwarp();
        if (lane == 0) xq4d::mbar_arrive(&red_full[buf]);
        kc0 += kStageChunks;
        if (kc0 >= kc_n) kc0 = 0;
    }
}

int sm_count()
{
    static std::atomic<int> cache[64];  // zero-initialised; atomics: first launches may race across threads
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

}  // namespace

cudaError_t xq4_launch_quantize_x(const void *x, int m, int k, void *q, void *d, cudaStream_t st)
{
    const long long items = (long long)m * (k / 32);
    const int warps_per_block = 8;
    const long long blocks = (items + warps_per_block - 1) / warps_per_block;
    if (blocks <= 0) return cudaSuccess;
    quantize_kernel<<<(unsigned)blocks, warps_per_block * 32, 0, st>>>(
        reinterpret_cast<const uint16_t *>(x), m, k, reinterpret_cast<int8_t *>(q), reinterpret_cast<uint16_t *>(d));
    return cudaGetLastError();
}

size_t xq4_w4a8_smem_bytes(int m, int k) { return smem_bytes(m < kMaxTok ? m : kMaxTok, xq4g_kc(k)); }

// m tokens in slices of up to 8 (one n8 MMA tile per slice; fewer when the
// staged activations of 8 would not fit in shared memory).
cudaError_t xq4_launch_w4a8(const uint8_t *pack, int n, int k, const void *qx, const void *dx, int m, void *y,
                            int out_f32, cudaStream_t st)
{
    static std::atomic<bool> attr_set[64];  // zero-initialised; atomics: first launches may race across threads
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(w4a8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int nb = xq4g_nb(n), kc = xq4g_kc(k);
    const size_t ysz = out_f32 ? 4 : 2;
    for (int t0 = 0, mt = 0; t0 < m; t0 += mt) {
        mt = m - t0 < kMaxTok ? m - t0 : kMaxTok;
        while (mt > 1 && smem_bytes(mt, kc) > (size_t)kMaxSmem) mt--;  // staged q_x must fit
        const size_t smem = smem_bytes(mt, kc);
        if (smem > (size_t)kMaxSmem) return cudaErrorInvalidValue;
        cudaLaunchConfig_t cfg = {};
        const int cap = sm_count() * (2 * (smem + 1024) <= 228 * 1024 ? 2 : 1);
        cfg.gridDim = dim3(nb < cap ? nb : cap);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(
            &cfg, w4a8_kernel, pack, n, k, nb, kc, reinterpret_cast<const int8_t *>(qx) + (size_t)t0 * k,
            reinterpret_cast<const uint16_t *>(dx) + (size_t)t0 * (k / 32), mt,
            reinterpret_cast<void *>(reinterpret_cast<char *>(y) + (size_t)t0 * n * ysz), out_f32);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Read and clear this unit's fault word on the current device.
unsigned int xq4_take_fault_w4a8()
{
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_xq4_fault, sizeof v) != cudaSuccess) return ~0u;
    cudaMemcpyToSymbol(g_xq4_fault, &zero, sizeof zero);
    return v;
}
