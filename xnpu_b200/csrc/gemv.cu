// gemv.cu -- K1: decode GEMV for m = 1..16 tokens over XQ4G int4 weights.
//
// y[m][n] = x[m][k] . dequant(W)^T with dequant w = RNE_bf16(q * scale)
// (crates/xnpu-cli/src/main.rs:3097-3125) and f32 accumulation
// (main.rs:2287-2296).  This is the B200 replacement for the reference's
// w4gemv2 / w4gemvu AIE kernels (invoked at main.rs:2171-2448, :3288-3898).
//
// Design (HBM-bound: ~0.56 B of weights per weight, 2*m flops per weight):
//  * One CTA per 16-row block, 8 warps split the 64-K chunks of the row
//    block round-robin; each lane streams one 16-byte code word per chunk
//    with ld.global.nc.L1::no_allocate (coalesced: a warp reads the unit's
//    512 contiguous code bytes) plus the 4-byte scale pair it needs.
//  * The 16 bytes are exactly the lane's mma.m16n8k16 A fragments for the
//    chunk's 4 K steps (xq4_layout.h).  Dequant per bf16x2 pair: one lop3
//    (nibble | 0x4300 -> 128+code), fma.rn.bf16x2 (-136 -> q, exact) and
//    fma.rn.bf16x2 by the broadcast scale (-> RNE_bf16(q*s), exact).
//  * The tensor core does the dot products (8 tokens per n8 tile; f32
//    accumulate), so CUDA-core issue is spent only on the unpack.
//  * Per-warp partial sums are reduced through shared memory in fixed warp
//    order (deterministic) and written once, RNE to bf16 or as f32.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kUnroll = 4;

template <int NT>
__global__ void __launch_bounds__(kWarps * 32)
gemv_kernel(const uint8_t *__restrict__ pack, int n, int k, int kc_n,
            const uint16_t *__restrict__ x, int m, void *__restrict__ y, int out_f32)
{
    const int rb = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *base = pack + (size_t)rb * kc_n * XQ4G_UNIT_BYTES;

    const uint16_t *xr[NT];
    bool tv[NT];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        int tok = g + 8 * nt;
        tv[nt] = tok < m;
        xr[nt] = x + (size_t)(tv[nt] ? tok : 0) * k;
    }
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;

    for (int c0 = warp; c0 < kc_n; c0 += kWarps * kUnroll) {
        uint4 cw[kUnroll];
        uint32_t sw[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int c = c0 + u * kWarps;
            if (c < kc_n) {
                const uint8_t *up = base + (size_t)c * XQ4G_UNIT_BYTES;
                cw[u] = xq4d::ldg_stream_v4(up + lane * 16);
                sw[u] = xq4d::ldg_stream_u32(up + XQ4G_CODE_BYTES + g * 8 + (t >> 1) * 4);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int c = c0 + u * kWarps;
            if (c < kc_n) {
                const int kbase = c * XQ4G_KCHUNK + 16 * t;
                uint4 xf[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    if (tv[nt] && kbase < k) {
                        xf[nt][0] = xq4d::ldg_v4(xr[nt] + kbase);
                        xf[nt][1] = xq4d::ldg_v4(xr[nt] + kbase + 8);
                    } else {
                        xf[nt][0] = make_uint4(0, 0, 0, 0);
                        xf[nt][1] = make_uint4(0, 0, 0, 0);
                    }
                }
                const uint32_t s_lo = __byte_perm(sw[u], 0, 0x1010);
                const uint32_t s_hi = __byte_perm(sw[u], 0, 0x3232);
                const uint32_t words[4] = {cw[u].x, cw[u].y, cw[u].z, cw[u].w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint32_t a[4];
                    xq4d::dequant_word(words[j], s_lo, s_hi, a);
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        const uint32_t *xw0 = reinterpret_cast<const uint32_t *>(&xf[nt][0]);
                        const uint32_t *xw1 = reinterpret_cast<const uint32_t *>(&xf[nt][1]);
                        const uint32_t b0 = j < 2 ? xw0[2 * j] : xw1[2 * j - 4];
                        const uint32_t b1 = j < 2 ? xw0[2 * j + 1] : xw1[2 * j - 3];
                        xq4d::mma_bf16_16816(acc[nt], a, b0, b1);
                    }
                }
            }
        }
    }

    // Cross-warp reduction: red[warp][nt][row*8 + tok]
    __shared__ float red[kWarps][NT][128];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        red[warp][nt][g * 8 + 2 * t] = acc[nt][0];
        red[warp][nt][g * 8 + 2 * t + 1] = acc[nt][1];
        red[warp][nt][(g + 8) * 8 + 2 * t] = acc[nt][2];
        red[warp][nt][(g + 8) * 8 + 2 * t + 1] = acc[nt][3];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < NT * 128; idx += kWarps * 32) {
        const int nt = idx >> 7, tl = (idx & 127) >> 4, r = idx & 15;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) s += red[w][nt][r * 8 + tl];
        const int tok = nt * 8 + tl, row = rb * XQ4G_ROWS + r;
        if (tok < m && row < n) {
            if (out_f32)
                reinterpret_cast<float *>(y)[(size_t)tok * n + row] = s;
            else
                reinterpret_cast<__nv_bfloat16 *>(y)[(size_t)tok * n + row] = __float2bfloat16_rn(s);
        }
    }
}

}  // namespace

// m in 1..16 per launch; larger m is split into 16-token slices.
cudaError_t xq4_launch_gemv(const uint8_t *pack, int n, int k, const void *x, int m, void *y,
                            int out_f32, cudaStream_t st)
{
    const int nb = xq4g_nb(n), kc = xq4g_kc(k);
    const size_t ysz = out_f32 ? 4 : 2;
    for (int t0 = 0; t0 < m; t0 += 16) {
        const int mt = m - t0 < 16 ? m - t0 : 16;
        const uint16_t *xs = reinterpret_cast<const uint16_t *>(x) + (size_t)t0 * k;
        void *ys = reinterpret_cast<char *>(y) + (size_t)t0 * n * ysz;
        if (mt <= 8)
            gemv_kernel<1><<<nb, kWarps * 32, 0, st>>>(pack, n, k, kc, xs, mt, ys, out_f32);
        else
            gemv_kernel<2><<<nb, kWarps * 32, 0, st>>>(pack, n, k, kc, xs, mt, ys, out_f32);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}
