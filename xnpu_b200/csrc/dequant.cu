// dequant.cu -- whole-matrix dequantization XQ4G -> bf16 [n][k].
//
// The device form of the reference's row dequant w4u_row_bf16
// (crates/xnpu-cli/src/main.rs:3102-3125): w = RNE_bf16(q * scale) for every
// weight.  q is unpacked with the same bit trick as the GEMV/GEMM kernels
// (128 + code, exact), then one fma.rn.bf16x2 subtracts 136 (exact) and one
// multiplies by the scale (a single RNE), so the result is the reference's
// dequantized value bit for bit.
#include <cuda_runtime.h>
#include <stdint.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

// One thread per (unit, lane): rows g and g+8 x 8 K of each of the two groups.
__global__ void __launch_bounds__(256)
dequant_kernel(const uint8_t *__restrict__ pack, int n, int k, int kc_n, size_t units,
               uint16_t *__restrict__ out)
{
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t unit = gid >> 5;
    if (unit >= units) return;
    const int lane = (int)(gid & 31), g = lane >> 2, t = lane & 3;
    const int rb = (int)(unit / kc_n), kc = (int)(unit % kc_n);
    const uint8_t *up = pack + unit * XQ4G_UNIT_BYTES;
    const uint4 cw = xq4d::ldg_stream_v4(up + lane * 16);
    const uint2 sw = *reinterpret_cast<const uint2 *>(up + XQ4G_CODE_BYTES + g * 8);
    const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
    const int r0 = rb * XQ4G_ROWS + g;
#pragma unroll
    for (int G = 0; G < 2; G++) {
        const int k0 = kc * XQ4G_KCHUNK + 32 * G + 8 * t;
        if (k0 >= k) break;  // K padding (k % 64 == 32)
        const uint32_t sg = G ? sw.y : sw.x;
        const uint32_t s_lo = __byte_perm(sg, 0, 0x1010), s_hi = __byte_perm(sg, 0, 0x3232);
        uint32_t a0[4], a1[4];
        xq4d::dequant_word(words[2 * G], s_lo, s_hi, a0);
        xq4d::dequant_word(words[2 * G + 1], s_lo, s_hi, a1);
        // row g: K 0..3 (a0 regs 0, 2), K 4..7 (a1 regs 0, 2); row g+8: regs 1, 3
        if (r0 < n)
            *reinterpret_cast<uint4 *>(out + (size_t)r0 * k + k0) = make_uint4(a0[0], a0[2], a1[0], a1[2]);
        if (r0 + 8 < n)
            *reinterpret_cast<uint4 *>(out + (size_t)(r0 + 8) * k + k0) = make_uint4(a0[1], a0[3], a1[1], a1[3]);
    }
}

}  // namespace

cudaError_t xq4_launch_dequant(const uint8_t *pack, int n, int k, void *out, cudaStream_t st)
{
    const int kc = xq4g_kc(k);
    const size_t units = (size_t)xq4g_nb(n) * kc;
    const size_t threads = units * 32;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    dequant_kernel<<<blocks, 256, 0, st>>>(pack, n, k, kc, units, reinterpret_cast<uint16_t *>(out));
    return cudaGetLastError();
}
