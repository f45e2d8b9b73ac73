// dequant.cu -- whole-matrix dequantization XQ4G -> bf16 [n][k].
//
// The device form of the reference's row dequant w4u_row_bf16
// (crates/xnpu-cli/src/main.rs:3102-3125): w = RNE_bf16(q * scale) for every
// weight.  It uses the same unpack as the GEMV/GEMM kernels (dequant_word), so
// a bit-exact match of this kernel against the oracle proves the kernels'
// operand values bit-exact too.
#include <cuda_runtime.h>
#include <stdint.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

// One thread per (unit, lane): 2 rows x 16 K.
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
    const uint32_t sw = xq4d::ldg_stream_u32(up + XQ4G_CODE_BYTES + g * 8 + (t >> 1) * 4);
    const uint32_t s_lo = __byte_perm(sw, 0, 0x1010), s_hi = __byte_perm(sw, 0, 0x3232);
    const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
    uint32_t lo[8], hi[8];  // row g / row g+8, 16 consecutive K as 8 bf16x2
#pragma unroll
    for (int j = 0; j < 4; j++) {
        uint32_t a[4];
        xq4d::dequant_word(words[j], s_lo, s_hi, a);
        lo[2 * j] = a[0];
        lo[2 * j + 1] = a[2];
        hi[2 * j] = a[1];
        hi[2 * j + 1] = a[3];
    }
    const int k0 = kc * XQ4G_KCHUNK + 16 * t;
    if (k0 >= k) return;  // K padding (k % 64 == 32)
    const int r0 = rb * XQ4G_ROWS + g;
    if (r0 < n) {
        uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)r0 * k + k0);
        dst[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        dst[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
    }
    if (r0 + 8 < n) {
        uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)(r0 + 8) * k + k0);
        dst[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        dst[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
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
