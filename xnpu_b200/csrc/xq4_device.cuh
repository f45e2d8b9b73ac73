// xq4_device.cuh -- device-side helpers shared by the sm_100a kernels.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

namespace xq4d {

// Streamed weight bytes: read once, do not pollute L1.
__device__ __forceinline__ uint4 ldg_stream_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint32_t ldg_stream_u32(const void *p)
{
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}

// Activations: small, reused by every row block, keep them cached.
__device__ __forceinline__ uint4 ldg_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// d = (a & b) | c
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c)
{
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// d = RNE_bf16x2(a * b + c), one rounding.
__device__ __forceinline__ uint32_t fma_bf16x2(uint32_t a, uint32_t b, uint32_t c)
{
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Dequantize one XQ4G code word (8 nibbles, codes q+8) into the four bf16x2
// mma A-fragment registers.  s_lo = (s_g, s_g), s_hi = (s_g+8, s_g+8).
//   p = (w >> 4s) & 0x000F000F | 0x43004300   -> bf16 pair (128+c0, 128+c1)
//   q = p * 1 + (-136)                          exact: c - 8 in [-8, 7]
//   a = q * s + (-0)                            RNE_bf16(q * s), sign of zero kept
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t s_lo, uint32_t s_hi, uint32_t (&a)[4])
{
    const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u;
    const uint32_t kOne = 0x3F803F80u, kNeg136 = 0xC308C308u, kNegZero = 0x80008000u;
    const uint32_t p0 = lop3_and_or(w, kMask, kMagic);
    const uint32_t p1 = lop3_and_or(w >> 4, kMask, kMagic);
    const uint32_t p2 = lop3_and_or(w >> 8, kMask, kMagic);
    const uint32_t p3 = lop3_and_or(w >> 12, kMask, kMagic);
    a[0] = fma_bf16x2(fma_bf16x2(p0, kOne, kNeg136), s_lo, kNegZero);
    a[1] = fma_bf16x2(fma_bf16x2(p1, kOne, kNeg136), s_hi, kNegZero);
    a[2] = fma_bf16x2(fma_bf16x2(p2, kOne, kNeg136), s_lo, kNegZero);
    a[3] = fma_bf16x2(fma_bf16x2(p3, kOne, kNeg136), s_hi, kNegZero);
}

// D += A(16x16, row) * B(16x8, col), bf16 in, f32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace xq4d
