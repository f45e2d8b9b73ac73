// xq4_device.cuh -- device-side helpers shared by the sm_100a kernels.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

// Set by a kernel whose bounded wait ran out (a pipeline that stopped making
// progress); the kernel returns instead of spinning forever.  One copy per
// translation unit (no relocatable device code); each unit that launches
// kernels with bounded waits exposes a host reader (xq4_take_fault_*), and
// xq4_device_fault() collects them.
static __device__ unsigned int g_xq4_fault;

#define XQ4_FAULT_GEMV_FULL 0x1u
#define XQ4_FAULT_GEMV_EMPTY 0x2u
#define XQ4_FAULT_GEMM_WAIT 0x4u
#define XQ4_FAULT_PEER_WAIT 0x8u  // a peer GPU's output words did not arrive in time
#define XQ4_FAULT_CHAIN_WAIT 0x10u  // a chain op's wait for the previous op ran out
#define XQ4_FAULT_ATTN_POS 0x20u    // decode attention given a position outside its cache (nothing written)

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
__device__ __forceinline__ float4 ldg_f4(const float4 *p)
{
    float4 r;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}
// L2-coherent 16-byte load (bypasses L1): for data another CTA of the same
// kernel may have written.
__device__ __forceinline__ uint4 ldcg_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
__device__ __forceinline__ uint16_t ldcg_u16(const uint16_t *p)
{
    uint16_t v;
    asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned *p, unsigned v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint2 ldg_v2(const void *p)
{
    uint2 r;
    asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
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

// Unpack one XQ4G code word into the four bf16x2 mma A-fragment registers
// holding p = 128 + code = q + 136, exactly (no arithmetic, 7 instructions).
__device__ __forceinline__ void unpack_word_p(uint32_t w, uint32_t (&a)[4])
{
    const uint32_t kMask = 0x000F000Fu, kMagic = 0x43004300u;
#ifdef XQ4_SHIFT_ON_FMA_PIPE
    // w >> 4s as the high word of w * 2^(32-4s): an integer multiply, which
    // leaves the integer ALU pipe to the lop3s
    a[0] = lop3_and_or(w, kMask, kMagic);
    a[1] = lop3_and_or(__umulhi(w, 1u << 28), kMask, kMagic);
    a[2] = lop3_and_or(__umulhi(w, 1u << 24), kMask, kMagic);
    a[3] = lop3_and_or(__umulhi(w, 1u << 20), kMask, kMagic);
#else
    a[0] = lop3_and_or(w, kMask, kMagic);
    a[1] = lop3_and_or(w >> 4, kMask, kMagic);
    a[2] = lop3_and_or(w >> 8, kMask, kMagic);
    a[3] = lop3_and_or(w >> 12, kMask, kMagic);
#endif
}

// Unpack one XQ4G code word into the four bf16x2 mma A-fragment registers
// holding q = code - 8 in [-8, 7], exactly: p = 128 + code, then p - 136.
__device__ __forceinline__ void unpack_word_q(uint32_t w, uint32_t (&a)[4])
{
    const uint32_t kOne = 0x3F803F80u, kNeg136 = 0xC308C308u;
    unpack_word_p(w, a);
#pragma unroll
    for (int i = 0; i < 4; i++) a[i] = fma_bf16x2(a[i], kOne, kNeg136);
}

// d = RNE_f16x2(a * b + c), one rounding.
__device__ __forceinline__ uint32_t fma_f16x2(uint32_t a, uint32_t b, uint32_t c)
{
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Unpack one XQ4G code word into the four f16x2 mma A-fragment registers.
// fp16 has 10 mantissa bits, so the nibbles at bits 0-3 and 4-7 of each half
// both sit inside the mantissa under the 1024 magic exponent:
//   (w & 0x000F000F) | 0x6400 -> 1024 + c        - 1032 -> q      (rows g)
//   (w & 0x00F000F0) | 0x6400 -> 1024 + 16c      - 1152 -> 16 q   (rows g+8)
// and the same on w >> 8 for nibbles 2/3.  One shift per word instead of
// three; every value is exact.  Registers 1 and 3 (rows g+8 of the fragment)
// carry the factor 16, which the caller folds into those rows' scale.
__device__ __forceinline__ void unpack_word_h16(uint32_t w, uint32_t (&a)[4])
{
    const uint32_t kMagic = 0x64006400u, kOne = 0x3C003C00u;
    const uint32_t kNeg1032 = 0xE408E408u, kNeg1152 = 0xE480E480u;
    const uint32_t w8 = w >> 8;
    a[0] = fma_f16x2(lop3_and_or(w, 0x000F000Fu, kMagic), kOne, kNeg1032);
    a[1] = fma_f16x2(lop3_and_or(w, 0x00F000F0u, kMagic), kOne, kNeg1152);
    a[2] = fma_f16x2(lop3_and_or(w8, 0x000F000Fu, kMagic), kOne, kNeg1032);
    a[3] = fma_f16x2(lop3_and_or(w8, 0x00F000F0u, kMagic), kOne, kNeg1152);
}

// Unpack one XQ4G code word into the four f16x2 mma A-fragment registers as
// fp16 subnormals: a half whose bits are a nibble value v (exponent field 0)
// is exactly v * 2^-24, so masking alone yields
//   w & 0x000F000F -> c * 2^-24          (rows g)
//   w & 0x00F000F0 -> 16 c * 2^-24       (rows g+8)
// and the same on w >> 8 for nibbles 2/3: one shift and four ANDs per word.
// The codes are c = q + 8; the caller removes the 8 * sum(x) this adds
// through the MMA's accumulator input.
__device__ __forceinline__ void unpack_word_c16(uint32_t w, uint32_t (&a)[4])
{
#ifdef XQ4_C16_SHIFT_IMAD
    // w >> 8 as the high word of w * 2^24: an integer multiply-high, which
    // issues to the FMA pipe and leaves the integer ALU pipe to the ANDs
    const uint32_t w8 = __umulhi(w, 1u << 24);
#else
    const uint32_t w8 = w >> 8;
#endif
    a[0] = w & 0x000F000Fu;
    a[1] = w & 0x00F000F0u;
    a[2] = w8 & 0x000F000Fu;
    a[3] = w8 & 0x00F000F0u;
}

// D = A(16x16, row) * B(16x8, col) + C, f16 in, f32 accumulate.
__device__ __forceinline__ void mma_f16_16816_c(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                                const float (&c)[4])
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %11, %12, %13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// D = A(16x16, row) * B(16x8, col), f16 in, f32 out (zero accumulator).
__device__ __forceinline__ void mma_f16_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    const float z = 0.f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

// D += A(16x16, row) * B(16x8, col), f16 in, f32 accumulate.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D = A(16x16, row) * B(16x8, col), bf16 in, f32 out (zero accumulator).
__device__ __forceinline__ void mma_bf16_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    const float z = 0.f;
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

// D = A(16x32 u8, row) * B(32x8 s8, col) + C, s32 (C = {c0, c1, c0, c1}).
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                               int c0, int c1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %11, %10, %11};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
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

// (d0, d1) += s * (x0, x1) as one packed f32x2 FMA (sm_100): two independent
// single-rounding FMAs in one issue slot.
__device__ __forceinline__ void ffma2(float &d0, float &d1, float s, float x0, float x1)
{
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %2};\n\t"
        "mov.b64 rb, {%3, %4};\n\t"
        "mov.b64 rd, {%0, %1};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rd;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "+f"(d0), "+f"(d1)
        : "f"(s), "f"(x0), "f"(x1));
}

// ------------------------------------------------------------ mbarrier / bulk
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// 64-bit words shared with other GPUs (system scope, no ordering): one
// aligned 64-bit access is single-copy atomic, so a reader sees a word whole.
__device__ __forceinline__ void st_sys_u64(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_sys_u32(unsigned *p, unsigned v)
{
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_sys_u32(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait: false if the phase did not complete within about 2 s.  A
// waiting thread is suspended in the barrier (up to 20 us per try) instead of
// spinning, so it leaves the issue slots to the warps doing the work.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t limit = (1u << 24))
{
    (void)limit;
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if (global_ns() - t0 > 2000000000ull) return false;
    }
}

// Shared-memory loads by 32-bit shared address (explicit ld.shared: the
// short-latency path, whatever the compiler can infer about a pointer).
__device__ __forceinline__ uint4 lds_v4(uint32_t a)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint2 lds_v2(uint32_t a)
{
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ float4 lds_f4(uint32_t a)
{
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a)
                 : "memory");
    return v;
}

// Bulk global -> shared copy (no multicast), completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory, and
// let the next grid start launching.  No-ops without the launch attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace xq4d
