// gemm_tc.cu -- K2: batched-decode / prefill dequant-GEMM (m >= 16) on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// y[m][n] = x[m][k] . dequant(W)^T with dequant(W) = RNE_bf16(q * scale), the
// reference's dequantized weights (crates/xnpu-cli/src/main.rs:3097-3125),
// bf16 operands and f32 accumulation.  The reference has no int4 GEMM; this is
// its GEMV (main.rs:2287-2296) extended to m rows over the dequantized
// weights.
//
// One CTA computes a 128-feature x BN-token output tile (BN = 256 for long
// inputs, m rounded up to 16 otherwise), streaming K in 64-wide stages:
//  * producer warp: per stage, 8 cp.async.bulk copies of the tile's packed
//    XQ4G units (8 row blocks x one 64-K chunk, 4.6 KB) and one TMA tensor
//    load of the x tile (BN x 64 bf16, 128-byte swizzle; no multicast), both
//    counted on the stage's mbarrier;
//  * 4 dequant warps: unpack + RNE_bf16(q * s) (fma.rn.bf16x2, exact as in the
//    dequant op) straight into the A operand tile in the canonical K-major
//    128-byte-swizzle layout (each lane owns whole 16-byte swizzle chunks),
//    fence.proxy.async, arrive;
//  * MMA warp: one elected thread issues 4 tcgen05.mma (M=128, N=BN, K=16)
//    per stage, A = dequantized weights, B = x, D in tensor memory, and a
//    tcgen05.commit that releases the stage;
//  * epilogue (the 4 dequant warps, one per 32-lane TMEM quarter):
//    tcgen05.ld the 128 x BN f32 accumulator, round, store y.
// Every mbarrier wait is bounded; a wait that runs out sets g_xq4_fault, the
// CTA skips the rest of its work, waits for its own MMAs (bounded) and frees
// its tensor memory before it returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

constexpr int kTileN = 128;     // features per CTA (MMA M)
constexpr int kTileK = 64;      // K per stage (one XQ4G chunk)
constexpr int kStages = 3;
constexpr int kDequantWarps = 4;
constexpr int kThreads = (kDequantWarps + 2) * 32;  // + producer warp + MMA warp
constexpr int kProducerWarp = kDequantWarps;
constexpr int kMmaWarp = kDequantWarps + 1;
constexpr int kATileBytes = kTileN * kTileK * 2;    // 16 KB bf16
constexpr int kPackedBytes = (kTileN / XQ4G_ROWS) * XQ4G_UNIT_BYTES;  // 4608

__host__ __device__ constexpr int x_tile_bytes(int bn) { return bn * kTileK * 2; }
// [x tiles | A tiles | packed | barriers | tmem address], x and A 1024-aligned
__host__ __device__ constexpr size_t smem_bytes(int bn)
{
    return 1024 /* alignment slack */ + (size_t)kStages * (x_tile_bytes(bn) + kATileBytes + kPackedBytes) +
           (3 * kStages + 1) * 8 + 16;
}

// ------------------------------------------------------------ tcgen05 helpers
// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 B in
// 8-row (1024 B) atoms; SBO = 1024 B between atoms, LBO unused (1), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr)
{
    return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D f32, A/B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     xq4d::smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            xq4d::smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(xq4d::smem_u32(bar))
        : "memory");
}

// 16-byte chunk j (0..7) of row r of a K-major 128-byte-swizzle tile.
__device__ __forceinline__ uint32_t sw128_offset(int r, int j)
{
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap xmap, const uint8_t *__restrict__ pack, int n, int k, int nb,
            int kc_n, int m, int bn, void *__restrict__ y, int out_f32)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *xt = smem;                                           // [stage][bn][64] bf16, swizzled
    uint8_t *at = xt + (size_t)kStages * x_tile_bytes(bn);        // [stage][128][64] bf16, swizzled
    uint8_t *pk = at + (size_t)kStages * kATileBytes;             // [stage][8 units]
    uint64_t *full = reinterpret_cast<uint64_t *>(pk + (size_t)kStages * kPackedBytes);
    uint64_t *a_full = full + kStages;
    uint64_t *empty = a_full + kStages;
    uint64_t *acc_full = empty + kStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_n = blockIdx.x, tile_m = blockIdx.y;
    const int rb0 = tile_n * (kTileN / XQ4G_ROWS);
    const int nrb = min(kTileN / XQ4G_ROWS, nb - rb0);  // row blocks in this tile
    const int m0 = tile_m * bn;
    const uint32_t tmem_cols = bn <= 32 ? 32 : (bn <= 64 ? 64 : (bn <= 128 ? 128 : 256));

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            xq4d::mbar_init(&full[s], 1);
            xq4d::mbar_init(&a_full[s], kDequantWarps * 32);
            xq4d::mbar_init(&empty[s], 1);
        }
        xq4d::mbar_init(acc_full, 1);
        xq4d::fence_barrier_init();
    }
    if (warp == kMmaWarp) {  // allocate the accumulator columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         xq4d::smem_u32(tmem_slot)),
                     "r"(tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool failed = false;

    if (warp == kProducerWarp) {  // ------------------------------ producer
        if (lane == 0) {
            const uint32_t bytes = (uint32_t)nrb * XQ4G_UNIT_BYTES + (uint32_t)x_tile_bytes(bn);
            int issued = 0;
            for (int kc = 0; kc < kc_n && !failed; kc++) {
                const int s = kc % kStages;
                const uint32_t fill = (uint32_t)(kc / kStages);
                if (fill > 0 && !xq4d::mbar_wait(&empty[s], (fill - 1) & 1)) {
                    failed = true;
                    break;
                }
                xq4d::mbar_arrive_expect_tx(&full[s], bytes);
                for (int u = 0; u < nrb; u++)
                    xq4d::bulk_g2s(pk + (size_t)s * kPackedBytes + u * XQ4G_UNIT_BYTES,
                                   pack + ((size_t)(rb0 + u) * kc_n + kc) * XQ4G_UNIT_BYTES, XQ4G_UNIT_BYTES,
                                   &full[s]);
                tma_load_2d(xt + (size_t)s * x_tile_bytes(bn), &xmap, kc * kTileK, m0, &full[s]);
                issued = kc + 1;
            }
            // no copy may still be landing in shared memory when the CTA exits
            for (int kc = max(0, issued - kStages); kc < issued; kc++)
                if (!xq4d::mbar_wait(&full[kc % kStages], (uint32_t)(kc / kStages) & 1)) failed = true;
        }
    } else if (warp == kMmaWarp) {  // ------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16(kTileN, bn);
            for (int kc = 0; kc < kc_n && !failed; kc++) {
                const int s = kc % kStages;
                const uint32_t par = (uint32_t)(kc / kStages) & 1;
                if (!xq4d::mbar_wait(&full[s], par) || !xq4d::mbar_wait(&a_full[s], par)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint64_t adesc = sw128_desc(xq4d::smem_u32(at + (size_t)s * kATileBytes));
                const uint64_t bdesc = sw128_desc(xq4d::smem_u32(xt + (size_t)s * x_tile_bytes(bn)));
#pragma unroll
                for (int kk = 0; kk < kTileK / 16; kk++)  // +32 bytes along K per step
                    mma_bf16_ss(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kc | kk) != 0);
                mma_commit(&empty[s]);  // stage free once these MMAs have read it
            }
            mma_commit(acc_full);  // accumulator complete (or whatever was issued)
        }
    } else {  // ------------------------------------------------ dequant + epilogue
        const int g = lane >> 2, t = lane & 3;
        for (int kc = 0; kc < kc_n && !failed; kc++) {
            const int s = kc % kStages;
            if (!xq4d::mbar_wait(&full[s], (uint32_t)(kc / kStages) & 1)) {
                failed = true;
                break;
            }
            uint8_t *a = at + (size_t)s * kATileBytes;
#pragma unroll
            for (int uu = 0; uu < 2; uu++) {  // this warp's two row blocks of the tile
                const int u = warp * 2 + uu;
                uint4 cw = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // q = 0
                uint2 sw = make_uint2(0, 0);
                if (u < nrb) {
                    const uint8_t *up = pk + (size_t)s * kPackedBytes + u * XQ4G_UNIT_BYTES;
                    cw = *reinterpret_cast<const uint4 *>(up + lane * 16);
                    sw = *reinterpret_cast<const uint2 *>(up + XQ4G_CODE_BYTES + g * 8);
                }
                const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
                for (int G = 0; G < 2; G++) {
                    const uint32_t sg = G ? sw.y : sw.x;
                    const uint32_t s_lo = __byte_perm(sg, 0, 0x1010), s_hi = __byte_perm(sg, 0, 0x3232);
                    uint32_t a0[4], a1[4];
                    xq4d::dequant_word(words[2 * G], s_lo, s_hi, a0);
                    xq4d::dequant_word(words[2 * G + 1], s_lo, s_hi, a1);
                    // rows g / g+8 of row block u: K 32G+8t .. +8 = swizzle chunk 4G+t
                    const int r0 = u * 16 + g, j = 4 * G + t;
                    *reinterpret_cast<uint4 *>(a + sw128_offset(r0, j)) = make_uint4(a0[0], a0[2], a1[0], a1[2]);
                    *reinterpret_cast<uint4 *>(a + sw128_offset(r0 + 8, j)) = make_uint4(a0[1], a0[3], a1[1], a1[3]);
                }
            }
            // each writer makes its stores visible to the tensor core, then arrives
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            xq4d::mbar_arrive(&a_full[s]);
        }
        // epilogue: TMEM lane = feature (32 per warp), column = token
        if (!xq4d::mbar_wait(acc_full, 0)) failed = true;
        if (!failed) {
            tc_fence_after();
            const int f = warp * 32 + lane;
            const int feat = rb0 * XQ4G_ROWS + f;
            for (int c0 = 0; c0 < bn; c0 += 16) {
                uint32_t r[16];
                tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const int tok = m0 + c0 + c;
                    if (tok < m && feat < n && f < nrb * XQ4G_ROWS) {
                        const float v = __uint_as_float(r[c]);
                        if (out_f32)
                            reinterpret_cast<float *>(y)[(size_t)tok * n + feat] = v;
                        else
                            reinterpret_cast<__nv_bfloat16 *>(y)[(size_t)tok * n + feat] = __float2bfloat16_rn(v);
                    }
                }
            }
        }
    }
    if (failed) atomicOr(&g_xq4_fault, XQ4_FAULT_GEMM_WAIT);
    // no MMA may still be writing the accumulator when it is freed
    if (warp == kMmaWarp && lane == 0) xq4d::mbar_wait(acc_full, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols)
                     : "memory");
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

}  // namespace

cudaError_t xq4_launch_gemm(const uint8_t *pack, int n, int k, const void *x, int m, void *y, int out_f32,
                            cudaStream_t st)
{
    auto encode = encode_fn();
    if (!encode) return cudaErrorNotSupported;
    const int bn = m >= 256 ? 256 : ((m + 15) / 16) * 16;
    CUtensorMap map;
    const cuuint64_t gdim[2] = {(cuuint64_t)k, (cuuint64_t)m};
    const cuuint64_t gstride[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTileK, (cuuint32_t)bn};
    const cuuint32_t estride[2] = {1, 1};
    CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), gdim, gstride, box,
                        estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = smem_bytes(256);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int nb = xq4g_nb(n), kc = xq4g_kc(k);
    dim3 grid((nb + kTileN / XQ4G_ROWS - 1) / (kTileN / XQ4G_ROWS), (m + bn - 1) / bn);
    gemm_kernel<<<grid, kThreads, smem_bytes(bn), st>>>(map, pack, n, k, nb, kc, m, bn, y, out_f32);
    return cudaGetLastError();
}

unsigned int xq4_take_fault_gemm()
{
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_xq4_fault, sizeof v) != cudaSuccess) return ~0u;
    cudaMemcpyToSymbol(g_xq4_fault, &zero, sizeof zero);
    return v;
}
