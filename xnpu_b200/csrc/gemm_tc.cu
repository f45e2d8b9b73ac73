// gemm_tc.cu -- K2: batched-decode / prefill dequant-GEMM (m >= 25) on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// y[m][n] = x[m][k] . dequant(W)^T with dequant(W) = RNE_bf16(q * scale), the
// reference's dequantized weights (crates/xnpu-cli/src/main.rs:3097-3125),
// bf16 operands and f32 accumulation.  The reference has no int4 GEMM; this is
// its GEMV (main.rs:2287-2296) extended to m rows over the dequantized
// weights.
//
// One CTA computes a 128-feature x BN-token output tile (BN = 256 for long
// inputs, m rounded up to 16 otherwise) over a range of K, in 64-wide stages,
// with three independent shared-memory rings:
//  * packed weights: P stages of 4 consecutive K chunks of the tile's 8 row
//    blocks (8 contiguous 2.3 KB runs, 18 KB), one 3-D TMA load each (no
//    multicast), filled ahead of use by the packed producer warp -- the
//    weights are the HBM stream (measured: TMA loads of single 576-byte
//    units ran at ~6 GB/s per CTA);
//  * x: D stages of the BN x 64 bf16 activation tile (TMA, 128-byte
//    swizzle, out-of-range rows/K zero filled), from the x producer warp;
//  * A: D stages of the dequantized 128 x 64 bf16 weight tile.
// The x and A rings advance together (depth D = 3), so one tcgen05.commit
// per stage frees both (the MMA thread's issue rate bounds the loop: each
// commit costs it ~125 ns, measured).
// Eight dequant warps (warp w = row block w of the tile) turn each packed
// stage into RNE_bf16(q * s) (fma.rn.bf16x2, exact as in the dequant op),
// stored straight into the A tile in the canonical K-major 128-byte-swizzle
// layout, each lane writing whole 16-byte swizzle chunks in an order that
// keeps every 8-lane phase on 8 distinct bank groups; fence.proxy.async;
// arrive.  One thread of the MMA warp issues 4 tcgen05.mma (M=128, N=BN,
// K=16) per stage into tensor memory and tcgen05.commit releases the A and x
// stages.  The epilogue (the dequant warps: 32 TMEM lanes x half the columns
// each) reads the accumulator with tcgen05.ld.
//
// Split-K: when the output has fewer tiles than the GPU has CTA slots (small
// m), S CTAs of one thread-block cluster take S slices of K for the same
// tile.  Each leaves its f32 partial tile in its own shared memory; after a
// cluster handshake on mbarriers (bounded waits), CTA z sums column slice z of
// all S partials in rank order through distributed shared memory
// (deterministic) and writes y.  No global workspace.
//
// Every mbarrier wait is bounded; a wait that runs out sets g_xq4_fault, the
// thread skips the rest of its work (never a barrier), waits for its own
// MMAs (bounded) and the CTA frees its tensor memory before it returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <atomic>
#include <cuda_bf16.h>
#include <stdint.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

constexpr int kTileN = 128;                      // features per CTA (MMA M)
constexpr int kTileK = 64;                       // K per stage (one XQ4G chunk)
constexpr int kRb = kTileN / XQ4G_ROWS;          // row blocks per tile (8)
constexpr int kDqWarps = 8;                      // dequant + epilogue warps
constexpr int kPackWarp = 8, kXWarp = 9, kMmaWarp = 10;
constexpr int kThreads = 11 * 32;
constexpr int kDqThreads = kDqWarps * 32;
constexpr int kATileBytes = kTileN * kTileK * 2;  // 16 KB bf16
constexpr int kPkChunks = 4;                     // K chunks per packed-weight stage
constexpr int kPackedBytes = kRb * kPkChunks * XQ4G_UNIT_BYTES;  // 18 KB: 8 runs of 2.3 KB
constexpr int kMaxSplit = 8;
constexpr int kMaxSmem = 227 * 1024;

__host__ __device__ constexpr int x_tile_bytes(int bn) { return bn * kTileK * 2; }
__host__ __device__ constexpr int n_bars(int P, int D) { return 2 * P + 3 * D + 3; }
// [A tiles | x tiles | packed | mbarriers | tmem address], all from a 1024-aligned base
__host__ __device__ constexpr size_t smem_bytes(int bn, int P, int D)
{
    return 1024 + (size_t)D * kATileBytes + (size_t)D * x_tile_bytes(bn) + (size_t)P * kPackedBytes +
           (size_t)n_bars(P, D) * 8 + 16;
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

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
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

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(xq4d::smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(xq4d::smem_u32(bar))
        : "memory");
}

// 16-byte chunk j (0..7) of row r of a K-major 128-byte-swizzle tile.
__device__ __forceinline__ uint32_t sw128_offset(int r, int j)
{
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}

// One dequant warp's view of one packed chunk: lane l's 16 code bytes and its
// row pair's two group scales (rows g, g + 8: bytes g * 8 of the scale run).
// Explicit ld.shared / st.shared: generic accesses here measured 4-5 % slower
// over the whole GEMM (m = 32 .. 2048).
struct PkChunk {
    uint4 cw;
    uint2 sw;
};
__device__ __forceinline__ PkChunk load_pk_chunk(const uint8_t *up, int lane)
{
    const uint32_t u = xq4d::smem_u32(up);
    return {xq4d::lds_v4(u + lane * 16), xq4d::lds_v2(u + XQ4G_CODE_BYTES + (lane >> 2) * 8)};
}
__device__ __forceinline__ void store_a16(uint8_t *a, uint32_t off, uint4 v)
{
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(xq4d::smem_u32(a) + off), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// ------------------------------------------------------------ cluster helpers
__device__ __forceinline__ uint32_t cluster_map(uint32_t local_saddr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_saddr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_saddr) : "memory");
}
// Bounded wait with cluster-scope acquire (sees peers' shared-memory writes
// released by their arrivals).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity)
{
    for (uint32_t i = 0; i < (1u << 24); i++) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(xq4d::smem_u32(bar)), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t cluster_saddr)
{
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_saddr) : "memory");
    return v;
}
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void store_out(void *y, int out_f32, size_t idx, float v)
{
    if (out_f32)
        reinterpret_cast<float *>(y)[idx] = v;
    else
        reinterpret_cast<__nv_bfloat16 *>(y)[idx] = __float2bfloat16_rn(v);
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap pmap, int n, int nb,
            int kc_n, int m, int bn, int P, int D, int S, int tile0, int tiles_n, void *__restrict__ y, int out_f32)
{
    extern __shared__ uint8_t smem_raw[];
    // the 1024-byte aligned base as an offset into the shared array: the
    // compiler keeps every access through it in the shared state space (an
    // integer round trip of the pointer made them generic: 1.5-2 % slower)
    uint8_t *smem = smem_raw + ((1024u - (xq4d::smem_u32(smem_raw) & 1023u)) & 1023u);
    const int X = D, A = D;                                 // x and A stages advance together
    uint8_t *at = smem;                                     // [D][128][64] bf16, swizzled
    uint8_t *xt = at + (size_t)A * kATileBytes;             // [D][bn][64] bf16, swizzled
    uint8_t *pk = xt + (size_t)X * x_tile_bytes(bn);        // [P][8 row blocks][4 chunks]
    uint64_t *pfull = reinterpret_cast<uint64_t *>(pk + (size_t)P * kPackedBytes);
    uint64_t *pempty = pfull + P;
    uint64_t *xfull = pempty + P;
    uint64_t *afull = xfull + X;
    uint64_t *sfree = afull + A;  // stage d's x and A slots free again (one MMA commit)
    uint64_t *accf = sfree + D;
    uint64_t *part_ready = accf + 1;  // split-K: arrivals of the S CTAs' partials
    uint64_t *part_done = part_ready + 1;  // split-K: the S CTAs finished reading
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(part_done + 1);
    float *part = reinterpret_cast<float *>(smem);  // split-K partial [bn][128] over the A/x rings

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // output tile tile0 + blockIdx.x, feature tiles fastest (CTAs that run
    // together share their x tiles in L2)
    const int tile = tile0 + (int)blockIdx.x, tile_n = tile % tiles_n, tile_m = tile / tiles_n, z = blockIdx.z;
    const int rb0 = tile_n * kRb;
    const int m0 = tile_m * bn;
    const int kc_beg = (int)((long long)z * kc_n / S), kc_end = (int)((long long)(z + 1) * kc_n / S);
    const int nk = kc_end - kc_beg;
    const uint32_t tmem_cols = bn <= 32 ? 32 : (bn <= 64 ? 64 : (bn <= 128 ? 128 : 256));

    if (threadIdx.x == 0) {
        for (int s = 0; s < P; s++) {
            xq4d::mbar_init(&pfull[s], 1);
            xq4d::mbar_init(&pempty[s], kDqWarps);
        }
        for (int s = 0; s < X; s++) {
            xq4d::mbar_init(&xfull[s], 1);
            xq4d::mbar_init(&sfree[s], 1);
        }
        for (int s = 0; s < A; s++) {
            xq4d::mbar_init(&afull[s], kDqWarps);
        }
        xq4d::mbar_init(accf, 1);
        xq4d::mbar_init(part_ready, S);
        xq4d::mbar_init(part_done, S);
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
    if (S > 1)
        cluster_sync_all();  // every CTA of the cluster has initialised its barriers
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool failed = false;
    // The next launch on the stream may start its prologue and weight loads
    // now (programmatic dependent launch); x (read below) and y (written in
    // the epilogue) wait for the previous launch to complete.
    xq4d::grid_dep_launch();

    // Ring positions advance incrementally (slot, phase parity): no integer
    // division by the runtime ring depths in the loops.
    if (warp == kPackWarp) {  // ------------------------------ packed-weight producer
        if (lane == 0) {
            const int npk = (nk + kPkChunks - 1) / kPkChunks;
            int s = 0, issued = 0;
            uint32_t ph = 0;
            for (int i = 0; i < npk; i++) {
                if (i >= P && !xq4d::mbar_wait(&pempty[s], ph ^ 1)) {
                    failed = true;
                    break;
                }
                // chunks past this CTA's K range are loaded and ignored; past
                // the matrix they read as zero
                xq4d::mbar_arrive_expect_tx(&pfull[s], kPackedBytes);
                tma_load_3d(pk + (size_t)s * kPackedBytes, &pmap, 0, kc_beg + i * kPkChunks, rb0, &pfull[s]);
                issued = i + 1;
                if (++s == P) {
                    s = 0;
                    ph ^= 1;
                }
            }
            // no copy may still be landing in shared memory when the CTA exits
            for (int i = max(0, issued - P); i < issued; i++)
                if (!xq4d::mbar_wait(&pfull[i % P], (uint32_t)(i / P) & 1)) failed = true;
        }
    } else if (warp == kXWarp) {  // ------------------------------ activation producer
        if (lane == 0) {
            xq4d::grid_dep_wait();
            const uint32_t bytes = (uint32_t)x_tile_bytes(bn);
            int s = 0, issued = 0;
            uint32_t ph = 0;
            for (int i = 0; i < nk; i++) {
                if (i >= X && !xq4d::mbar_wait(&sfree[s], ph ^ 1)) {
                    failed = true;
                    break;
                }
                xq4d::mbar_arrive_expect_tx(&xfull[s], bytes);
                tma_load_2d(xt + (size_t)s * x_tile_bytes(bn), &xmap, (kc_beg + i) * kTileK, m0, &xfull[s]);
                issued = i + 1;
                if (++s == X) {
                    s = 0;
                    ph ^= 1;
                }
            }
            for (int i = max(0, issued - X); i < issued; i++)
                if (!xq4d::mbar_wait(&xfull[i % X], (uint32_t)(i / X) & 1)) failed = true;
        }
    } else if (warp == kMmaWarp) {  // ------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16(kTileN, bn);
            const uint32_t a_base = xq4d::smem_u32(at), x_base = xq4d::smem_u32(xt);
            int sx = 0, sa = 0;
            uint32_t px = 0, pa = 0;
            for (int i = 0; i < nk; i++) {
                if (!xq4d::mbar_wait(&xfull[sx], px) || !xq4d::mbar_wait(&afull[sa], pa)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint64_t adesc = sw128_desc(a_base + (uint32_t)sa * kATileBytes);
                const uint64_t bdesc = sw128_desc(x_base + (uint32_t)sx * (uint32_t)x_tile_bytes(bn));
#pragma unroll
                for (int kk = 0; kk < kTileK / 16; kk++)  // +32 bytes along K per step
                    mma_bf16_ss(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0);
                mma_commit(&sfree[sa]);  // x and A stage free once these MMAs have read it (sx == sa)
                if (++sx == X) {
                    sx = 0;
                    px ^= 1;
                }
                if (++sa == A) {
                    sa = 0;
                    pa ^= 1;
                }
            }
            mma_commit(accf);  // accumulator complete (or whatever was issued)
        }
    } else {  // ------------------------------------------------ dequant (warp = row block)
        const int g = lane >> 2, t = lane & 3;
        const int gsel = g & 1;  // store order: keeps each 8-lane phase on 8 distinct chunk columns
        int sp = 0, c = 0, sa = 0;  // packed stage slot, chunk within it, A slot
        uint32_t pp = 0, pa = 0;
        for (int i = 0; i < nk && !failed; i++) {
            if (c == 0 && !xq4d::mbar_wait(&pfull[sp], pp)) {
                failed = true;
                break;
            }
            // the box lands as [row block][chunk][576 B]
            const uint8_t *up = pk + (size_t)sp * kPackedBytes + (warp * kPkChunks + c) * XQ4G_UNIT_BYTES;
            const PkChunk pc = load_pk_chunk(up, lane);
            const uint4 cw = pc.cw;
            const uint2 sw = pc.sw;
            __syncwarp();
            const bool stage_done = c == kPkChunks - 1 || i == nk - 1;
            if (lane == 0 && stage_done) xq4d::mbar_arrive(&pempty[sp]);  // packed stage read: refill it
            if (++c == kPkChunks) {
                c = 0;
                if (++sp == P) {
                    sp = 0;
                    pp ^= 1;
                }
            }
            if (i >= A && !xq4d::mbar_wait(&sfree[sa], pa ^ 1)) {
                failed = true;
                break;
            }
            const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
            uint4 lo[2], hi[2];  // rows g / g+8, K 32G+8t .. +8 for group G
#pragma unroll
            for (int G = 0; G < 2; G++) {
                const uint32_t sg = G ? sw.y : sw.x;
                const uint32_t s_lo = __byte_perm(sg, 0, 0x1010), s_hi = __byte_perm(sg, 0, 0x3232);
                uint32_t a0[4], a1[4];
                xq4d::dequant_word(words[2 * G], s_lo, s_hi, a0);
                xq4d::dequant_word(words[2 * G + 1], s_lo, s_hi, a1);
                lo[G] = make_uint4(a0[0], a0[2], a1[0], a1[2]);
                hi[G] = make_uint4(a0[1], a0[3], a1[1], a1[3]);
            }
            uint8_t *a = at + (size_t)sa * kATileBytes;
            const int r0 = warp * XQ4G_ROWS + g;  // swizzle chunk of (row, group G) = 4G + t
            store_a16(a, sw128_offset(r0, 4 * gsel + t), gsel ? lo[1] : lo[0]);
            store_a16(a, sw128_offset(r0, 4 * (1 - gsel) + t), gsel ? lo[0] : lo[1]);
            store_a16(a, sw128_offset(r0 + 8, 4 * gsel + t), gsel ? hi[1] : hi[0]);
            store_a16(a, sw128_offset(r0 + 8, 4 * (1 - gsel) + t), gsel ? hi[0] : hi[1]);
            // each writer makes its stores visible to the tensor core; one
            // arrival per warp (256 arrivals on one mbarrier serialise: they
            // cost ~1 us per stage, measured)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(&afull[sa]);
            if (++sa == A) {
                sa = 0;
                pa ^= 1;
            }
        }
    }

    // ---------------------------------------------------------------- epilogue
    // Dequant warp w reads TMEM lanes 32*(w%4).. (features) and columns
    // [h*bn/2, (h+1)*bn/2) (tokens), h = w / 4.
    const bool epi = warp < kDqWarps;
    if (epi) {
        xq4d::grid_dep_wait();
        if (!xq4d::mbar_wait(accf, 0)) failed = true;
        tc_fence_after();
        const int q4 = warp & 3, h = warp >> 2;
        const int f = q4 * 32 + lane;  // feature within the tile = TMEM lane
        const int feat = rb0 * XQ4G_ROWS + f;
        const int c_half = bn / 2;
        for (int c0 = h * c_half; c0 < (h + 1) * c_half; c0 += 8) {
            uint32_t r[8];
            tmem_ld8(tmem + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float v = failed ? 0.f : __uint_as_float(r[c]);
                if (S > 1) {
                    part[(size_t)(c0 + c) * kTileN + f] = v;
                } else {
                    const int tok = m0 + c0 + c;
                    if (!failed && tok < m && feat < n) store_out(y, out_f32, (size_t)tok * n + feat, v);
                }
            }
        }
    }
    if (S > 1) {
        // Split-K: every CTA of the cluster signals that its partial is in
        // place, then CTA z sums column slice z of the S partials in rank
        // order and writes it; a CTA leaves only after every peer has
        // finished reading its shared memory.
        asm volatile("bar.sync 1, %0;" ::"r"(kThreads) : "memory");
        if (threadIdx.x == 0) {
            asm volatile("fence.acq_rel.cluster;" ::: "memory");
            for (int r = 0; r < S; r++) remote_arrive(cluster_map(xq4d::smem_u32(part_ready), (uint32_t)r));
        }
        if (epi) {
            if (!mbar_wait_cluster(part_ready, 0)) failed = true;
            const int c_lo = (int)((long long)z * bn / S), c_hi = (int)((long long)(z + 1) * bn / S);
            const int f = threadIdx.x & (kTileN - 1), feat = rb0 * XQ4G_ROWS + f;
            const uint32_t part_s = xq4d::smem_u32(part);
            // four columns' S partials in flight per thread, each column's
            // summed in rank order
            constexpr int kCols = 4, kStep = kDqThreads / kTileN;
            for (int c0 = c_lo + (threadIdx.x >> 7); c0 < c_hi; c0 += kCols * kStep) {
                float v[kCols][kMaxSplit];
#pragma unroll
                for (int j = 0; j < kCols; j++) {
                    const int c = c0 + j * kStep;
                    const uint32_t off = (uint32_t)((c * kTileN + f) * 4);
#pragma unroll
                    for (int r = 0; r < kMaxSplit; r++)
                        v[j][r] = (c < c_hi && r < S) ? ld_cluster_f32(cluster_map(part_s + off, (uint32_t)r)) : 0.f;
                }
#pragma unroll
                for (int j = 0; j < kCols; j++) {
                    const int c = c0 + j * kStep;
                    float sum = 0.f;
#pragma unroll
                    for (int r = 0; r < kMaxSplit; r++)
                        if (r < S) sum += v[j][r];
                    const int tok = m0 + c;
                    if (!failed && c < c_hi && tok < m && feat < n) store_out(y, out_f32, (size_t)tok * n + feat, sum);
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kThreads) : "memory");
        if (threadIdx.x == 0) {
            for (int r = 0; r < S; r++) remote_arrive(cluster_map(xq4d::smem_u32(part_done), (uint32_t)r));
            if (!mbar_wait_cluster(part_done, 0)) failed = true;
        }
    }
    if (failed) atomicOr(&g_xq4_fault, XQ4_FAULT_GEMM_WAIT);
    // no MMA may still be writing the accumulator when it is freed
    if (warp == kMmaWarp && lane == 0) xq4d::mbar_wait(accf, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols)
                     : "memory");
}

// ------------------------------------------------------- persistent variant
// Whole waves of tiles when one CTA fills an SM (BN > 64): each CTA walks the
// tiles blockIdx.x, blockIdx.x + gridDim.x, ... of its launch.  The three
// rings run on across tiles (the next tile's weights, x and A stream while the
// current tile's last MMAs run), and the accumulator alternates between two
// tensor-memory halves: four epilogue warps read out and store tile j while
// the MMAs of tile j + 1 fill the other half.  Per tile this saves a CTA
// launch, its prologue and an epilogue that nothing overlapped.
constexpr int kEpiWarp0 = 11, kEpiWarps = 4;
constexpr int kPtThreads = (kEpiWarp0 + kEpiWarps) * 32;

__host__ __device__ constexpr size_t pt_smem_bytes(int bn, int P, int D)
{
    return 1024 + (size_t)D * kATileBytes + (size_t)D * x_tile_bytes(bn) + (size_t)P * kPackedBytes +
           (size_t)(2 * P + 3 * D + 4) * 8 + 16;
}

__global__ void __launch_bounds__(kPtThreads, 1)
gemm_pt_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap pmap, int n, int kc_n,
               int m, int bn, int P, int D, int tile0, int count, int tiles_n, void *__restrict__ y, int out_f32)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (xq4d::smem_u32(smem_raw) & 1023u)) & 1023u);  // as gemm_kernel
    const uint32_t xbytes = (uint32_t)x_tile_bytes(bn);
    uint8_t *at = smem;                            // [D][128][64] bf16, swizzled
    uint8_t *xt = at + (size_t)D * kATileBytes;     // [D][bn][64] bf16, swizzled
    uint8_t *pk = xt + (size_t)D * xbytes;          // [P][8 row blocks][4 chunks]
    uint64_t *pfull = reinterpret_cast<uint64_t *>(pk + (size_t)P * kPackedBytes);
    uint64_t *pempty = pfull + P;
    uint64_t *xfull = pempty + P;
    uint64_t *afull = xfull + D;
    uint64_t *sfree = afull + D;  // stage d's x and A slots free again (one MMA commit)
    uint64_t *accf = sfree + D;   // [2] accumulator half complete
    uint64_t *acce = accf + 2;    // [2] accumulator half read out
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acce + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntl = (count - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;  // this CTA's tiles
    const int nk = kc_n;
    const uint32_t acc_cols = bn <= 32 ? 32 : (bn <= 64 ? 64 : (bn <= 128 ? 128 : 256));
    const auto tile_of = [&](int j, int &rb0, int &m0) {
        const int t = tile0 + (int)blockIdx.x + j * (int)gridDim.x;
        rb0 = (t % tiles_n) * kRb;
        m0 = (t / tiles_n) * bn;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < P; s++) {
            xq4d::mbar_init(&pfull[s], 1);
            xq4d::mbar_init(&pempty[s], kDqWarps);
        }
        for (int s = 0; s < D; s++) {
            xq4d::mbar_init(&xfull[s], 1);
            xq4d::mbar_init(&sfree[s], 1);
            xq4d::mbar_init(&afull[s], kDqWarps);
        }
        for (int h = 0; h < 2; h++) {
            xq4d::mbar_init(&accf[h], 1);
            xq4d::mbar_init(&acce[h], kEpiWarps);
        }
        xq4d::fence_barrier_init();
    }
    if (warp == kMmaWarp) {  // two accumulator halves
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         xq4d::smem_u32(tmem_slot)),
                     "r"(2 * acc_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool failed = false;
    xq4d::grid_dep_launch();  // as gemm_kernel: x and y wait for the previous launch below

    if (warp == kPackWarp) {  // ------------------------------ packed-weight producer
        if (lane == 0) {
            const int npk = (nk + kPkChunks - 1) / kPkChunks;
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            for (int j = 0; j < ntl && !failed; j++) {
                int rb0, m0;
                tile_of(j, rb0, m0);
                for (int i = 0; i < npk; i++) {
                    if (issued >= P && !xq4d::mbar_wait(&pempty[s], ph ^ 1)) {
                        failed = true;
                        break;
                    }
                    xq4d::mbar_arrive_expect_tx(&pfull[s], kPackedBytes);
                    tma_load_3d(pk + (size_t)s * kPackedBytes, &pmap, 0, i * kPkChunks, rb0, &pfull[s]);
                    issued++;
                    if (++s == P) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            // no copy may still be landing in shared memory when the CTA exits
            for (long long q = issued > P ? issued - P : 0; q < issued; q++)
                if (!xq4d::mbar_wait(&pfull[q % P], (uint32_t)(q / P) & 1)) failed = true;
        }
    } else if (warp == kXWarp) {  // ------------------------------ activation producer
        if (lane == 0) {
            xq4d::grid_dep_wait();
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            for (int j = 0; j < ntl && !failed; j++) {
                int rb0, m0;
                tile_of(j, rb0, m0);
                for (int i = 0; i < nk; i++) {
                    if (issued >= D && !xq4d::mbar_wait(&sfree[s], ph ^ 1)) {
                        failed = true;
                        break;
                    }
                    xq4d::mbar_arrive_expect_tx(&xfull[s], xbytes);
                    tma_load_2d(xt + (size_t)s * xbytes, &xmap, i * kTileK, m0, &xfull[s]);
                    issued++;
                    if (++s == D) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            for (long long q = issued > D ? issued - D : 0; q < issued; q++)
                if (!xq4d::mbar_wait(&xfull[q % D], (uint32_t)(q / D) & 1)) failed = true;
        }
    } else if (warp == kMmaWarp) {  // ------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16(kTileN, bn);
            const uint32_t a_base = xq4d::smem_u32(at), x_base = xq4d::smem_u32(xt);
            int sl = 0;
            uint32_t ph = 0;
            for (int j = 0; j < ntl && !failed; j++) {
                const int h = j & 1;
                // the epilogue has read this half's previous tile
                if (j >= 2 && !xq4d::mbar_wait(&acce[h], (uint32_t)((j >> 1) - 1) & 1)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)h * acc_cols;
                for (int i = 0; i < nk; i++) {
                    if (!xq4d::mbar_wait(&xfull[sl], ph) || !xq4d::mbar_wait(&afull[sl], ph)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = sw128_desc(a_base + (uint32_t)sl * kATileBytes);
                    const uint64_t bdesc = sw128_desc(x_base + (uint32_t)sl * xbytes);
#pragma unroll
                    for (int kk = 0; kk < kTileK / 16; kk++)
                        mma_bf16_ss(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0);
                    mma_commit(&sfree[sl]);
                    if (++sl == D) {
                        sl = 0;
                        ph ^= 1;
                    }
                }
                mma_commit(&accf[h]);  // this tile's accumulator complete (or whatever was issued)
            }
        }
    } else if (warp < kDqWarps) {  // ---------------------------- dequant (warp = row block)
        const int g = lane >> 2, t = lane & 3;
        const int gsel = g & 1;
        int sp = 0, c = 0, sa = 0;
        uint32_t pp = 0, pa = 0;
        long long cnt = 0;
        for (int j = 0; j < ntl && !failed; j++) {
            for (int i = 0; i < nk && !failed; i++, cnt++) {
                if (c == 0 && !xq4d::mbar_wait(&pfull[sp], pp)) {
                    failed = true;
                    break;
                }
                const uint8_t *up = pk + (size_t)sp * kPackedBytes + (warp * kPkChunks + c) * XQ4G_UNIT_BYTES;
                const PkChunk pc = load_pk_chunk(up, lane);
                const uint4 cw = pc.cw;
                const uint2 sw = pc.sw;
                __syncwarp();
                // a tile's packed stages hold 4 chunks each, the last one
                // whatever remains of K
                if (c == kPkChunks - 1 || i == nk - 1) {
                    if (lane == 0) xq4d::mbar_arrive(&pempty[sp]);
                    c = 0;
                    if (++sp == P) {
                        sp = 0;
                        pp ^= 1;
                    }
                } else {
                    c++;
                }
                if (cnt >= D && !xq4d::mbar_wait(&sfree[sa], pa ^ 1)) {
                    failed = true;
                    break;
                }
                const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
                uint4 lo[2], hi[2];
#pragma unroll
                for (int G = 0; G < 2; G++) {
                    const uint32_t sg = G ? sw.y : sw.x;
                    const uint32_t s_lo = __byte_perm(sg, 0, 0x1010), s_hi = __byte_perm(sg, 0, 0x3232);
                    uint32_t a0[4], a1[4];
                    xq4d::dequant_word(words[2 * G], s_lo, s_hi, a0);
                    xq4d::dequant_word(words[2 * G + 1], s_lo, s_hi, a1);
                    lo[G] = make_uint4(a0[0], a0[2], a1[0], a1[2]);
                    hi[G] = make_uint4(a0[1], a0[3], a1[1], a1[3]);
                }
                uint8_t *a = at + (size_t)sa * kATileBytes;
                const int r0 = warp * XQ4G_ROWS + g;
                store_a16(a, sw128_offset(r0, 4 * gsel + t), gsel ? lo[1] : lo[0]);
                store_a16(a, sw128_offset(r0, 4 * (1 - gsel) + t), gsel ? lo[0] : lo[1]);
                store_a16(a, sw128_offset(r0 + 8, 4 * gsel + t), gsel ? hi[1] : hi[0]);
                store_a16(a, sw128_offset(r0 + 8, 4 * (1 - gsel) + t), gsel ? hi[0] : hi[1]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) xq4d::mbar_arrive(&afull[sa]);
                if (++sa == D) {
                    sa = 0;
                    pa ^= 1;
                }
            }
        }
    } else {  // ------------------------------------------------ epilogue warps
        // warp w reads TMEM lanes 32 * (w % 4).. (the tile's features), every column
        xq4d::grid_dep_wait();  // y may be read by the previous launch
        const int q4 = warp & 3, f = q4 * 32 + lane;
        for (int j = 0; j < ntl; j++) {
            const int h = j & 1;
            if (!xq4d::mbar_wait(&accf[h], (uint32_t)(j >> 1) & 1)) failed = true;
            tc_fence_after();
            int rb0, m0;
            tile_of(j, rb0, m0);
            const int feat = rb0 * XQ4G_ROWS + f;
            for (int c0 = 0; c0 < bn; c0 += 8) {
                uint32_t r[8];
                tmem_ld8(tmem + (uint32_t)h * acc_cols + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const int tok = m0 + c0 + c;
                    if (!failed && tok < m && feat < n) store_out(y, out_f32, (size_t)tok * n + feat, __uint_as_float(r[c]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(&acce[h]);  // the MMAs may refill this half
        }
    }
    if (failed) atomicOr(&g_xq4_fault, XQ4_FAULT_GEMM_WAIT);
    // no MMA may still be writing the accumulator when it is freed: the MMA
    // thread waits for its last commit of each half (bounded)
    if (warp == kMmaWarp && lane == 0)
        for (int j = ntl > 2 ? ntl - 2 : 0; j < ntl; j++) xq4d::mbar_wait(&accf[j & 1], (uint32_t)(j >> 1) & 1);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kMmaWarp)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * acc_cols)
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

cudaError_t xq4_launch_gemm(const uint8_t *pack, int n, int k, const void *x, int m, void *y, int out_f32,
                            cudaStream_t st)
{
    auto encode = encode_fn();
    if (!encode) return cudaErrorNotSupported;
    const int nb = xq4g_nb(n), kc = xq4g_kc(k);
    const int bn = m >= 256 ? 256 : ((m + 15) / 16) * 16;
    // ring depths: deep weight prefetch, shallow x; two CTAs per SM up to bn = 64
    const int D = 3;                                   // x / A stages
    const int P = bn <= 64 ? 2 : (bn <= 128 ? 4 : 3);  // 18 KB packed stages
    const size_t smem = smem_bytes(bn, P, D);
    if (smem > (size_t)kMaxSmem) return cudaErrorInvalidValue;
    const int per_sm = 2 * (smem + 1024) <= 228 * 1024 ? 2 : 1;

    CUtensorMap xmap, pmap;
    {
        const cuuint64_t gdim[2] = {(cuuint64_t)k, (cuuint64_t)m};
        const cuuint64_t gstride[1] = {(cuuint64_t)k * 2};
        const cuuint32_t box[2] = {(cuuint32_t)kTileK, (cuuint32_t)bn};
        const cuuint32_t estride[2] = {1, 1};
        if (encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), gdim, gstride, box, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    {
        // XQ4G image as [row block][chunk][144 u32]: one box = 4 consecutive
        // chunks of the 8 row blocks of a 128-feature tile (rows past nb and
        // chunks past KC read as zero)
        const cuuint64_t gdim[3] = {XQ4G_UNIT_BYTES / 4, (cuuint64_t)kc, (cuuint64_t)nb};
        const cuuint64_t gstride[2] = {XQ4G_UNIT_BYTES, (cuuint64_t)kc * XQ4G_UNIT_BYTES};
        const cuuint32_t box[3] = {XQ4G_UNIT_BYTES / 4, kPkChunks, kRb};
        const cuuint32_t estride[3] = {1, 1, 1};
        if (encode(&pmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(pack), gdim, gstride, box,
                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    static std::atomic<bool> attr_set[64];  // zero-initialised; atomics: first launches may race across threads
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_pt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int tiles_n = (nb + kRb - 1) / kRb, tiles_m = (m + bn - 1) / bn;
    const long long tiles = (long long)tiles_n * tiles_m;
    if (tiles > (1ll << 30)) return cudaErrorInvalidValue;
    const long long slots = (long long)sm_count() * per_sm;
    // Whole waves of tiles first; the tiles of a last, partial wave (or all
    // of them when they leave CTA slots idle) in a second launch whose K is
    // split over a cluster of S >= 2 CTAs per tile, at least 4 chunks per
    // slice (a last wave of more than half the slots stays in the first).
    // (Prefill 2048 x 4096 -> 14336: 896 tiles on 148 slots were 7 waves, the
    // last of 8 tiles.)  The second launch's weight loads and prologue overlap
    // the first one's tail (programmatic dependent launch).
    long long full = tiles / slots * slots, rest = tiles - full;
    if (rest * 2 > slots) {  // a last wave that cannot be split: one launch
        full = tiles;
        rest = 0;
    }
    const auto launch = [&](long long tile0, long long count, int S) -> cudaError_t {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)count, 1, S);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = S;
        cfg.attrs = attr;
        cfg.numAttrs = S > 1 ? 2 : 1;
        return cudaLaunchKernelEx(&cfg, gemm_kernel, xmap, pmap, n, nb, kc, m, bn, P, D, S, (int)tile0, tiles_n, y,
                                  out_f32);
    };
    // one CTA fills an SM and every CTA has two tiles or more: the persistent
    // kernel walks the whole waves (with one tile per CTA it has nothing to
    // overlap, and its four epilogue warps drain a tile slower than eight)
    if (full >= 2 * slots && per_sm == 1) {
        const size_t pt_smem = pt_smem_bytes(bn, P, D);
        if (pt_smem > (size_t)kMaxSmem) return cudaErrorInvalidValue;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)std::min(full, slots));
        cfg.blockDim = dim3(kPtThreads);
        cfg.dynamicSmemBytes = pt_smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_pt_kernel, xmap, pmap, n, kc, m, bn, P, D, 0, (int)full,
                                               tiles_n, y, out_f32);
            e != cudaSuccess)
            return e;
    } else if (full > 0) {
        if (cudaError_t e = launch(0, full, 1); e != cudaSuccess) return e;
    }
    if (rest == 0) return cudaSuccess;
    int S = (int)(slots / rest);
    if (S > kMaxSplit) S = kMaxSplit;
    if (S > kc / 4) S = kc / 4;
    if (S < 1) S = 1;
    return launch(full, rest, S);
}

unsigned int xq4_take_fault_gemm()
{
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_xq4_fault, sizeof v) != cudaSuccess) return ~0u;
    cudaMemcpyToSymbol(g_xq4_fault, &zero, sizeof zero);
    return v;
}
