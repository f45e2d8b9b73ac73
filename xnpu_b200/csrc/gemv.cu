// gemv.cu -- K1: decode GEMV for m = 1..16 tokens over XQ4G int4 weights.
//
// y[m][n] = sum_k (q[n][k] * s[n][k/32]) * x[m][k], the reference's GEMV
// (crates/xnpu-cli/src/main.rs:2287-2296: w = nibble * scale in f32, no
// intermediate rounding, f32 accumulation, one final rounding).  This is the
// B200 replacement for the reference's w4gemv2 / w4gemvu AIE kernels (invoked
// at main.rs:2171-2448, :3288-3898).
//
// Design (HBM-bound: 0.5625 B of weights per weight, 2*m flops per weight):
//  * Persistent grid, two CTAs per SM.  CTA c owns the contiguous row blocks
//    [c*nb/G, (c+1)*nb/G); in the XQ4G layout that is ONE contiguous byte
//    range, streamed front to back.  Two independent CTAs per SM (rather than
//    one twice as large) let the next kernel's CTA move into an SM as soon as
//    one of them finishes.
//  * A producer thread copies the range into a shared-memory ring with
//    cp.async.bulk (the bulk-copy engine, no multicast): 3 stages of 32
//    consecutive 64-K chunks (18 KB) of one row block, completion counted on
//    a per-stage mbarrier; 110 KB in flight per SM.
//  * 8 consumer warps take four chunks each per stage (independent
//    instruction streams per warp; the partial sums accumulate with packed
//    f32x2 FMAs).  A lane's 16 code bytes are exactly its
//    mma.m16n8k16 A fragments for the chunk's 4 K steps, and each K step lies
//    in one 32-K scale group (xq4_layout.h).  The tensor core forms
//    T = sum q*x over a group's 32 K (two K steps, f32) and the group adds
//    s * T in f32.  In exact arithmetic that is sum (q*s)*x, the reference's
//    formula with the weight never rounded (the rounded RNE_bf16(q*s) is the
//    dequant op's output, dequant.cu); only the f32 summation order differs.
//  * Unpack, bf16 path: one lop3 per pair (p = 128 + code, bf16 magic) after a
//    shift of the word by 0/4/8/12, then fma.rn.bf16x2 (q = p - 136, exact).
//  * Unpack, fp16 path (few-token decode on large matrices: m <= 8, the
//    staged activations fit, at least 96K chunks): codes enter the MMA as
//    fp16 subnormals (a half whose bits are the nibble value v is exactly
//    v * 2^-24), so a code word needs one shift and four ANDs; the zero
//    point (q = c - 8) is removed through the MMA's accumulator input, which
//    starts each group at -8 * sum(x) (group sums computed once per CTA).  x
//    is staged once per CTA in shared memory as fp16 scaled by a per-token
//    power of two chosen from the token's max |x| (exact for every value
//    within 2^30 of that max; below it the fp16 rounding error is under
//    2^-40 of the max); the output is scaled back by 2^24 and the inverse
//    power of two (exact).
//  * At the end of a row block each warp leaves its partial sums in one of
//    three shared-memory buffers and carries on; a dedicated reducer warp
//    waits for the 8 partials, sums them in fixed warp order (deterministic)
//    and writes the outputs once.  No consumer warp ever waits for another
//    (measured: a rotating reducer among the consumers cost 16% of the
//    compute time).
//  * Programmatic dependent launch: the producer starts streaming weights
//    before griddepcontrol.wait; only the consumers (which read x and write
//    y) wait for the preceding kernel.
//  * Every mbarrier wait is bounded; a wait that runs out sets g_xq4_fault and
//    the kernel returns.
#include <cuda_runtime.h>
#include <atomic>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdlib.h>

#include "xq4_internal.h"
#include "xq4_layout.h"
#include "xq4_device.cuh"

namespace {

// Tuning (measured on B200, see the header): 2 CTAs per SM, each with 8
// consumer warps and a 3-stage ring of 32-chunk (18 KB) stages (4 in the
// chain kernel).  3 CTAs per SM cap the registers at 64 and spill.
#ifndef XQ4_GEMV_STAGES
#define XQ4_GEMV_STAGES 3
#endif
#ifndef XQ4_GEMV_WARPS
#define XQ4_GEMV_WARPS 8
#endif
#ifndef XQ4_GEMV_STAGE_CHUNKS
#define XQ4_GEMV_STAGE_CHUNKS 32
#endif
constexpr int kConsumerWarps = XQ4_GEMV_WARPS;
constexpr int kStageChunks = XQ4_GEMV_STAGE_CHUNKS;  // chunks per ring stage (576 B each)
constexpr int kCpw = kStageChunks / kConsumerWarps;  // chunks per consumer warp per stage
#ifndef XQ4_GEMV_CHUNKS_IN_FLIGHT
#define XQ4_GEMV_CHUNKS_IN_FLIGHT 2
#endif
// chunks whose operands a single-token consumer warp holds in registers at
// once (measured on B200, m = 1: 1 and 2 are equal and 7 % faster than 4,
// which delays the first MMA of a stage behind more loads)
constexpr int kChunksInFlight = XQ4_GEMV_CHUNKS_IN_FLIGHT;
static_assert(kCpw % kChunksInFlight == 0, "chunks in flight must divide a warp's chunks per stage");
constexpr int kStages = XQ4_GEMV_STAGES;
#ifndef XQ4_GEMV_CTAS_PER_SM
#define XQ4_GEMV_CTAS_PER_SM 2
#endif
constexpr int kCtasPerSm = XQ4_GEMV_CTAS_PER_SM;  // resident CTAs per SM (grid = SMs x this)
constexpr int kStageBytes = kStageChunks * XQ4G_UNIT_BYTES;
constexpr int kStageXBytes = kStageChunks * XQ4G_KCHUNK * 2;  // one token's fp16 x for a stage's chunks
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;     // one thread issues the bulk copies
constexpr int kReducerWarp = kConsumerWarps + 1;  // sums the row blocks' partials, writes y
constexpr int kThreads = kConsumerThreads + 64;
constexpr int kRedBufs = 3;  // row-block partial buffers in flight
constexpr int kBarBytes = ((2 * kStages + 2 * kRedBufs) * 8 + 127) & ~127;  // ring + reduce mbarriers, padded
static_assert(kBarBytes >= (2 * kStages + 2 * kRedBufs) * 8, "barrier region too small");
constexpr int kMaxSmem = 227 * 1024;
// fp16 path limits: m * k_padded activations staged per CTA, and the staged
// x plus the correction table (k_padded * (2m + 1) bytes) small enough that
// two CTAs still fit on an SM.
constexpr int kXhMaxElems = 20480;
// The fp16 path's activation staging is a block-wide prologue of 1.5-4 us
// on the critical path; it pays for itself only on large matrices (measured
// on B200 at m = 1: 28672 x 4096 and 128256 x 4096 are faster with it,
// 14336 x 4096, 6144 x 4096, 4096 x 4096 and 4096 x 14336 without).
constexpr long long kXhMinChunks = XQ4_XH_MIN_CHUNKS;
constexpr int kXhMaxBytes = 46080;
__host__ __device__ constexpr bool xh_fits(int m, int kp)
{
    return m <= 8 && m * kp <= kXhMaxElems && kp * (2 * m + 1) <= kXhMaxBytes;
}

// Shared-memory plan: [barriers | partials | token maxima | fp16 x | correction table | ring]
__host__ __device__ constexpr size_t xh_offset(int nt) { return kBarBytes + (size_t)kRedBufs * kConsumerWarps * nt * 128 * 4; }
__host__ __device__ inline size_t tbl_offset(int nt, int m, int kc_n)
{
    return xh_offset(nt) + 64 + (size_t)m * kc_n * XQ4G_KCHUNK * 2;
}
__host__ __device__ inline size_t ring_offset(int nt, bool xh, int m, int kc_n)
{
    size_t o = xh_offset(nt);
    if (xh) o = tbl_offset(nt, m, kc_n) + (size_t)kc_n * 64;  // + one float4 per (chunk, lane quad)
    return (o + 127) & ~(size_t)127;
}
__host__ __device__ inline size_t smem_bytes(int nt, bool xh, int m, int kc_n)
{
    return ring_offset(nt, xh, m, kc_n) + (size_t)kStages * kStageBytes;
}

// One ring stage for one consumer warp: its chunks kc0 + warp + c*16.  The
// activation runs are loaded before the stage wait so their latency overlaps
// it.  SAFE handles a partial stage (chunks past kc_n) and, on the bf16 path,
// a K tail that is not a whole chunk (k % 64 == 32); the fast path has no
// per-chunk tests.  On the fp16 path xr points at the token's fp16 row in
// shared memory (zero padded to whole chunks).
// XG (fp16 path only): the fp16 activations and the correction table come
// from global memory (xr = the prepared fp16 rows, tblg = the table) instead
// of this CTA's shared-memory staging.
// M1 (one token): only the MMA's column 0 -- token 0, in lanes t = 0 -- is
// live, so each group's scale goes onto the two live accumulators (rows g and
// g+8) with two plain FMAs instead of two packed pair FMAs over all four.
// XS (chain, one token, whole stage; implies XH, XG and M1): the stage holds,
// after its weights, the chunks' fp16 activation slice and their one-token
// zero-point entries ({z, z, 16 z, 16 z} per group, the MMA's accumulator
// input as it stands); both are read from shared memory after the stage wait.
template <int NT, bool SAFE, bool XH, bool COH = false, bool XG = false, bool M1 = false, bool XS = false>
__device__ __forceinline__ bool consume_stage(uint32_t stage, uint64_t *full, uint32_t phase, int kc0,
                                              int kc_n, int k, const uint16_t *const (&xr)[NT],
                                              const uint32_t (&xs)[NT], uint32_t tbl, int warp, int lane,
                                              float (&acc)[NT][4], const float4 *tblg = nullptr)
{
    static_assert(!XS || (NT == 1 && !SAFE && XH && XG && M1), "XS: one token, whole stage, fp16 path");
    // chunks whose activation runs are held in registers at once (bounds
    // the register file for 16-token tiles)
    constexpr int R = NT == 1 ? kChunksInFlight : 2;
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int c0 = 0; c0 < kCpw; c0 += R) {
        uint4 xf[R][NT][2];  // 8 K of group 0 and 8 K of group 1, per chunk
        if (XS && c0 == 0 && !xq4d::mbar_wait(full, phase)) return false;
#pragma unroll
        for (int c = 0; c < R; c++) {
            const int kc = kc0 + warp + (c0 + c) * kConsumerWarps;
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int G2 = 0; G2 < 2; G2++) {
                    const int kb = kc * XQ4G_KCHUNK + 32 * G2 + 8 * t;
                    if (XS) {
                        const int cl = warp + (c0 + c) * kConsumerWarps;  // chunk within the stage
                        xf[c][nt][G2] = xq4d::lds_v4(stage + kStageBytes + 2 * (cl * XQ4G_KCHUNK + 32 * G2 + 8 * t));
                    } else if (XH && XG) {
                        xf[c][nt][G2] = (!SAFE || kc < kc_n) ? xq4d::ldg_v4(xr[nt] + kb) : make_uint4(0, 0, 0, 0);
                    } else if (XH) {
                        xf[c][nt][G2] = (!SAFE || kc < kc_n) ? xq4d::lds_v4(xs[nt] + 2 * kb)
                                                             : make_uint4(0, 0, 0, 0);
                    } else if (!SAFE || (kc < kc_n && kb < k)) {
                        xf[c][nt][G2] = COH ? xq4d::ldcg_v4(xr[nt] + kb) : xq4d::ldg_v4(xr[nt] + kb);
                    } else {
                        xf[c][nt][G2] = make_uint4(0, 0, 0, 0);
                    }
                }
        }
        if (!XS && c0 == 0 && !xq4d::mbar_wait(full, phase)) return false;
        // fp16 path: zero-point corrections of the chunk's two groups; from
        // the prepared table (XG) they are the MMA's accumulator inputs as
        // they stand, {z(2t), z(2t+1), 16 z(2t), 16 z(2t+1)} per group
        float4 zc[R][2];
        if (XH) {
#pragma unroll
            for (int c = 0; c < R; c++) {
                const int kc = kc0 + warp + (c0 + c) * kConsumerWarps;
                const bool in = !SAFE || kc < kc_n;
                if (XS) {
                    const int cl = warp + (c0 + c) * kConsumerWarps;
                    zc[c][0] = xq4d::lds_f4(stage + kStageBytes + kStageXBytes + 32 * cl);
                    zc[c][1] = xq4d::lds_f4(stage + kStageBytes + kStageXBytes + 32 * cl + 16);
                } else if (XG) {
                    zc[c][0] = in ? xq4d::ldg_f4(tblg + (kc * 4 + t) * 2) : make_float4(0.f, 0.f, 0.f, 0.f);
                    zc[c][1] = in ? xq4d::ldg_f4(tblg + (kc * 4 + t) * 2 + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
                } else {
                    zc[c][0] = in ? xq4d::lds_f4(tbl + 16 * (kc * 4 + t)) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        uint4 cw[R];
        uint2 sw[R];
#pragma unroll
        for (int c = 0; c < R; c++) {
            const int cl = warp + (c0 + c) * kConsumerWarps;  // chunk within the stage
            const uint32_t up = stage + cl * XQ4G_UNIT_BYTES;
            if (!SAFE || kc0 + cl < kc_n) {
                cw[c] = xq4d::lds_v4(up + lane * 16);
                sw[c] = xq4d::lds_v2(up + XQ4G_CODE_BYTES + g * 8);
            } else {
                cw[c] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);  // q = 0
                sw[c] = make_uint2(0, 0);
            }
        }
#pragma unroll
        for (int c = 0; c < R; c++) {
            const uint32_t words[4] = {cw[c].x, cw[c].y, cw[c].z, cw[c].w};
#pragma unroll
            for (int G2 = 0; G2 < 2; G2++) {
                const uint32_t sg = G2 ? sw[c].y : sw[c].x;
                const float s_lo = __uint_as_float(sg << 16);    // row g
                float s_hi = __uint_as_float(sg & 0xFFFF0000u);  // row g+8
                uint32_t a0[4], a1[4];
                if (XH) {  // rows g+8 carry 16*c (unpack_word_c16): their sums are 16x until the row block ends
                    xq4d::unpack_word_c16(words[2 * G2], a0);
                    xq4d::unpack_word_c16(words[2 * G2 + 1], a1);
                } else {
                    xq4d::unpack_word_q(words[2 * G2], a0);
                    xq4d::unpack_word_q(words[2 * G2 + 1], a1);
                }
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    float tacc[4];
                    if (XH) {
                        // accumulator starts at -8 * sum(x) of the group
                        // (x 2^-24; x 16 for rows g+8): the MMA then yields
                        // 2^-24 * sum((c - 8) * x) = 2^-24 * sum(q * x)
                        float cin[4];
                        if (XG) {
                            cin[0] = zc[c][G2].x;
                            cin[1] = zc[c][G2].y;
                            cin[2] = zc[c][G2].z;
                            cin[3] = zc[c][G2].w;
                        } else {
                            const float z0 = G2 ? zc[c][0].z : zc[c][0].x, z1 = G2 ? zc[c][0].w : zc[c][0].y;
                            cin[0] = z0;
                            cin[1] = z1;
                            cin[2] = 16.f * z0;
                            cin[3] = 16.f * z1;
                        }
                        xq4d::mma_f16_16816_c(tacc, a0, xf[c][nt][G2].x, xf[c][nt][G2].y, cin);
                        xq4d::mma_f16_16816(tacc, a1, xf[c][nt][G2].z, xf[c][nt][G2].w);
                    } else {
                        xq4d::mma_bf16_16816_z(tacc, a0, xf[c][nt][G2].x, xf[c][nt][G2].y);
                        xq4d::mma_bf16_16816(tacc, a1, xf[c][nt][G2].z, xf[c][nt][G2].w);
                    }
                    if (M1) {
                        acc[nt][0] = __fmaf_rn(s_lo, tacc[0], acc[nt][0]);
                        acc[nt][2] = __fmaf_rn(s_hi, tacc[2], acc[nt][2]);
                    } else {
                        xq4d::ffma2(acc[nt][0], acc[nt][1], s_lo, tacc[0], tacc[1]);
                        xq4d::ffma2(acc[nt][2], acc[nt][3], s_hi, tacc[2], tacc[3]);
                    }
                }
            }
        }
    }
    return true;
}

// Power-of-two exponent that brings a token's max |x| (bf16 magnitude bits)
// into [2^14, 2^15); 0 for an all-zero token.
__device__ __forceinline__ int tok_exponent(unsigned mx)
{
    const int ex = (int)(mx >> 7) - 127;  // exponent of the max
    return mx == 0 ? 0 : min(max(14 - ex, -252), 254);
}

// 2^e as a product of two normal floats (e in [-252, 254]).
__device__ __forceinline__ void pow2_split(int e, float &f1, float &f2)
{
    const int e1 = e / 2, e2 = e - e1;
    f1 = __int_as_float((e1 + 127) << 23);
    f2 = __int_as_float((e2 + 127) << 23);
}

// Poison a communicator whose peer wait ran out: this rank's word, every
// peer's word and the host-mapped flag (idempotent plain stores).
__device__ __forceinline__ void p2p_poison(const xq4_p2p_poison &p, int nranks)
{
    for (int q = 0; q < nranks; q++)
        if (p.word[q]) xq4d::st_sys_u32(p.word[q], 1u);
    if (p.host) xq4d::st_sys_u32(p.host, 1u);
}

// Lane 0 reads this rank's poison word and the warp agrees on it; a poisoned
// communicator exchanges nothing, raises fault bit 0x8 and flags the host.
__device__ __forceinline__ bool p2p_usable(const xq4_p2p_poison &p, int rank, int lane)
{
    unsigned v = lane == 0 ? xq4d::ld_sys_u32(p.word[rank]) : 0u;
    v = __shfl_sync(0xffffffffu, v, 0);
    if (v && lane == 0) {
        atomicOr(&g_xq4_fault, XQ4_FAULT_PEER_WAIT);
        if (p.host) xq4d::st_sys_u32(p.host, 1u);
    }
    return v == 0u;
}

// Copy the peers' words i = tid, tid + nthr, ... < total_w of an inbox
// (value bits | epoch << 32) into y (bf16 or f32 values) once each carries
// epoch e; idx_of(i) gives word i's index in the inbox half and in y (the same
// [tok][n_total] position; below XQ4_FUSED_MAX_VALUES).  Eight loads per
// thread are in flight together: one at a time, the loop cost a round trip
// to memory per nthr words.  False when a word is still stale after the
// bounded wait (2 s from t0).
template <class IdxF>
__device__ __forceinline__ bool gather_inbox(const unsigned long long *in, unsigned e, int total_w, int tid,
                                             int nthr, uint64_t t0, bool out_f32, void *y, IdxF idx_of)
{
    constexpr int kBatch = 8;
    for (int i0 = tid; i0 < total_w; i0 += nthr * kBatch) {
        int idx[kBatch];
        unsigned long long w[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
            const int i = i0 + nthr * j;
            idx[j] = i < total_w ? idx_of(i) : -1;
            w[j] = idx[j] >= 0 ? xq4d::ld_sys_u64(in + idx[j]) : 0ull;
        }
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
            if (idx[j] < 0) continue;
            while ((unsigned)(w[j] >> 32) != e) {
                if (xq4d::global_ns() - t0 > 2000000000ull) return false;
                __nanosleep(32);
                w[j] = xq4d::ld_sys_u64(in + idx[j]);
            }
            if (out_f32)
                reinterpret_cast<uint32_t *>(y)[idx[j]] = (uint32_t)w[j];
            else
                reinterpret_cast<uint16_t *>(y)[idx[j]] = (uint16_t)w[j];
        }
    }
    return true;
}

template <int NT, bool XH, bool P2P>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
gemv_kernel(const uint8_t *__restrict__ pack, int n, int k, int nb, int kc_n,
            const uint16_t *__restrict__ x, int m, void *__restrict__ y, int out_f32,
            const __grid_constant__ xq4_p2p_out p2p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kStages;
    uint64_t *red_full = empty + kStages;     // [kRedBufs]: all 16 partials written
    uint64_t *red_free = red_full + kRedBufs;  // [kRedBufs]: reduction done, buffer reusable
    float *red = reinterpret_cast<float *>(smem + kBarBytes);
    unsigned *tok_max = reinterpret_cast<unsigned *>(smem + xh_offset(NT));  // fp16 path: [8] max |x| bits
    uint16_t *xh = reinterpret_cast<uint16_t *>(smem + xh_offset(NT) + 64);  // fp16 path: [m][kp]
    float4 *tbl = reinterpret_cast<float4 *>(smem + tbl_offset(NT, m, kc_n));  // fp16 path: [kc][4]
    uint8_t *ring = smem + ring_offset(NT, XH, m, kc_n);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int rb0 = (int)((long long)cta * nb / G), rb1 = (int)((long long)(cta + 1) * nb / G);
    const int spr = (kc_n + kStageChunks - 1) / kStageChunks;  // stages per row block
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
        if (XH)
            for (int i = 0; i < 8; i++) tok_max[i] = 0;
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
        // Row block rbl's 8 partials arrive in buffer rbl % kRedBufs; sum
        // them in warp order (deterministic), write the 16 rows, free the
        // buffer.  The consumers never wait for this unless all buffers are
        // still being reduced.
        xq4d::grid_dep_wait();
        // P2P: this call's epoch (the previous fused launch on this rank
        // completed before grid_dep_wait returned) and its inbox half
        const unsigned e = P2P ? *reinterpret_cast<volatile const unsigned *>(p2p.epoch) + 1u : 0u;
        const size_t half = P2P ? (size_t)(e & 1u) * p2p.half_words : 0;
        // a poisoned communicator (an earlier call gave up on a peer): local rows only
        const bool xchg = P2P && p2p_usable(p2p.poison, p2p.rank, lane);
        const float *red_c = red;
        bool alive = true;
        for (int rbl = 0; rbl < rb1 - rb0; rbl++) {
            const int buf = rbl % kRedBufs;
            const uint32_t use = (uint32_t)(rbl / kRedBufs);
            if (!xq4d::mbar_wait(&red_full[buf], use & 1)) {
                atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                alive = false;  // P2P: still counted below, so the epoch advances
                break;
            }
            const float *rd = red_c + (size_t)buf * kConsumerWarps * NT * 128;  // [warp][tok][row]
            const int rb = rb0 + rbl;
            for (int o = lane; o < m * 16; o += 32) {  // o = tok * 16 + row
                const int tok = o >> 4, r = o & 15;
                float sum = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; w++) sum += rd[(size_t)w * NT * 128 + o];
                const int row = rb * XQ4G_ROWS + r;
                if (row < n) {
                    if (XH) {  // undo 2^-24 and the token's power of two (exact)
                        float f1, f2;
                        pow2_split(24 - tok_exponent(tok_max[tok]), f1, f2);
                        sum = sum * f1 * f2;
                    }
                    if (P2P) {  // this rank's row: the local full output + one word per peer
                        const size_t idx = (size_t)tok * p2p.n_total + p2p.row_off + row;
                        uint32_t bits;
                        if (out_f32) {
                            reinterpret_cast<float *>(y)[idx] = sum;
                            bits = __float_as_uint(sum);
                        } else {
                            const __nv_bfloat16 h = __float2bfloat16_rn(sum);
                            reinterpret_cast<__nv_bfloat16 *>(y)[idx] = h;
                            bits = __bfloat16_as_ushort(h);
                        }
                        const unsigned long long word = ((unsigned long long)e << 32) | bits;
                        for (int q = 0; xchg && q < p2p.nranks; q++)
                            if (q != p2p.rank) xq4d::st_sys_u64(p2p.inbox[q] + half + idx, word);
                    } else if (out_f32) {
                        reinterpret_cast<float *>(y)[(size_t)tok * n + row] = sum;
                    } else {
                        reinterpret_cast<__nv_bfloat16 *>(y)[(size_t)tok * n + row] = __float2bfloat16_rn(sum);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(&red_free[buf]);
        }
        if (P2P) {
            // The peers' rows of this CTA's row range (their CTA with the
            // same index computes them: equal shards, equal grids), from the
            // inbox into the full output.  Every CTA sends all its words
            // before it waits, so no wait depends on a waiting CTA.
            const int r0 = rb0 * XQ4G_ROWS, span = min(rb1 * XQ4G_ROWS, n) - r0;
            const unsigned long long *in = p2p.inbox[p2p.rank] + half;
            const int per_peer = m * span, total_w = (p2p.nranks - 1) * per_peer;
            const uint64_t t0 = xq4d::global_ns();
            if (alive && xchg &&
                !gather_inbox(in, e, total_w, lane, 32, t0, out_f32 != 0, y, [&](int i) {
                    const int qi = i / per_peer, rem = i - qi * per_peer;
                    const int tok = rem / span, row = r0 + (rem - tok * span);
                    const int q = qi < p2p.rank ? qi : qi + 1;
                    return tok * p2p.n_total + q * n + row;
                })) {
                atomicOr(&g_xq4_fault, XQ4_FAULT_PEER_WAIT);
                p2p_poison(p2p.poison, p2p.nranks);
            }
            // the last CTA of this launch advances the epoch: every CTA has
            // read it by the time it counts itself here
            __syncwarp();
            if (lane == 0 && atomicAdd(p2p.cnt, 1u) == gridDim.x - 1) {
                *p2p.cnt = 0u;
                *reinterpret_cast<volatile unsigned *>(p2p.epoch) = e;
            }
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    xq4d::grid_dep_wait();  // x is written, y may be read, by the neighbouring kernels

    if (XH) {
        // Stage x as fp16 with a per-token power of two: max|x| * 2^e lies in
        // [2^14, 2^15).  One pass: every consumer thread loads its 16-byte
        // runs of the flat [m][k] activation into registers (all loads in
        // flight together), the per-token maxima meet in shared memory, and
        // the same registers are scaled, converted and stored.  k is a
        // multiple of 32, so a run never straddles a token.
        constexpr int kRuns = (kXhMaxElems / 8 + kConsumerThreads - 1) / kConsumerThreads;
        const int runs = k / 8, total_runs = m * runs;
        uint4 v[kRuns];
#pragma unroll
        for (int j = 0; j < kRuns; j++) {
            const int r = threadIdx.x + j * kConsumerThreads;
            v[j] = r < total_runs ? xq4d::ldg_v4(x + 8 * (size_t)r) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < kRuns; j++) {
            if (j * kConsumerThreads >= total_runs) break;  // uniform across the block
            const int r = min(threadIdx.x + j * kConsumerThreads, total_runs - 1);
            const int tok = r / runs;
            const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
            unsigned mx = 0;  // max |x| as bf16 magnitude bits (ordered like the values)
#pragma unroll
            for (int h = 0; h < 4; h++) mx = max(mx, max(w[h] & 0x7FFFu, (w[h] >> 16) & 0x7FFFu));
            const int tok0 = __shfl_sync(0xffffffffu, tok, 0);
            if (__all_sync(0xffffffffu, tok == tok0)) {  // the warp's runs are one token's
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if (lane == 0 && mx) atomicMax(&tok_max[tok0], mx);
            } else if (mx) {
                atomicMax(&tok_max[tok], mx);
            }
        }
        float *tblf = reinterpret_cast<float *>(tbl);
        for (int i = threadIdx.x; i < kc_n * 16; i += kConsumerThreads) tblf[i] = 0.f;
        xq4d::named_bar_sync(1, kConsumerThreads);
        // Convert, store, and sum each 32-K group of the staged values (the
        // four runs of a group sit in four consecutive lanes): the zero-point
        // correction table entry (chunk, lane quad t) holds -8 * 2^-24 *
        // {X(G0, 2t), X(G0, 2t+1), X(G1, 2t), X(G1, 2t+1)}, X = group sum.
#pragma unroll
        for (int j = 0; j < kRuns; j++) {
            if (j * kConsumerThreads >= total_runs) break;  // uniform across the block
            const int r = threadIdx.x + j * kConsumerThreads;
            float part = 0.f;
            int tok = 0, kk = 0;
            if (r < total_runs) {
                tok = r / runs;
                kk = 8 * (r - tok * runs);
                float f1, f2;
                pow2_split(tok_exponent(tok_max[tok]), f1, f2);
                const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
                uint32_t h2[4];
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    const float lo = __uint_as_float(w[h] << 16) * f1 * f2;
                    const float hi = __uint_as_float(w[h] & 0xFFFF0000u) * f1 * f2;
                    const __half2 p = __floats2half2_rn(lo, hi);
                    h2[h] = *reinterpret_cast<const uint32_t *>(&p);
                    const float2 pf = __half22float2(p);
                    part += pf.x + pf.y;
                }
                *reinterpret_cast<uint4 *>(xh + (size_t)tok * kp + kk) = make_uint4(h2[0], h2[1], h2[2], h2[3]);
            }
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            if (r < total_runs && (r & 3) == 0) {
                const int grp = kk >> 5;  // group index along K
                tblf[((grp >> 1) * 4 + (tok >> 1)) * 4 + (grp & 1) * 2 + (tok & 1)] = -8.f * 0x1p-24f * part;
            }
        }
        // zero the K padding of every token (k % 64 == 32: one half chunk)
        const int pad_runs = (kp - k) / 8;
        for (int i = threadIdx.x; i < m * pad_runs; i += kConsumerThreads)
            *reinterpret_cast<uint4 *>(xh + (size_t)(i / pad_runs) * kp + k + 8 * (i % pad_runs)) =
                make_uint4(0, 0, 0, 0);
        xq4d::named_bar_sync(1, kConsumerThreads);
    }

    const int g = lane >> 2, t = lane & 3;
    // B column g of the mma is token g (+8*nt).  A column past m only feeds
    // output columns that are never written, so those lanes read token 0's
    // row instead of being predicated off.
    const uint16_t *xr[NT];
    uint32_t xs[NT];  // fp16 path: shared addresses of the token rows
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int tok = g + 8 * nt;
        xr[nt] = XH ? xh + (size_t)(tok < m ? tok : 0) * kp : x + (size_t)(tok < m ? tok : 0) * k;
        xs[nt] = XH ? xq4d::smem_u32(xr[nt]) : 0u;
    }
    const uint32_t tbl_s = xq4d::smem_u32(tbl), ring_s = xq4d::smem_u32(ring);
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;

    int slot = 0, rbl = 0, kc0 = 0;
    uint32_t phase = 0;
    const bool k_whole = (k % XQ4G_KCHUNK) == 0;
    for (int i = 0; i < total; i++) {
        const uint32_t stage = ring_s + (uint32_t)slot * kStageBytes;
        const bool fast = (XH || k_whole) && kc0 + kStageChunks <= kc_n;
        bool ok;
#ifndef XQ4_CHAIN_NO_M1
        if (NT == 1 && m == 1 && fast)  // one token: the M1 form
            ok = consume_stage<NT, false, XH, false, false, true>(stage, &full[slot], phase, kc0, kc_n, k, xr, xs, tbl_s,
                                                                  warp, lane, acc);
        else
#endif
            ok = fast ? consume_stage<NT, false, XH>(stage, &full[slot], phase, kc0, kc_n, k, xr, xs, tbl_s, warp, lane, acc)
                      : consume_stage<NT, true, XH>(stage, &full[slot], phase, kc0, kc_n, k, xr, xs, tbl_s, warp, lane, acc);
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
            // Every warp leaves its partial in buffer rbl % kRedBufs and moves
            // on; the reducer warp sums them.  A warp waits only before
            // reusing a buffer whose reduction is still running.
            kc0 = 0;
            const int buf = rbl % kRedBufs;
            const uint32_t use = (uint32_t)(rbl / kRedBufs);
            if (use > 0 && !xq4d::mbar_wait(&red_free[buf], (use - 1) & 1)) {
                atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                return;
            }
            float *rd = red + (size_t)buf * kConsumerWarps * NT * 128;  // [warp][tok][row]
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float *r = rd + (size_t)warp * NT * 128 + (size_t)nt * 128;
                const float hs = XH ? 0.0625f : 1.f;  // fp16 path: rows g+8 summed 16 * c
                r[(2 * t) * 16 + g] = acc[nt][0];
                r[(2 * t + 1) * 16 + g] = acc[nt][1];
                r[(2 * t) * 16 + g + 8] = acc[nt][2] * hs;
                r[(2 * t + 1) * 16 + g + 8] = acc[nt][3] * hs;
                acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
            }
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(&red_full[buf]);
            rbl++;
        }
    }
}

// ------------------------------------------------------------------ GEMV chain
// One persistent launch over a list of GEMVs (m <= 8 each, bf16 path), the
// B200 form of the reference's chained op submission (crates/xnpu-cli/src/
// main.rs:1611-1635, and the projection stream of cmd_run_w4layer,
// main.rs:2487-2499).  Same warp roles as gemv_kernel.  CTA c owns one
// contiguous share of each segment's row blocks (its visits, below); the
// producer streams visit after visit through one ring, so the next op's
// weights are already in flight while the
// consumers finish the current one, and the per-launch ramp and tail of
// separate kernels happen once per chain.  An op marked wait_prev starts a
// segment and reads its x only after every CTA has written the previous
// segment's outputs: the reducers count the CTAs done with each segment
// (release), one consumer thread per CTA waits for the count (acquire,
// bounded) and releases the other consumer warps through an mbarrier.  x is
// then read through L2 (ld.global.cg): it may have been written earlier in
// the same launch.
#ifndef XQ4_CHAIN_STAGES
#define XQ4_CHAIN_STAGES 4
#endif
constexpr int kChainStages = XQ4_CHAIN_STAGES;
static_assert(kStageChunks == XQ4_GEMV_STAGE_CHUNKS_ABI, "the host splits chain work in these stages");
// A chain stage: the weights of kStageChunks chunks, then, for a one-token
// fp16-path op, the slices of its activation image (kStageChunks * 64 fp16)
// and of its one-token zero-point table (kStageChunks * 2 float4) that those
// chunks read -- copied in by the same bulk-copy engine, so that the
// consumers' hot loop reads shared memory only.
constexpr int kChainXBytes = kStageXBytes;
constexpr int kChainTBytes = kStageChunks * 2 * 16;
constexpr int kChainStageBytes = kStageBytes + kChainXBytes + kChainTBytes;
// ring full/empty, reduce full/free, and the consumers' op barrier
constexpr int kChainBarBytes = ((2 * kChainStages + 2 * kRedBufs + 1) * 8 + 127) & ~127;
constexpr size_t kChainRingOff = kChainBarBytes + (size_t)kRedBufs * kConsumerWarps * 128 * 4;
constexpr size_t kChainSmem = kChainRingOff + (size_t)kChainStages * kChainStageBytes;
static_assert(kChainStageBytes % 128 == 0, "stage alignment");
static_assert(kChainRingOff % 128 == 0, "ring alignment");
static_assert((kChainSmem + 1024) * kCtasPerSm <= 228 * 1024, "kCtasPerSm chain CTAs per SM");

// A CTA's work is its list of visits, built at chain create: one per op in
// which it owns row blocks, {op, rb0, rb1, seg << 2 | last << 1 | first}
// (first / last: the CTA's first / last visit in segment seg).  CTA c owns the
// row blocks whose first stage falls in its share [c*U/G, (c+1)*U/G) of its
// segment's U stages, so in a long chain of independent ops it visits one or
// two ops: walking every op instead (a table load, and for the reducer a
// release, per op) delayed the last CTAs' first stage by microseconds per op.
constexpr int kVisitFirst = 1, kVisitLast = 2;

// Prep for the chain's fp16 path: one CTA per activation converts it as the
// single-op GEMV's fp16 staging does (the same per-token power of two, the
// same conversions and the same order of the group sums, so the outputs are
// bit-identical to that path), into global memory.
constexpr int kPrepThreads = 256;

__global__ void __launch_bounds__(kPrepThreads)
chain_prep_kernel(const xq4_chain_prep_dev *__restrict__ preps)
{
    // let the chain launch now (its producers stream weights meanwhile; its
    // consumers wait for this grid); x may come from the preceding kernel
    xq4d::grid_dep_launch();
    xq4d::grid_dep_wait();
    const xq4_chain_prep_dev p = preps[blockIdx.x];
    const uint16_t *x = reinterpret_cast<const uint16_t *>(p.x);
    const int kp = p.kc * XQ4G_KCHUNK, runs = p.k / 8, total_runs = p.m * runs;
    __shared__ unsigned smax[8];
    __shared__ float sinv[8];
    if (threadIdx.x < 8) smax[threadIdx.x] = 0u;
    if (p.w4a8) {  // groups past K and tokens past m keep zero entries
        for (int i = threadIdx.x; i < p.kc * 2 * 8; i += kPrepThreads) p.qtbl[i] = make_int2(0, 0);
    } else {
        for (int i = threadIdx.x; i < p.kc * 32; i += kPrepThreads) p.tbl[i] = 0.f;
        if (p.m == 1)  // a half chunk's missing group keeps a zero entry
            for (int i = threadIdx.x; i < p.kc * 2; i += kPrepThreads) p.tbl1[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (p.norm) {
        // RMSNorm (crates/xnpu-cli/src/main.rs:4714-4724), inv = 1 / sqrt(mean
        // of squares + eps), with the sum of squares in a fixed order, so the
        // result is the same on every run: thread i sums its runs i, i + 256,
        // ... (each run's 8 values in order), a butterfly adds a warp's 32
        // sums, thread 0 adds the 8 warps' sums in warp order.  Every thread
        // has its runs' loads in flight together.
        __shared__ float wsum[kPrepThreads / 32];
        const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int tk = 0; tk < p.m; tk++) {
            float ss = 0.f;
#pragma unroll 4
            for (int r = threadIdx.x; r < runs; r += kPrepThreads) {
                const uint4 v = xq4d::ldcg_v4(x + (size_t)tk * p.k + 8 * (size_t)r);
                const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    const float lo = __uint_as_float(wd[h] << 16), hi = __uint_as_float(wd[h] & 0xFFFF0000u);
                    ss = __fadd_rn(ss, __fmul_rn(lo, lo));
                    ss = __fadd_rn(ss, __fmul_rn(hi, hi));
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
            if (lane == 0) wsum[w] = ss;
            __syncthreads();
            if (threadIdx.x == 0) {
                float t = 0.f;
                for (int i = 0; i < kPrepThreads / 32; i++) t = __fadd_rn(t, wsum[i]);
                sinv[tk] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)p.k), p.eps)));
            }
            __syncthreads();
        }
    }
    __syncthreads();
    // one run of 8 activations (of token `tok`, starting at element kk), as
    // the GEMV consumes them: normalised first when the op asks for it
    const auto run_words = [&](int r, int tok, int kk, uint32_t (&w)[4]) {
        const uint4 v = xq4d::ldcg_v4(x + 8 * (size_t)r);
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
        if (p.norm) {
            const float inv = sinv[tok];
            const uint4 g = *reinterpret_cast<const uint4 *>(p.norm_w + kk);
            const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const float lo = __fmul_rn(__fmul_rn(__uint_as_float(w[h] << 16), inv), __uint_as_float(gw[h] << 16));
                const float hi = __fmul_rn(__fmul_rn(__uint_as_float(w[h] & 0xFFFF0000u), inv),
                                           __uint_as_float(gw[h] & 0xFFFF0000u));
                w[h] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
                       ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
            }
        }
    };
    for (int r = threadIdx.x; r < total_runs; r += kPrepThreads) {
        const int tok = r / runs;
        uint32_t w[4];
        run_words(r, tok, 8 * (r - tok * runs), w);
        unsigned mx = 0;
#pragma unroll
        for (int h = 0; h < 4; h++) mx = max(mx, max(w[h] & 0x7FFFu, (w[h] >> 16) & 0x7FFFu));
        if (mx) atomicMax(&smax[tok], mx);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    if (p.w4a8) {
        // W4A8: per 32-K group (four consecutive runs, four neighbouring
        // lanes) the reference's quantizer (w4u_quantize_x, main.rs:2955-2986):
        // d = RNE_bf16(max|x| / 127), q = clamp(rne(x / d), -127, 127); an
        // all-zero group gives q = 0 and d = 0.  q is stored with its bytes
        // in the integer MMA's slot order (0, 2, 1, 3 within each 4), the
        // table entry is {-8 * sum(q), f32 bits of d} per (group, token).
        for (int base = 0; base < total_runs; base += kPrepThreads) {  // uniform trip count: shuffles below
            const int r = base + threadIdx.x;
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            int tok = 0, kk = 0;
            if (r < total_runs) {
                tok = r / runs;
                kk = 8 * (r - tok * runs);
                uint32_t w[4];
                run_words(r, tok, kk, w);
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    v[2 * h] = __uint_as_float(w[h] << 16);
                    v[2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
                }
            }
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            uint32_t qb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int qs = 0;
            float df = 0.f;
            if (amax != 0.f) {
                df = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(amax, 127.f)));
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int q = (int)fminf(fmaxf(rintf(__fdiv_rn(v[i], df)), -127.f), 127.f);
                    qs += q;
                    qb[i] = (uint32_t)q & 0xFFu;
                }
            }
            qs += __shfl_xor_sync(0xffffffffu, qs, 1);
            qs += __shfl_xor_sync(0xffffffffu, qs, 2);
            if (r < total_runs) {
                const uint32_t w0 = qb[0] | (qb[2] << 8) | (qb[1] << 16) | (qb[3] << 24);
                const uint32_t w1 = qb[4] | (qb[6] << 8) | (qb[5] << 16) | (qb[7] << 24);
                *reinterpret_cast<uint2 *>(p.qx + (size_t)tok * kp + kk) = make_uint2(w0, w1);
                if ((lane & 3) == 0) p.qtbl[(size_t)(kk >> 5) * 8 + tok] = make_int2(-8 * qs, __float_as_int(df));
            }
        }
        const int pad_runs = (kp - p.k) / 8;
        for (int i = threadIdx.x; i < p.m * pad_runs; i += kPrepThreads)
            *reinterpret_cast<uint2 *>(p.qx + (size_t)(i / pad_runs) * kp + p.k + 8 * (i % pad_runs)) = make_uint2(0, 0);
        return;
    }
    for (int base = 0; base < total_runs; base += kPrepThreads) {  // uniform trip count: shuffles below
        const int r = base + threadIdx.x;
        float part = 0.f;
        int tok = 0, kk = 0;
        if (r < total_runs) {
            tok = r / runs;
            kk = 8 * (r - tok * runs);
            float f1, f2;
            pow2_split(tok_exponent(smax[tok]), f1, f2);
            uint32_t w[4];
            run_words(r, tok, kk, w);
            uint32_t h2[4];
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const float lo = __uint_as_float(w[h] << 16) * f1 * f2;
                const float hi = __uint_as_float(w[h] & 0xFFFF0000u) * f1 * f2;
                const __half2 hp = __floats2half2_rn(lo, hi);
                h2[h] = *reinterpret_cast<const uint32_t *>(&hp);
                const float2 pf = __half22float2(hp);
                part += pf.x + pf.y;
            }
            *reinterpret_cast<uint4 *>(p.img + (size_t)tok * kp + kk) = make_uint4(h2[0], h2[1], h2[2], h2[3]);
        }
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        if (r < total_runs && (lane & 3) == 0) {
            // (chunk, lane quad, group of the chunk): {z(2t), z(2t+1), 16 z(2t), 16 z(2t+1)}
            const int grp = kk >> 5;  // group index along K
            const float z = -8.f * 0x1p-24f * part;
            float *e = p.tbl + (((grp >> 1) * 4 + (tok >> 1)) * 2 + (grp & 1)) * 4 + (tok & 1);
            e[0] = z;
            e[2] = 16.f * z;
            if (p.m == 1) p.tbl1[grp] = make_float4(z, z, 16.f * z, 16.f * z);  // [chunk][group]
        }
    }
    const int pad_runs = (kp - p.k) / 8;  // k % 64 == 32: one half chunk per token
    for (int i = threadIdx.x; i < p.m * pad_runs; i += kPrepThreads)
        *reinterpret_cast<uint4 *>(p.img + (size_t)(i / pad_runs) * kp + p.k + 8 * (i % pad_runs)) = make_uint4(0, 0, 0, 0);
    if (threadIdx.x < 8) p.max[threadIdx.x] = smax[threadIdx.x];
}

// A chain stage of a W4A8 op: the integer tensor-core path of w4a8_kernel
// (gemv_w4a8.cu), operation for operation, with the activation from the
// prep's int8 image: per 32-K group one mma.m16n8k32 u8 x s8 of the raw
// codes against q_x, accumulator input -8 * sum(q_x), then
// acc += (s_w * d_x) * T in f32.
__device__ __forceinline__ bool consume_stage_w4a8(uint32_t stage, uint64_t *full, uint32_t phase, int kc0, int kc_n,
                                                   const uint8_t *xrow, const int2 *qtbl, int warp, int lane,
                                                   float (&acc)[4])
{
    const int g = lane >> 2, t = lane & 3;
    // two chunks at a time: their int8 activations and group entries (the
    // prep's output, L2-resident) are loaded before the stage wait and
    // before the chunks' code words, so the loads' latency overlaps it
    constexpr int R = 2;
#pragma unroll
    for (int c0 = 0; c0 < kCpw; c0 += R) {
        uint2 bx[R][2];
        uint4 ex[R][2];  // {cx(2t), d(2t), cx(2t+1), d(2t+1)}
#pragma unroll
        for (int c = 0; c < R; c++) {
            const int kc = kc0 + warp + (c0 + c) * kConsumerWarps;
#pragma unroll
            for (int G2 = 0; G2 < 2; G2++) {
                const int grp = kc * 2 + G2;
                bx[c][G2] = kc < kc_n ? xq4d::ldg_v2(xrow + grp * 32 + 8 * t) : make_uint2(0, 0);
                ex[c][G2] = kc < kc_n ? xq4d::ldg_v4(qtbl + grp * 8 + 2 * t) : make_uint4(0, 0, 0, 0);
            }
        }
        if (c0 == 0 && !xq4d::mbar_wait(full, phase)) return false;
#pragma unroll
        for (int c = 0; c < R; c++) {
            const int cl = warp + (c0 + c) * kConsumerWarps;  // chunk within the stage
            if (kc0 + cl >= kc_n) continue;
            const uint32_t up = stage + cl * XQ4G_UNIT_BYTES;
            const uint4 cw = xq4d::lds_v4(up + lane * 16);
            const uint2 sw = xq4d::lds_v2(up + XQ4G_CODE_BYTES + g * 8);
            const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
            for (int G2 = 0; G2 < 2; G2++) {
                const uint2 bb = bx[c][G2];
                const uint4 e = ex[c][G2];
                const uint32_t w0 = words[2 * G2], w1 = words[2 * G2 + 1];
                const uint32_t a[4] = {w0 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu,
                                       (w1 >> 4) & 0x0F0F0F0Fu};
                int T[4];
                xq4d::mma_u8s8_16832(T, a, bb.x, bb.y, (int)e.x, (int)e.z);
                const uint32_t sg = G2 ? sw.y : sw.x;
                const float s_lo = __uint_as_float(sg << 16), s_hi = __uint_as_float(sg & 0xFFFF0000u);
                const float d0 = __uint_as_float(e.y), d1 = __uint_as_float(e.w);
                acc[0] = fmaf(s_lo * d0, (float)T[0], acc[0]);
                acc[1] = fmaf(s_lo * d1, (float)T[1], acc[1]);
                acc[2] = fmaf(s_hi * d0, (float)T[2], acc[2]);
                acc[3] = fmaf(s_hi * d1, (float)T[3], acc[3]);
            }
        }
    }
    return true;
}

// The peers' rows of this CTA's ranges of the sharded ops among its visits
// [vf, vl] go from the inbox into y, threads tid = 0..nthr-1 sharing the
// words.  Each peer's CTA with this index computed them (equal shards, equal
// chains), and every CTA sends its words before it waits, so no wait depends
// on a waiting CTA.  A word still stale after the bounded wait raises fault
// bit 0x8 and poisons the communicator.
__device__ __forceinline__ void chain_gather(const xq4_chain_op_dev *__restrict__ ops, const xq4_chain_plan &plan,
                                             const xq4_chain_p2p &p2p, int vf, int vl, unsigned e, size_t half,
                                             int tid, int nthr)
{
    const uint64_t t0 = xq4d::global_ns();
    for (int s = vf; s <= vl; s++) {
        const int4 si = __ldg(plan.visits + s);
        const xq4_chain_op_dev so = ops[si.x];
        if (!so.shard) continue;
        // this CTA's output rows of the op (row pairs for SwiGLU; row blocks
        // hold 16 rows, so a range never splits a pair)
        const int sh = so.swiglu ? 1 : 0;
        const int r0 = (si.y * XQ4G_ROWS) >> sh, span = (min(si.z * XQ4G_ROWS, so.n) >> sh) - r0;
        if (span <= 0) continue;
        const int ns = so.n >> sh;
        const size_t stride = (size_t)so.n_total >> sh;
        const unsigned long long *in = p2p.inbox[p2p.rank] + half + so.inbox_off;
        const int per_peer = so.m * span, total_w = (p2p.nranks - 1) * per_peer;
        if (!gather_inbox(in, e, total_w, tid, nthr, t0, so.out_f32 != 0, so.y, [&](int i) {
                const int qi = i / per_peer, rem = i - qi * per_peer;
                const int tok = rem / span, row = r0 + (rem - tok * span);
                const int q = qi < p2p.rank ? qi : qi + 1;
                return (int)(tok * stride) + q * ns + row;
            })) {
            atomicOr(&g_xq4_fault, XQ4_FAULT_PEER_WAIT);
            p2p_poison(p2p.poison, p2p.nranks);
            return;
        }
    }
}

// W8: the chain holds W4A8 ops.  The W4A8 path is compiled only into that
// instantiation: inside the register-capped fp16 kernel it cost the fp16 ops
// 6 % (measured on B200, the 32-layer decode set).
template <bool W8>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
gemv_chain_kernel(const xq4_chain_op_dev *__restrict__ ops, const __grid_constant__ xq4_chain_plan plan,
                  const __grid_constant__ xq4_chain_p2p p2p)
{
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kChainStages;
    uint64_t *red_full = empty + kChainStages;
    uint64_t *red_free = red_full + kRedBufs;
    uint64_t *op_bar = red_free + kRedBufs;  // consumers meet here before an op that waits
    float *red = reinterpret_cast<float *>(smem + kChainBarBytes);
    uint8_t *ring = smem + kChainRingOff;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int v0 = __ldg(plan.vstart + cta), v1 = __ldg(plan.vstart + cta + 1);  // this CTA's visits
    unsigned *const done = plan.done;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kChainStages; s++) {
            xq4d::mbar_init(&full[s], 1);
            xq4d::mbar_init(&empty[s], kConsumerWarps);
        }
        for (int b = 0; b < kRedBufs; b++) {
            xq4d::mbar_init(&red_full[b], kConsumerWarps);
            xq4d::mbar_init(&red_free[b], 1);
        }
        xq4d::mbar_init(op_bar, kConsumerWarps);
        xq4d::fence_barrier_init();
    }
    __syncthreads();
    xq4d::grid_dep_launch();

    if (warp == kProducerWarp) {  // ------------------------------ producer
        if (lane == 0) {
            int slot = 0, i = 0;
            uint32_t phase = 0;
            bool alive = true;
            bool prep_done = false;  // the x and table slices are the prep kernel's output
            for (int v = v0; v < v1 && alive; v++) {
                const int4 vi = __ldg(plan.visits + v);
                const xq4_chain_op_dev op = ops[vi.x];
                const int rb0 = vi.y, rb1 = vi.z;
                for (int rb = rb0; rb < rb1 && alive; rb++) {
                    for (int kc0 = 0; kc0 < op.kc; kc0 += kStageChunks, i++) {
                        if (i >= kChainStages && !xq4d::mbar_wait(&empty[slot], phase ^ 1)) {
                            atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_EMPTY);
                            alive = false;
                            break;
                        }
                        const int cnt = min(kStageChunks, op.kc - kc0);
                        const uint32_t bytes = (uint32_t)cnt * XQ4G_UNIT_BYTES;
                        // one-token fp16 op, whole stage: its x and table slices come along
                        const bool xs = op.xh && op.m == 1 && cnt == kStageChunks;
                        uint8_t *dst = ring + (size_t)slot * kChainStageBytes;
                        xq4d::mbar_arrive_expect_tx(&full[slot], bytes + (xs ? kChainXBytes + kChainTBytes : 0));
                        xq4d::bulk_g2s(dst, op.pack + ((size_t)rb * op.kc + kc0) * XQ4G_UNIT_BYTES, bytes, &full[slot]);
                        if (xs) {
                            if (!prep_done) {  // weights stream before this; the slices only after the prep
                                xq4d::grid_dep_wait();
                                prep_done = true;
                            }
                            xq4d::bulk_g2s(dst + kStageBytes, op.xh_img + (size_t)kc0 * XQ4G_KCHUNK, kChainXBytes,
                                           &full[slot]);
                            xq4d::bulk_g2s(dst + kStageBytes + kChainXBytes, op.xh_tbl1 + (size_t)kc0 * 2, kChainTBytes,
                                           &full[slot]);
                        }
                        if (++slot == kChainStages) {
                            slot = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
        }
        return;
    }

    if (warp == kReducerWarp) {  // ------------------------------ reducer
        xq4d::grid_dep_wait();
        // sharded ops: this launch's inbox epoch (the communicator's previous
        // inbox user on this stream completed before grid_dep_wait returned)
        const unsigned e = p2p.nranks > 1 ? *reinterpret_cast<volatile const unsigned *>(p2p.epoch) + 1u : 0u;
        const size_t half = p2p.nranks > 1 ? (size_t)(e & 1u) * p2p.half_words : 0;
        // a poisoned communicator (an earlier call gave up on a peer): local rows only
        const bool xchg = p2p.nranks > 1 && p2p_usable(p2p.poison, p2p.rank, lane);
        int rbl = 0, pend = v0;  // visits [pend, v] may hold sharded rows whose peer copies are not in y yet
        bool alive = true;
        for (int v = v0; v < v1; v++) {
            const int4 vi = __ldg(plan.visits + v);
            const xq4_chain_op_dev op = ops[vi.x];
            const int rb0 = vi.y, rb1 = vi.z, seg = vi.w >> 2;
            // output row stride and this rank's first output row (a SwiGLU op
            // writes one value per row pair)
            const size_t ystride = (size_t)(op.shard ? op.n_total : op.n) >> (op.swiglu ? 1 : 0);
            const int yoff = op.shard ? (op.row_off >> (op.swiglu ? 1 : 0)) : 0;
            for (int rb = rb0; alive && rb < rb1; rb++) {
                // the row block's outputs o = base + lane (o = tok * 16 + row
                // in the block), j = base / 32: the sum of the 8 consumer
                // warps' partials in warp order; for a W4A8 op, over the row
                // block's stages (2048-K chunks), each chunk's sum rounded to
                // bf16 and the partials added in f32 in chunk order, as
                // w4a8_kernel (the reference's w4u_read_c, main.rs:3066-3091)
                float val[4] = {0.f, 0.f, 0.f, 0.f};
                // a residual no op of this chain writes: loaded before the
                // consumers hand over the row block
                float resv[4] = {0.f, 0.f, 0.f, 0.f};
                if (op.residual && op.res_ext) {
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int oo = 32 * j + lane, row = rb * XQ4G_ROWS + (oo & 15);
                        if (oo < op.m * 16 && row < op.n)
                            resv[j] = __uint_as_float((uint32_t)xq4d::ldcg_u16(op.residual + (size_t)(oo >> 4) * op.n + row)
                                                      << 16);
                    }
                }
                const int nst = (W8 && op.w4a8) ? op.spr : 1;
                for (int st = 0; st < nst; st++, rbl++) {
                    const int buf = rbl % kRedBufs;
                    const uint32_t use = (uint32_t)(rbl / kRedBufs);
                    if (!xq4d::mbar_wait(&red_full[buf], use & 1)) {
                        atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                        alive = false;  // still counted below, so no other CTA waits on this one
                        break;
                    }
                    const float *rd = red + (size_t)buf * kConsumerWarps * 128;  // [warp][tok][row]
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int oo = 32 * j + lane;
                        if (oo < op.m * 16) {
                            float sum = 0.f;
#pragma unroll
                            for (int w = 0; w < kConsumerWarps; w++) sum += rd[(size_t)w * 128 + oo];
                            if (W8 && op.w4a8) {
                                const float part = __bfloat162float(__float2bfloat16_rn(sum));
                                val[j] = st == 0 ? part : val[j] + part;
                            } else {
                                val[j] = sum;
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) xq4d::mbar_arrive(&red_free[buf]);
                }
                if (!alive) break;
#pragma unroll
                for (int j = 0; j < 4; j++) {  // uniform trip count: SwiGLU pairs lanes
                    const int base = 32 * j;
                    if (base >= op.m * 16) break;
                    const int oo = base + lane;
                    const int tok = oo >> 4, r = oo & 15;
                    const int row = rb * XQ4G_ROWS + r;
                    const bool valid = oo < op.m * 16 && row < op.n;
                    float sum = val[j];
                    if (valid && op.xh) {  // undo 2^-24 and the token's power of two (exact)
                        float f1, f2;
                        pow2_split(24 - tok_exponent(op.xh_max[tok]), f1, f2);
                        sum = sum * f1 * f2;
                    }
                    if (op.swiglu) {
                        // rows 2i (gate) and 2i+1 (up) sit in neighbouring
                        // lanes; the reference's swiglu_bf16 (main.rs:
                        // 4732-4745) on the op's bf16 outputs
                        const float hb = __bfloat162float(__float2bfloat16_rn(sum));
                        const float u = __shfl_xor_sync(0xffffffffu, hb, 1);
                        if (valid && !(r & 1)) {
                            const float gs = __fmul_rn(hb, __fdiv_rn(1.f, __fadd_rn(1.f, expf(-hb))));
                            const __nv_bfloat16 h = __float2bfloat16_rn(__fmul_rn(gs, u));
                            const size_t idx = (size_t)tok * ystride + yoff + (row >> 1);
                            reinterpret_cast<__nv_bfloat16 *>(op.y)[idx] = h;
                            if (op.shard && xchg) {  // one word per peer (value bits + epoch)
                                const unsigned long long word =
                                    ((unsigned long long)e << 32) | (uint32_t)__bfloat16_as_ushort(h);
                                for (int q = 0; q < p2p.nranks; q++)
                                    if (q != p2p.rank) xq4d::st_sys_u64(p2p.inbox[q] + half + op.inbox_off + idx, word);
                            }
                        }
                        continue;
                    }
                    if (!valid) continue;
                    if (op.residual) {  // add_bf16 (main.rs:4726-4730) of the op's bf16 output
                        const size_t ri = (size_t)tok * op.n + row;
                        const float hb = __bfloat162float(__float2bfloat16_rn(sum));
                        const float res = op.res_ext ? resv[j]
                                                     : __uint_as_float((uint32_t)xq4d::ldcg_u16(op.residual + ri) << 16);
                        reinterpret_cast<__nv_bfloat16 *>(op.y)[ri] = __float2bfloat16_rn(__fadd_rn(hb, res));
                        continue;
                    }
                    {
                        const size_t idx = (size_t)tok * ystride + yoff + row;
                        uint32_t bits;
                        if (op.out_f32) {
                            reinterpret_cast<float *>(op.y)[idx] = sum;
                            bits = __float_as_uint(sum);
                        } else {
                            const __nv_bfloat16 h = __float2bfloat16_rn(sum);
                            reinterpret_cast<__nv_bfloat16 *>(op.y)[idx] = h;
                            bits = __bfloat16_as_ushort(h);
                        }
                        if (op.shard && xchg) {  // one word per peer (value bits + epoch)
                            const unsigned long long word = ((unsigned long long)e << 32) | bits;
                            for (int q = 0; q < p2p.nranks; q++)
                                if (q != p2p.rank) xq4d::st_sys_u64(p2p.inbox[q] + half + op.inbox_off + idx, word);
                        }
                    }
                }
            }
            if (!(vi.w & kVisitLast)) continue;
            // The CTA's last visit in its segment: before a later segment may
            // read them, the peers' rows of its ranges of the segment's
            // sharded ops go from the inbox into y (the last segment's
            // rows are copied by the consumer warps, after their last stage).
            if (xchg && alive && seg + 1 < plan.n_seg)
                chain_gather(ops, plan, p2p, pend, v, e, half, lane, 32);
            pend = v + 1;
            // this CTA's rows of the segment are written (the warp barrier
            // orders every lane's stores before lane 0's release); no
            // segment waits for the last one
            __syncwarp();
            if (lane == 0 && seg + 1 < plan.n_seg) xq4d::red_release_gpu_add(&done[seg], 1u);
        }
        // the last CTA out leaves the counters zeroed for the next launch and
        // advances the inbox epoch (every CTA read it before counting here)
        if (lane == 0 && atomicAdd(&done[plan.n_seg], 1u) == (unsigned)G - 1) {
            for (int q = 0; q <= plan.n_seg; q++) done[q] = 0u;
            if (p2p.nranks > 1) *reinterpret_cast<volatile unsigned *>(p2p.epoch) = e;
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    xq4d::grid_dep_wait();
    // this launch's inbox epoch, read before this CTA's reducer can count
    // out (after which the last CTA out advances it)
    const unsigned ep = p2p.nranks > 1 ? *reinterpret_cast<volatile const unsigned *>(p2p.epoch) + 1u : 0u;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t ring_s = xq4d::smem_u32(ring);
    const uint32_t xs[1] = {0u};
    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    int slot = 0, rbl = 0;
    uint32_t phase = 0, waits = 0;
    for (int v = v0; v < v1; v++) {
        const int4 vi = __ldg(plan.visits + v);
        const xq4_chain_op_dev op = ops[vi.x];
        const int seg = vi.w >> 2;
        if ((vi.w & kVisitFirst) && seg > 0) {
            // The CTA's first visit in a segment after the first: every CTA
            // that visits the previous segment is done with it (and, through
            // the waits those CTAs passed, with every earlier segment).  Warp
            // 0 sees the count (acquire), then the consumer warps meet on an
            // mbarrier (release / acquire within the CTA): a bounded wait, so
            // a warp that gave up earlier cannot hold the others forever.
            if (warp == 0 && lane == 0) {
                const uint64_t t0 = xq4d::global_ns();
                const unsigned want = __ldg(plan.seg_cnt + seg - 1);
                while (xq4d::ld_acquire_gpu_u32(&done[seg - 1]) < want) {
                    if (xq4d::global_ns() - t0 > 2000000000ull) {
                        atomicOr(&g_xq4_fault, XQ4_FAULT_CHAIN_WAIT);
                        break;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(op_bar);
            if (!xq4d::mbar_wait(op_bar, waits & 1u)) atomicOr(&g_xq4_fault, XQ4_FAULT_CHAIN_WAIT);
            waits++;
        }
        const int tok = g < op.m ? g : 0;
        const uint16_t *const xr[1] = {op.xh ? op.xh_img + (size_t)tok * op.kc * XQ4G_KCHUNK
                                             : reinterpret_cast<const uint16_t *>(op.x) + (size_t)tok * op.k};
        const uint8_t *const qrow = (W8 && op.w4a8) ? op.qx_img + (size_t)tok * op.kc * XQ4G_KCHUNK : nullptr;
        const int rb0 = vi.y, rb1 = vi.z;
        const bool k_whole = (op.k % XQ4G_KCHUNK) == 0;
        const float hs = op.xh ? 0.0625f : 1.f;  // fp16 path: rows g+8 summed 16 * c
        // the warp's partials to buffer rbl % kRedBufs: per row block, or per
        // stage (one 2048-K chunk partial) for a W4A8 op
        const auto handoff = [&]() -> bool {
            const int buf = rbl % kRedBufs;
            const uint32_t use = (uint32_t)(rbl / kRedBufs);
            if (use > 0 && !xq4d::mbar_wait(&red_free[buf], (use - 1) & 1)) return false;
            float *r = red + (size_t)buf * kConsumerWarps * 128 + (size_t)warp * 128;
            r[(2 * t) * 16 + g] = acc[0][0];
            r[(2 * t + 1) * 16 + g] = acc[0][1];
            r[(2 * t) * 16 + g + 8] = acc[0][2] * hs;
            r[(2 * t + 1) * 16 + g + 8] = acc[0][3] * hs;
            acc[0][0] = acc[0][1] = acc[0][2] = acc[0][3] = 0.f;
            __syncwarp();
            if (lane == 0) xq4d::mbar_arrive(&red_full[buf]);
            rbl++;
            return true;
        };
        for (int rb = rb0; rb < rb1; rb++) {
            for (int kc0 = 0; kc0 < op.kc; kc0 += kStageChunks) {
                const uint32_t stage = ring_s + (uint32_t)slot * kChainStageBytes;
                const bool whole = kc0 + kStageChunks <= op.kc;
                bool ok;
                if (W8 && op.w4a8)
                    ok = consume_stage_w4a8(stage, &full[slot], phase, kc0, op.kc, qrow, op.qx_tbl, warp, lane,
                                            acc[0]);
                else
#ifndef XQ4_CHAIN_NO_M1
                if (op.xh && op.m == 1 && whole)  // one token, fp16 path, whole stage: x and table in the stage
                    ok = consume_stage<1, false, true, false, true, true, true>(stage, &full[slot], phase, kc0, op.kc,
                                                                               op.k, xr, xs, 0u, warp, lane, acc);
                else
#endif
                if (op.xh)  // fp16 path: K padding is zero in the image
                    ok = whole ? consume_stage<1, false, true, false, true>(stage, &full[slot], phase, kc0, op.kc, op.k,
                                                                           xr, xs, 0u, warp, lane, acc, op.xh_tbl)
                               : consume_stage<1, true, true, false, true>(stage, &full[slot], phase, kc0, op.kc, op.k,
                                                                          xr, xs, 0u, warp, lane, acc, op.xh_tbl);
                else
                    ok = (k_whole && whole)
                             ? consume_stage<1, false, false, true>(stage, &full[slot], phase, kc0, op.kc, op.k, xr, xs,
                                                                    0u, warp, lane, acc)
                             : consume_stage<1, true, false, true>(stage, &full[slot], phase, kc0, op.kc, op.k, xr, xs,
                                                                   0u, warp, lane, acc);
                if (!ok) {
                    atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                    return;
                }
                __syncwarp();
                if (lane == 0) xq4d::mbar_arrive(&empty[slot]);
                if (++slot == kChainStages) {
                    slot = 0;
                    phase ^= 1;
                }
                if (W8 && op.w4a8 && !handoff()) {
                    atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                    return;
                }
            }
            if (!(W8 && op.w4a8) && !handoff()) {  // row block complete
                atomicOr(&g_xq4_fault, XQ4_FAULT_GEMV_FULL);
                return;
            }
        }
    }
    // the last segment's copy-in of the peers' rows, shared by the consumer
    // warps (one warp walking it alone cost tens of microseconds of the
    // launch's tail at 8 ranks)
    if (p2p.nranks > 1 && v1 > v0) {
        int vf = v1;
        while (vf > v0 && (__ldg(plan.visits + vf - 1).w >> 2) == plan.n_seg - 1) vf--;
        if (vf < v1 && p2p_usable(p2p.poison, p2p.rank, lane))
            chain_gather(ops, plan, p2p, vf, v1 - 1, ep, (size_t)(ep & 1u) * p2p.half_words,
                         warp * 32 + lane, kConsumerThreads);
    }
}

int sm_count_of_current_device()
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

// Kernels whose CTAs wait for one another (the fused gather's peer waits,
// the chain's op waits) need their whole grid resident at once; the bounded
// waits would otherwise run out and leave wrong outputs behind a fault bit.
// XQ4_RESIDENT_CTAS_PER_SM (environment, diagnostics) replaces the occupancy
// query's answer, to emulate SMs held by another context.
bool whole_grid_resident(const void *kernel, int threads, size_t smem, int grid)
{
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (const char *f = getenv("XQ4_RESIDENT_CTAS_PER_SM"))
        if (*f) per_sm = atoi(f);
    return (long long)per_sm * sm_count_of_current_device() >= grid;
}

template <int NT, bool XH, bool P2P>
cudaError_t launch_one(const uint8_t *pack, int n, int k, const uint16_t *x, int m, void *y, int out_f32,
                       cudaStream_t st, const xq4_p2p_out &p2p)
{
    static std::atomic<bool> attr_set[64];  // zero-initialised; atomics: first launches may race across threads
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_kernel<NT, XH, P2P>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const int nb = xq4g_nb(n), kc = xq4g_kc(k);
    const size_t smem = smem_bytes(NT, XH, m, kc);
    if (smem > (size_t)kMaxSmem) return cudaErrorInvalidValue;  // never for the paths chosen below
    const int sms = sm_count_of_current_device();
    const int grid = nb < sms * kCtasPerSm ? nb : sms * kCtasPerSm;
    if (P2P && p2p.nranks > 1 && !whole_grid_resident((const void *)gemv_kernel<NT, XH, P2P>, kThreads, smem, grid))
        return cudaErrorCooperativeLaunchTooLarge;
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
    return cudaLaunchKernelEx(&cfg, gemv_kernel<NT, XH, P2P>, pack, n, k, nb, kc, x, m, y, out_f32, p2p);
}

}  // namespace

// m in 1..16 per launch; larger m is split into 16-token slices.
cudaError_t xq4_launch_gemv(const uint8_t *pack, int n, int k, const void *x, int m, void *y, int out_f32,
                            cudaStream_t st, const xq4_p2p_out *p2p)
{
    const xq4_p2p_out none{};
    if (p2p && m > 16) return cudaErrorInvalidValue;  // one launch per sharded call
    static_assert(xh_offset(2) + 128 + (size_t)kStages * kStageBytes <= (size_t)kMaxSmem, "bf16 plan too large");
    static_assert(xh_offset(1) + 64 + (size_t)kXhMaxBytes + 128 + (size_t)kStages * kStageBytes <= (size_t)kMaxSmem / 2 - 1024,
                  "fp16 plan too large for two CTAs per SM");
    const size_t ysz = out_f32 ? 4 : 2;
    const int kp = xq4g_kc(k) * XQ4G_KCHUNK;
    const uint8_t *p = reinterpret_cast<const uint8_t *>(pack);
    for (int t0 = 0; t0 < m; t0 += 16) {
        const int mt = m - t0 < 16 ? m - t0 : 16;
        const uint16_t *xs = reinterpret_cast<const uint16_t *>(x) + (size_t)t0 * k;
        void *ys = reinterpret_cast<char *>(y) + (size_t)t0 * n * ysz;
        cudaError_t e;
        const bool xh = xh_fits(mt, kp) && (long long)xq4g_nb(n) * xq4g_kc(k) >= kXhMinChunks;
        if (p2p)
            e = xh ? launch_one<1, true, true>(p, n, k, xs, mt, ys, out_f32, st, *p2p)
                   : (mt <= 8 ? launch_one<1, false, true>(p, n, k, xs, mt, ys, out_f32, st, *p2p)
                              : launch_one<2, false, true>(p, n, k, xs, mt, ys, out_f32, st, *p2p));
        else
            e = xh ? launch_one<1, true, false>(p, n, k, xs, mt, ys, out_f32, st, none)
                   : (mt <= 8 ? launch_one<1, false, false>(p, n, k, xs, mt, ys, out_f32, st, none)
                              : launch_one<2, false, false>(p, n, k, xs, mt, ys, out_f32, st, none));
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

size_t xq4_gemv_chain_smem() { return kChainSmem; }

// Set the chain kernel's shared-memory attribute on the current device and
// check that its whole grid can be resident (its op waits need that).
// The chain kernels' shared-memory attribute, once per device.
static cudaError_t chain_attrs()
{
    static std::atomic<bool> attr_set[64];  // zero-initialised; atomics: first launches may race across threads
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_chain_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kChainSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemv_chain_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kChainSmem);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    return cudaSuccess;
}

cudaError_t xq4_gemv_chain_prepare()
{
    if (cudaError_t e = chain_attrs(); e != cudaSuccess) return e;
    const int grid = sm_count_of_current_device() * kCtasPerSm;
    if (!whole_grid_resident((const void *)gemv_chain_kernel<false>, kThreads, kChainSmem, grid) ||
        !whole_grid_resident((const void *)gemv_chain_kernel<true>, kThreads, kChainSmem, grid))
        return cudaErrorCooperativeLaunchTooLarge;
    return cudaSuccess;
}

int xq4_gemv_chain_grid() { return sm_count_of_current_device() * kCtasPerSm; }

cudaError_t xq4_launch_gemv_chain(const xq4_chain_op_dev *ops, const xq4_chain_plan &plan, int grid,
                                  const xq4_chain_prep_dev *preps, int n_preps, const xq4_chain_p2p &p2p,
                                  bool has_w4a8, cudaStream_t st)
{
    if (n_preps > 0) {  // the fp16 images first; the chain's producers start meanwhile (PDL)
        cudaLaunchConfig_t pc = {};
        pc.gridDim = dim3(n_preps);
        pc.blockDim = dim3(kPrepThreads);
        pc.stream = st;
        cudaLaunchAttribute pa[1];
        pa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        pa[0].val.programmaticStreamSerializationAllowed = 1;
        pc.attrs = pa;
        pc.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&pc, chain_prep_kernel, preps);
        if (e != cudaSuccess) return e;
    }
    if (cudaError_t e = chain_attrs(); e != cudaSuccess) return e;  // residency was checked at chain create
    cudaLaunchConfig_t cfg = {};
    // every CTA resident (the op waits need it; checked at chain create); the
    // grid the range table was built for
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kChainSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return has_w4a8 ? cudaLaunchKernelEx(&cfg, gemv_chain_kernel<true>, ops, plan, p2p)
                    : cudaLaunchKernelEx(&cfg, gemv_chain_kernel<false>, ops, plan, p2p);
}

// Read and clear this unit's fault word on the current device.
unsigned int xq4_take_fault_gemv()
{
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_xq4_fault, sizeof v) != cudaSuccess) return ~0u;
    cudaMemcpyToSymbol(g_xq4_fault, &zero, sizeof zero);
    return v;
}
