// attn.cu -- decode attention of one token: the attention side of the
// reference's decode step (crates/xnpu-cli/src/main.rs:4817-4857 and
// :4967-5033), one kernel launch per layer.
//
// Input is the token's qkv projection output, bf16 [heads*128 | nkv*128 (k) |
// nkv*128 (v)].  The kernel
//   * rotates q and k by the rotate-half RoPE of position pos (rope_apply,
//     main.rs:4829-4839), one bf16 rounding;
//   * applies the per-head RMSNorm over 128 with weights shared by the heads
//     (qk_rms_bf16, main.rs:4844-4857), when its weights are given;
//   * appends k and v to the layer's KV cache at pos ([nkv][cache_seq][128]
//     bf16, the reference's layout);
//   * runs GQA attention of every q head over positions 0..pos: scores
//     (K q)/sqrt(128), softmax with the max subtracted, sum of w_t v_t, one
//     bf16 rounding (attention_bf16, main.rs:4967-5033).
//
// Work split (HBM-bound on the cache: 512 B per position per kv head): CTA
// (split, kv) takes positions [split*span, (split+1)*span) of kv head kv for
// the q heads of its group; each of its 4 warps owns q heads, each lane a
// position in the scores pass and 4 of the 128 dims in the P.V pass.  A CTA
// leaves (max, sum, acc[128]) per head; the last CTA of a kv head to finish
// (counter) merges the splits.  With one split the result is the reference's
// formula as written: max over all positions, w_t = exp(s_t - max), the sum
// and the P.V in ascending t.
//
// Exactness: RoPE, the q/k norm and every score use the reference's operation
// order with single roundings (no contraction), and the RoPE table is
// computed on the host with the same f32 formula as the reference's
// rope_table (main.rs:4817-4827), so q, k and the scores are bit-identical to
// it.  The softmax uses CUDA's expf, the split merge and the lane-parallel sum
// of the weights reorder f32 additions: outputs agree to about one bf16 ulp.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <algorithm>
#include <mutex>
#include <new>
#include <vector>

#include "xq4_internal.h"
#include "xq4_device.cuh"

namespace {

constexpr int kHd = 128;          // head dim (fixed by the reference's model family)
constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kKStride = kHd + 2; // K row stride in shared memory (bf16): rows on distinct banks
constexpr int kMaxGroup = 8;      // q heads per kv head
constexpr int kMaxSpan = 384;     // positions per CTA (its K and V rows and scores in shared memory)
constexpr int kMaxSplits = 64;    // splits per kv head (the merge covers them in two lane rounds)
#ifndef XQ4_ATTN_MIN_SPAN
#define XQ4_ATTN_MIN_SPAN 32
#endif
constexpr int kMinSpan = XQ4_ATTN_MIN_SPAN;  // positions a split takes before the token uses another split (measured)
// One split's partial of one head in the workspace: max, sum, two pad words
// (so that acc starts 16 bytes in), acc[128]; 528 bytes, a multiple of 16.
constexpr int kRec = 4 + kHd;
constexpr int kRecAcc = 4;

struct attn_params {
    const uint16_t *qkv;
    const uint16_t *q_norm, *k_norm;  // [128] bf16, or NULL
    const float *rope;                // [cache_seq][128]: cos[64] then sin[64]; NULL = no RoPE
    uint16_t *kc, *vc;                // [nkv][cache_seq][128]
    const int *pos;                   // the token's position (device)
    uint16_t *out;                    // [heads][128]
    float *ws;                        // [heads][splits][kRec]: max, sum, pad, acc
    unsigned *cnt;                    // [nkv] CTAs done (left zeroed)
    int heads, nkv, cache_seq, splits;
    int span;                         // positions the score area holds per head (a split's most)
};

// Floats of the score area, rounded up so that the tiles after it stay
// 16-byte aligned.
__host__ __device__ inline size_t sc_floats(int G, int span) { return ((size_t)G * span + 3) & ~(size_t)3; }

__device__ __forceinline__ float bf(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t to_bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

// RoPE (and the per-head norm) of one head of 128 by one warp: src -> dst
// (bf16 bits, shared memory), f32 copy in dstf when given.  Lane l owns the
// rotation pairs (l, l+64) and (l+32, l+96).
__device__ void rope_norm_head(const uint16_t *src, const float *cs, const uint16_t *nw, uint16_t *dst, float *dstf,
                               int lane)
{
    for (int jj = 0; jj < 2; jj++) {
        const int j = lane + 32 * jj;
        const float x1 = bf(src[j]), x2 = bf(src[j + 64]);
        if (cs) {  // out[j] = x1 c - x2 s, out[j+64] = x2 c + x1 s (main.rs:4829-4839)
            const float c = cs[j], s = cs[64 + j];
            dst[j] = to_bf(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
            dst[j + 64] = to_bf(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
        } else {
            dst[j] = src[j];
            dst[j + 64] = src[j + 64];
        }
    }
    __syncwarp();
    if (nw) {
        // qk_rms_bf16 (main.rs:4844-4857): sequential f32 sum of squares by
        // one lane, inv = 1 / sqrt(mean + 1e-5), out = RNE(x * inv * w)
        float inv = 0.f;
        if (lane == 0) {
            float sum = 0.f;
            for (int j = 0; j < kHd; j++) {
                const float v = bf(dst[j]);
                sum = __fadd_rn(sum, __fmul_rn(v, v));
            }
            inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, 128.f), 1e-5f)));
        }
        inv = __shfl_sync(0xffffffffu, inv, 0);
        for (int j = lane; j < kHd; j += 32) dst[j] = to_bf(__fmul_rn(__fmul_rn(bf(dst[j]), inv), bf(nw[j])));
        __syncwarp();
    }
    if (dstf)
        for (int j = lane; j < kHd; j += 32) dstf[j] = bf(dst[j]);
    __syncwarp();
}

// Asynchronous global -> shared copies (nothing held in registers while in
// flight); completion by cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(xq4d::smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Scores of rows tb + lane + 32 u (u < U) of the span against q: each over j
// ascending (d = sum_j k[t][j] * q[j], main.rs:5006-5011), U independent
// sums per lane; rows past the span read the last row and are dropped.
template <int U>
__device__ __forceinline__ void score_rows(const float *q, const uint16_t *kt, int tb, int nt, int lane, float rs,
                                           float *scrow, float &m)
{
    float d[U];
    const uint32_t *kr[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
        d[u] = 0.f;
        kr[u] = reinterpret_cast<const uint32_t *>(kt + min(tb + lane + 32 * u, nt - 1) * kKStride);
    }
    for (int j2 = 0; j2 < kHd / 2; j2++) {
        const float q0 = q[2 * j2], q1 = q[2 * j2 + 1];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const uint32_t w = kr[u][j2];
            d[u] = __fadd_rn(d[u], __fmul_rn(__uint_as_float(w << 16), q0));
            d[u] = __fadd_rn(d[u], __fmul_rn(__uint_as_float(w & 0xFFFF0000u), q1));
        }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
        const int t = tb + lane + 32 * u;
        if (t < nt) {
            const float dv = __fdiv_rn(d[u], rs);
            scrow[t] = dv;
            m = fmaxf(m, dv);
        }
    }
}

__global__ void __launch_bounds__(kThreads)
attn_decode_kernel(const attn_params p)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int G = p.heads / p.nkv;
    float *qf = reinterpret_cast<float *>(smem);                                     // [G][128]
    float *sc = qf + kMaxGroup * kHd;                                                // [G][span]
    uint16_t *vt = reinterpret_cast<uint16_t *>(sc + sc_floats(G, p.span));         // [span][128]
    uint16_t *kt = vt + (size_t)p.span * kHd;                                        // [span][kKStride]
    uint16_t *tmp = kt + (size_t)p.span * kKStride;                                  // [kWarps][128] bf16 scratch
    __shared__ bool last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, kv = blockIdx.y;
    // the next kernel (the o projection's chain) may launch now and stream
    // its weights while this one runs; it reads this kernel's output only
    // after its own griddepcontrol.wait
    xq4d::grid_dep_launch();
    xq4d::grid_dep_wait();  // qkv and the cache come from the preceding kernels
    const int pos = *p.pos;
    if (pos < 0 || pos >= p.cache_seq) {  // the host cannot check a device-resident position
        if (threadIdx.x == 0) atomicOr(&g_xq4_fault, XQ4_FAULT_ATTN_POS);
        return;
    }
    const int s = pos + 1;
    // splits for this token: at least kMinSpan positions each (a split is
    // latency-bound, and the merge reads every split), at most p.splits;
    // never more positions than the span the shared memory was sized for
    const int nsp = min(p.splits, max(1, (s + kMinSpan - 1) / kMinSpan));
    const int span = (s + nsp - 1) / nsp;
    const int t0 = split * span, t1 = min(s, t0 + span);
    const int nt = max(0, t1 - t0);
    const float *cs = p.rope ? p.rope + (size_t)pos * kHd : nullptr;

    // every K and V row of the span in flight at once (the token's own row,
    // position pos, comes from this kernel instead): V by 16-byte
    // asynchronous copies, K by 16-byte loads into registers (its rows land
    // at a padded stride, 4-byte aligned; 4-byte asynchronous copies ran at a
    // few GB/s per CTA), stored once the q heads are rotated
    const size_t base = ((size_t)kv * p.cache_seq + t0) * kHd;
    for (int i = threadIdx.x; i < nt * (kHd / 8); i += kThreads) {
        const int r = i / (kHd / 8), c = i % (kHd / 8);
        if (t0 + r != pos) cp_async16(vt + r * kHd + 8 * c, p.vc + base + (size_t)r * kHd + 8 * c);
    }
    // K in batches of 64 rows (8 pieces per thread); the first batch's loads
    // are in flight while the q heads are rotated
    constexpr int kKBatch = 8;
    const int kpieces = nt * (kHd / 8);
    uint4 kreg[kKBatch];
    const auto k_load = [&](int b0) {
#pragma unroll
        for (int u = 0; u < kKBatch; u++) {
            const int i = b0 + threadIdx.x + u * kThreads, r = i / (kHd / 8), c = i % (kHd / 8);
            if (i < kpieces && t0 + r != pos)
                kreg[u] = __ldcs(reinterpret_cast<const uint4 *>(p.kc + base + (size_t)r * kHd + 8 * c));
        }
    };
    const auto k_store = [&](int b0) {
#pragma unroll
        for (int u = 0; u < kKBatch; u++) {
            const int i = b0 + threadIdx.x + u * kThreads, r = i / (kHd / 8), c = i % (kHd / 8);
            if (i < kpieces && t0 + r != pos) {
                uint32_t *d = reinterpret_cast<uint32_t *>(kt + r * kKStride + 8 * c);
                d[0] = kreg[u].x;
                d[1] = kreg[u].y;
                d[2] = kreg[u].z;
                d[3] = kreg[u].w;
            }
        }
    };
    k_load(0);
    // q heads of this group: RoPE + norm, kept in f32 (while the rows land)
    for (int hg = warp; hg < G; hg += kWarps)
        rope_norm_head(p.qkv + (size_t)(kv * G + hg) * kHd, cs, p.q_norm, tmp + warp * kHd, qf + hg * kHd, lane);
    // the CTA holding position pos appends the token's k (RoPE + norm) and v,
    // to the caches and straight into its rows of the span
    if (pos >= t0 && pos < t1 && warp == 0) {
        uint16_t *kr = kt + (pos - t0) * kKStride, *vr = vt + (pos - t0) * kHd;
        rope_norm_head(p.qkv + (size_t)(p.heads + kv) * kHd, cs, p.k_norm, kr, nullptr, lane);
        const uint16_t *v = p.qkv + (size_t)(p.heads + p.nkv + kv) * kHd;
        for (int j = lane; j < kHd; j += 32) vr[j] = v[j];
        __syncwarp();
        const size_t row = ((size_t)kv * p.cache_seq + pos) * kHd;
        for (int j = lane; j < kHd; j += 32) {
            p.kc[row + j] = kr[j];
            p.vc[row + j] = vr[j];
        }
    }
    k_store(0);
    for (int b0 = kKBatch * kThreads; b0 < kpieces; b0 += kKBatch * kThreads) {
        k_load(b0);
        k_store(b0);
    }
    cp_async_wait_all();
    __syncthreads();

    const float rs = sqrtf(128.f);  // (128f32).sqrt(): exact to f32 rounding
    float mx[kMaxGroup / kWarps];
    for (int i = 0; i < kMaxGroup / kWarps; i++) mx[i] = -INFINITY;
    // pass 1: the scores; lane l takes positions l, l+32, ... of the span
    for (int hg = warp, i = 0; hg < G; hg += kWarps, i++) {
        const float *q = qf + hg * kHd;
        float m = -INFINITY;
        int tb = 0;  // rows of 128, then of 64 and 32: no lane sums a row past the span twice over
        for (; nt - tb > 64; tb += 128) score_rows<4>(q, kt, tb, nt, lane, rs, sc + hg * span, m);
        if (nt - tb > 32) {
            score_rows<2>(q, kt, tb, nt, lane, rs, sc + hg * span, m);
            tb += 64;
        }
        if (nt - tb > 0) score_rows<1>(q, kt, tb, nt, lane, rs, sc + hg * span, m);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        mx[i] = m;
    }
    // pass 2: weights w_t = exp(s_t - max), their sum, and sum_t w_t v_t
    // (each lane owns dims 4*lane..4*lane+3, t ascending)
    float acc[kMaxGroup / kWarps][4] = {};
    float sum[kMaxGroup / kWarps] = {};
    for (int hg = warp, i = 0; hg < G; hg += kWarps, i++)
        for (int t = lane; t < nt; t += 32) {
            float *e = sc + hg * span + t;
            *e = expf(__fsub_rn(*e, mx[i]));
            sum[i] = __fadd_rn(sum[i], *e);
        }
    __syncwarp();
    for (int hg = warp, i = 0; hg < G; hg += kWarps, i++)
        for (int r = 0; r < nt; r++) {
            const float w = sc[hg * span + r];
            const uint2 v = *reinterpret_cast<const uint2 *>(vt + r * kHd + 4 * lane);
            acc[i][0] = __fadd_rn(acc[i][0], __fmul_rn(w, __uint_as_float(v.x << 16)));
            acc[i][1] = __fadd_rn(acc[i][1], __fmul_rn(w, __uint_as_float(v.x & 0xFFFF0000u)));
            acc[i][2] = __fadd_rn(acc[i][2], __fmul_rn(w, __uint_as_float(v.y << 16)));
            acc[i][3] = __fadd_rn(acc[i][3], __fmul_rn(w, __uint_as_float(v.y & 0xFFFF0000u)));
        }
    // this split's (max, sum, acc) per head
    for (int hg = warp, i = 0; hg < G; hg += kWarps, i++) {
        float sm = sum[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
        float *w = p.ws + ((size_t)(kv * G + hg) * p.splits + split) * kRec;
        if (lane == 0) {
            w[0] = mx[i];
            w[1] = t1 > t0 ? sm : 0.f;
        }
        *reinterpret_cast<float4 *>(w + kRecAcc + 4 * lane) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
    // the last CTA of this kv head merges the splits: the barrier orders the
    // CTA's record writes before thread 0's count, whose release (gpu scope,
    // cumulative) publishes them; its acquire, and the barrier after it,
    // order every other CTA's records before the merge's reads
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.cnt + kv) : "memory");
        last = prev == (unsigned)p.splits - 1;
    }
    __syncthreads();
    if (!last) return;
    // splits that hold positions (the rest are empty for this token)
    const int used = (s + span - 1) / span;
    for (int hg = warp; hg < G; hg += kWarps) {
        const float *w = p.ws + (size_t)(kv * G + hg) * p.splits * kRec;
        // lane-parallel over the splits: the maximum, each split's factor
        // exp(m_s - M), and the weighted sum of the split sums
        float ms[2], ls[2], M = -INFINITY;
        for (int r = 0; r < 2; r++) {
            const int sp = lane + 32 * r;
            ms[r] = sp < used ? __ldcg(w + (size_t)sp * kRec) : -INFINITY;
            ls[r] = sp < used ? __ldcg(w + (size_t)sp * kRec + 1) : 0.f;
            M = fmaxf(M, ms[r]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float f[2], L = 0.f;
        for (int r = 0; r < 2; r++) {
            f[r] = ls[r] == 0.f ? 0.f : (used == 1 ? 1.f : expf(__fsub_rn(ms[r], M)));
            L = __fadd_rn(L, __fmul_rn(ls[r], f[r]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) L = __fadd_rn(L, __shfl_xor_sync(0xffffffffu, L, o));
        // sum_s f_s acc_s, s ascending: every lane's 4 dims, sixteen splits'
        // loads in flight together (a few at a time cost a round trip each)
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        for (int sp0 = 0; sp0 < used; sp0 += 16) {
            float4 a[16];
#pragma unroll
            for (int j = 0; j < 16; j++)
                a[j] = sp0 + j < used
                           ? __ldcg(reinterpret_cast<const float4 *>(w + (size_t)(sp0 + j) * kRec + kRecAcc + 4 * lane))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int sp = sp0 + j;
                if (sp >= used) break;
                const float fs = __shfl_sync(0xffffffffu, f[sp >> 5], sp & 31);
                o[0] = __fadd_rn(o[0], __fmul_rn(a[j].x, fs));
                o[1] = __fadd_rn(o[1], __fmul_rn(a[j].y, fs));
                o[2] = __fadd_rn(o[2], __fmul_rn(a[j].z, fs));
                o[3] = __fadd_rn(o[3], __fmul_rn(a[j].w, fs));
            }
        }
        uint16_t *out = p.out + (size_t)(kv * G + hg) * kHd + 4 * lane;
        for (int c = 0; c < 4; c++) out[c] = to_bf(__fdiv_rn(o[c], L));
    }
    if (threadIdx.x == 0) p.cnt[kv] = 0u;  // ready for the next launch
}

}  // namespace

// Read and clear this unit's fault word on the current device.
unsigned int xq4_take_fault_attn()
{
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_xq4_fault, sizeof v) != cudaSuccess) return ~0u;
    cudaMemcpyToSymbol(g_xq4_fault, &zero, sizeof zero);
    return v;
}

struct xq4_attn {
    xq4_device *dev;
    int ordinal;
    int heads, nkv, cache_seq, splits, span;
    float *rope;      // device [cache_seq][128], or NULL
    float *ws;        // device partials
    unsigned *cnt;    // device [nkv]
    size_t smem;
};

// The kernel's dynamic shared-memory limit is one attribute per device for
// every attention handle: it only ever grows, so that creating a handle with
// a smaller plan leaves the launches of an earlier, larger one valid.
static cudaError_t raise_smem_limit(int ordinal, size_t smem)
{
    static std::mutex mu;
    static size_t limit[64];
    std::lock_guard<std::mutex> lock(mu);
    if (ordinal >= 0 && ordinal < 64 && limit[ordinal] >= smem) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && ordinal >= 0 && ordinal < 64) limit[ordinal] = smem;
    return e;
}

extern "C" int xq4_attn_create(xq4_device *dev, int heads, int nkv, int cache_seq, float rope_base, xq4_attn **out)
{
    xq4_clear_error();
    if (!dev || !out) return xq4_fail(XQ4_EINVAL, "NULL argument");
    *out = nullptr;
    if (heads <= 0 || nkv <= 0 || heads % nkv || heads / nkv > kMaxGroup)
        return xq4_fail(XQ4_EINVAL, "heads %d / kv heads %d: need a multiple, at most %d q heads per kv head", heads,
                        nkv, kMaxGroup);
    if (cache_seq <= 0 || cache_seq > (1 << 20)) return xq4_fail(XQ4_EINVAL, "cache_seq %d out of range", cache_seq);
    if (!(rope_base >= 0.f)) return xq4_fail(XQ4_EINVAL, "rope_base must be >= 0 (0 = no RoPE)");
    const int ordinal = xq4_device_ordinal(dev);
    cudaError_t e = cudaSetDevice(ordinal);
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ordinal);
    // splits per kv head: about two CTAs per SM over all kv heads, each split
    // at most kMaxSpan positions and at least one tile
    int splits = (2 * sms + nkv - 1) / nkv;
    splits = std::max(splits, (cache_seq + kMaxSpan - 1) / kMaxSpan);
    splits = std::min(splits, (cache_seq + 31) / 32);
    splits = std::min(splits, kMaxSplits);
    const int span = (cache_seq + splits - 1) / splits;
    if (span > kMaxSpan)
        return xq4_fail(XQ4_EINVAL, "cache_seq %d needs more than %d splits of at most %d positions", cache_seq,
                        kMaxSplits, kMaxSpan);
    splits = (cache_seq + span - 1) / span;
    const int G = heads / nkv;
    // the score area holds a split's positions: at most `span` when every
    // split is in use, fewer than kMinSpan otherwise (see the kernel)
    const int span_max = std::max(span, kMinSpan);
    xq4_attn *a = new (std::nothrow) xq4_attn{dev, ordinal, heads, nkv, cache_seq, splits, span_max, nullptr,
                                              nullptr, nullptr, 0};
    if (!a) return xq4_fail(XQ4_ENOMEM, "host allocation");
    a->smem = sizeof(float) * ((size_t)kMaxGroup * kHd + sc_floats(G, span_max)) +
              sizeof(uint16_t) * ((size_t)span_max * kKStride + (size_t)span_max * kHd + (size_t)kWarps * kHd);
    const size_t ws_bytes = sizeof(float) * (size_t)heads * splits * kRec;
    if (rope_base > 0.f) {
        // the reference's rope_table (main.rs:4817-4827) at every position, in
        // f32 with the C library's powf/cosf/sinf as the reference calls them
        std::vector<float> t((size_t)cache_seq * kHd);
        for (int pos = 0; pos < cache_seq; pos++)
            for (int j = 0; j < 64; j++) {
                const float inv = powf(rope_base, -(float)j / 64.f);
                const float ang = (float)pos * inv;
                t[(size_t)pos * kHd + j] = cosf(ang);
                t[(size_t)pos * kHd + 64 + j] = sinf(ang);
            }
        e = cudaMalloc(&a->rope, t.size() * sizeof(float));
        if (e == cudaSuccess) e = cudaMemcpy(a->rope, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaMalloc(&a->ws, ws_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&a->cnt, sizeof(unsigned) * nkv);
    if (e == cudaSuccess) e = cudaMemset(a->cnt, 0, sizeof(unsigned) * nkv);
    if (e == cudaSuccess) e = raise_smem_limit(ordinal, a->smem);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(a->rope);
        cudaFree(a->ws);
        cudaFree(a->cnt);
        delete a;
        return xq4_fail(XQ4_ENOMEM, "attention set-up: %s", cudaGetErrorString(e));
    }
    *out = a;
    return XQ4_OK;
}

extern "C" int xq4_attn_destroy(xq4_attn *a)
{
    xq4_clear_error();
    if (!a) return XQ4_OK;
    cudaSetDevice(a->ordinal);
    cudaError_t e = cudaDeviceSynchronize();
    cudaFree(a->rope);
    cudaFree(a->ws);
    cudaFree(a->cnt);
    delete a;
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "attention destroy: %s", cudaGetErrorString(e));
    return XQ4_OK;
}

extern "C" int xq4_attn_decode(xq4_attn *a, const void *qkv_dev, const void *q_norm_w_dev, const void *k_norm_w_dev,
                               void *k_cache_dev, void *v_cache_dev, const int *pos_dev, void *out_dev, void *stream)
{
    xq4_clear_error();
    if (!a || !qkv_dev || !k_cache_dev || !v_cache_dev || !pos_dev || !out_dev)
        return xq4_fail(XQ4_EINVAL, "NULL argument");
    if (((uintptr_t)qkv_dev & 15) || ((uintptr_t)k_cache_dev & 15) || ((uintptr_t)v_cache_dev & 15) ||
        ((uintptr_t)out_dev & 7) || ((uintptr_t)q_norm_w_dev & 1) || ((uintptr_t)k_norm_w_dev & 1) ||
        ((uintptr_t)pos_dev & 3))
        return xq4_fail(XQ4_EINVAL, "qkv and the caches must be 16-byte aligned, out 8-byte aligned");
    cudaError_t e = cudaSetDevice(a->ordinal);
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    attn_params p{};
    p.qkv = (const uint16_t *)qkv_dev;
    p.q_norm = (const uint16_t *)q_norm_w_dev;
    p.k_norm = (const uint16_t *)k_norm_w_dev;
    p.rope = a->rope;
    p.kc = (uint16_t *)k_cache_dev;
    p.vc = (uint16_t *)v_cache_dev;
    p.pos = pos_dev;
    p.out = (uint16_t *)out_dev;
    p.ws = a->ws;
    p.cnt = a->cnt;
    p.heads = a->heads;
    p.nkv = a->nkv;
    p.cache_seq = a->cache_seq;
    p.splits = a->splits;
    p.span = a->span;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->splits, a->nkv);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = a->smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, attn_decode_kernel, p);
    if (e != cudaSuccess) return xq4_fail(XQ4_ECUDA, "attention launch: %s", cudaGetErrorString(e));
    return XQ4_OK;
}
