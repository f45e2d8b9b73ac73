// xq4_internal.h -- private declarations shared by the libxq4 translation units.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "../../include/xq4.h"

// Record a failure message for xq4_last_error_string() and return `code`.
int xq4_fail(int code, const char *fmt, ...)
#if defined(__GNUC__)
    __attribute__((format(printf, 2, 3)))
#endif
    ;
void xq4_clear_error(void);

// repack.cpp
int xq4_check_desc(const xq4_layout_desc *desc, size_t src_len, int *r0, int *r1);
int xq4_repack_rows(const void *src, size_t src_len, const xq4_layout_desc *desc, int r0, int r1,
                    uint8_t *dst);

#ifdef __CUDACC__
#include <cuda_runtime.h>


// Column-sharded GEMV with the gather inside the kernel.  Every output value
// travels to each peer as one 64-bit word in the peer's inbox: the value's
// bits in the low half, the call's epoch in the high half.  A single aligned
// 64-bit store is seen whole or not at all, so a word whose epoch matches is
// complete and no fence or completion flag is needed.  Inboxes have two
// halves used by epoch parity: no rank gets more than one call ahead of
// another (a call ends only after the peers' words of that call arrived), so a
// half is never rewritten while a rank still reads it.
//
// A peer wait that runs out leaves the ranks' epochs out of step for good (the
// rank that gave up has advanced its epoch, its peers have not), after which a
// later call could accept a word of another call whose tag happens to match.
// So the kernel that gives up poisons the communicator: it sets the poison
// word in its own inbox header and in every peer's, and the host-mapped flag
// the host checks before each call.  A kernel that starts on a poisoned
// communicator skips the exchange (it writes its own rows only), raises fault
// bit 0x8 and sets the host flag; the host refuses further calls.
#define XQ4_MAX_RANKS 8
struct xq4_p2p_poison {
    unsigned *word[XQ4_MAX_RANKS];  // rank q's poison word (peer-mapped; [rank] is local)
    unsigned *host;                 // device address of the host-mapped flag
};
struct xq4_p2p_out {
    int nranks, rank;
    int n_total;                                // rows of the full output (n x nranks)
    int row_off;                                // this rank's first row
    unsigned long long *inbox[XQ4_MAX_RANKS];   // rank q's inbox (peer-mapped; [rank] is local)
    size_t half_words;                          // words per parity half (>= m x n_total)
    unsigned *cnt;                              // local: CTAs of the current launch that are done
    unsigned *epoch;                            // local: fused calls this rank has completed
    xq4_p2p_poison poison;
};

// 64-K chunks per ring stage of the GEMV kernels (gemv.cu checks it).
#define XQ4_GEMV_STAGE_CHUNKS_ABI 32

// One op of a GEMV chain, as the chain kernel reads it (device memory).
struct xq4_chain_op_dev {
    const uint8_t *pack;  // XQ4G weights
    const void *x;        // bf16 [m][k]
    void *y;              // [m][n], bf16 or f32
    int n, k, nb, kc;     // rows, K, row blocks, 64-K chunks
    int m, out_f32;
    int wait_prev;        // read x only after every CTA has written the previous op's y
    int xh;               // x comes from a prepared fp16 image (below) instead of x
    const uint16_t *xh_img;    // [m][kc*64] fp16, x scaled by a per-token power of two
    const float4 *xh_tbl;      // [kc][4][2]: the zero-point MMA accumulator inputs per group
    const float4 *xh_tbl1;     // m == 1: [kc][2] the same inputs of token 0, {z, z, 16 z, 16 z} per group
    const unsigned *xh_max;    // [8] per-token max |x| (bf16 magnitude bits)
    // Work split: a segment is a run of ops of which only the first waits
    // for its predecessor; its row blocks, weighted by ring stages, are cut
    // into one contiguous share per CTA.
    long long seg_start;  // stages of the segment before this op
    long long seg_units;  // stages of the whole segment
    int spr;              // stages per row block
    // Column-sharded op (the weight is this rank's row shard, y the full
    // m x n_total output): rows go to the peers as inbox words.
    int shard;
    int n_total, row_off;
    long long inbox_off;  // the op's first word in an inbox half
    // Epilogues: y = RNE(RNE(Wx) + residual) (not with shard), or SwiGLU of
    // the row pairs (2i, 2i+1) into y[tok][n/2] (sharded: y[tok][n_total/2],
    // this rank's pairs from row_off/2).
    const uint16_t *residual;
    int res_ext;          // no op of the chain writes the residual: the reducer may read it early
    int swiglu;
    // W4A8 (the reference's NPU numerics): x quantized by the prep to int8
    // per 32-K group; per group one integer MMA, times s_w * d_x; each stage
    // (2048 K) is one chunk partial, rounded to bf16 and summed in f32.
    int w4a8;
    const uint8_t *qx_img;     // [m][kc*64] int8, bytes 0,2,1,3 within each 4 (the MMA's slot order)
    const int2 *qx_tbl;        // [groups][8 tokens]: {-8 * sum(q_x), bits of f32(d_x)}
};

// The chain's work plan, built at chain create.  A segment is a run of ops
// of which only the first waits for its predecessor.  Each CTA has a list of
// visits, one per op in which it owns row blocks: {op, rb0, rb1, seg << 2 |
// last << 1 | first}, first / last marking its first / last visit in the
// segment.
struct xq4_chain_plan {
    const int4 *visits;
    const int *vstart;        // [grid + 1]: CTA c's visits are [vstart[c], vstart[c + 1])
    const unsigned *seg_cnt;  // [n_seg]: CTAs with a visit in the segment
    unsigned *done;           // [n_seg + 1]: CTAs done with the segment; [n_seg]: CTAs out
    int n_seg;
};

// The chain's communicator side (nranks == 1: no sharded op).
struct xq4_chain_p2p {
    int nranks, rank;
    unsigned long long *inbox[XQ4_MAX_RANKS];  // rank q's inbox (peer-mapped; [rank] is local)
    size_t half_words;
    unsigned *epoch;               // the communicator's inbox epoch (shared with the fused GEMV)
    xq4_p2p_poison poison;
};
struct xq4_comm;
// Map the communicator's inboxes if not done yet (collective) and describe
// them for a chain on `dev`.
int xq4_comm_chain_p2p(struct xq4_comm *comm, const struct xq4_device *dev, struct xq4_chain_p2p *out);
int xq4_comm_nranks(const struct xq4_comm *comm);
int xq4_comm_rank(const struct xq4_comm *comm);
// XQ4_OK, or the status to return when an earlier call on the communicator
// gave up waiting for a peer (the communicator is unusable from then on).
int xq4_comm_check_usable(const struct xq4_comm *comm);


// One activation the chain reads through the fp16 path, converted once per
// run (before the chain's consumers start) by the prep kernel.
struct xq4_chain_prep_dev {
    const void *x;        // bf16 [m][k]
    uint16_t *img;
    float *tbl;
    float4 *tbl1;         // m == 1: the one-token table (xq4_chain_op_dev::xh_tbl1)
    unsigned *max;
    int m, k, kc, norm;   // norm: RMS-normalise x with norm_w first
    const uint16_t *norm_w;
    float eps;
    int w4a8;             // quantize to int8 (qx, qtbl) instead of the fp16 image
    uint8_t *qx;          // [m][kc*64] (xq4_chain_op_dev::qx_img)
    int2 *qtbl;           // [kc*2][8] (xq4_chain_op_dev::qx_tbl)
};

// A weight resident in HBM, in XQ4G layout.
struct xq4_weight {
    struct xq4_device *dev;
    int ordinal;       // device ordinal (destroy does not touch `dev`)
    int n, k;          // logical rows / reduction length
    int nb, kc;        // row blocks, 64-K chunks
    uint8_t *d_pack;   // xq4g_bytes(n, k) bytes
    size_t bytes;
};

// Smallest m that runs the tensor-core GEMM; below it the decode GEMV (in
// 16-token launches) streams the weights.  Measured on B200 (gate
// 14336x4096): GEMV 19 us at m = 16 and 29 us at m = 24 against the GEMM's
// 33 and 35 us; equal near m = 28; the GEMM is ahead from m = 32.
// Chunks (16 rows x 64 K) from which the fp16 activation path pays for its
// prologue (the single-op GEMV's staging, the chain's prep launch); below it
// both run the bf16 path.
#define XQ4_XH_MIN_CHUNKS 98304LL
#ifndef XQ4_GEMM_MIN_M
#define XQ4_GEMM_MIN_M 25
#endif
static inline bool xq4_use_gemv(int m) { return m < XQ4_GEMM_MIN_M; }

// Kernel launchers (gemv.cu, gemm_tc.cu, dequant.cu).  All return cudaError_t
// of the launch; arguments are validated by the callers in api.cu.
cudaError_t xq4_launch_gemv(const uint8_t *pack, int n, int k, const void *x, int m, void *y,
                            int out_f32, cudaStream_t st,
                            const struct xq4_p2p_out *p2p = nullptr);
// One persistent launch over a chain of GEMVs (m <= 8 each) by the plan
// (per-CTA visit lists and segment counters, the counters left zeroed at the
// end of the launch), built for `grid` = xq4_gemv_chain_grid() at create.
// has_w4a8: the chain holds W4A8 ops (the kernel instantiation with that path).
cudaError_t xq4_launch_gemv_chain(const struct xq4_chain_op_dev *ops, const struct xq4_chain_plan &plan, int grid,
                                  const struct xq4_chain_prep_dev *preps, int n_preps,
                                  const struct xq4_chain_p2p &p2p, bool has_w4a8, cudaStream_t st);
// CTAs of a chain launch on the current device.
int xq4_gemv_chain_grid();
size_t xq4_gemv_chain_smem();
// Set up the chain kernel on the current device; cudaErrorCooperativeLaunchTooLarge
// when its grid (2 CTAs per SM) cannot all be resident at once.
cudaError_t xq4_gemv_chain_prepare();
cudaError_t xq4_launch_gemm(const uint8_t *pack, int n, int k, const void *x, int m, void *y,
                            int out_f32, cudaStream_t st);
cudaError_t xq4_launch_dequant(const uint8_t *pack, int n, int k, void *out, cudaStream_t st);
cudaError_t xq4_launch_quantize_x(const void *x, int m, int k, void *q, void *d, cudaStream_t st);
cudaError_t xq4_launch_w4a8(const uint8_t *pack, int n, int k, const void *qx, const void *dx, int m, void *y,
                            int out_f32, cudaStream_t st);
unsigned int xq4_take_fault_gemv();
unsigned int xq4_take_fault_gemm();
unsigned int xq4_take_fault_w4a8();
unsigned int xq4_take_fault_attn();
cudaStream_t xq4_device_cuda_stream(struct xq4_device *dev);
int xq4_device_ordinal(const struct xq4_device *dev);
#endif
