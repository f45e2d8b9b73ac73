/*
 * q4nx_oracle.c -- CPU restatement of xnpu's int4 ("w4" / Q4NX) weight path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline.  Nothing in the shipped library (xnpu_b200/, libxq4.so) links,
 * loads or calls it; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker.
 *
 * Every function restates one piece of the reference (nzinfo/xnpu, Rust) and
 * cites the file:line it follows.  The reference cannot be compiled in this
 * environment (no Rust toolchain), so this C restatement stands in for it.
 * Pinning: the bit-exact known-answer test (KAT) of crates/xnpu-cli/src/main.rs
 * :2164-2299 has an exactly-computable answer, and tests/golden/ holds vectors
 * produced by the reference's own importer functions (tools/w4_import.py
 * spot_rows / write_golden, executed from the reference source).  Real-weight
 * quantization (the external IRON quantize_and_pack) is NOT shipped with the
 * reference: that part is parity-unpinned.
 *
 * Build: g++/gcc with -O2 -ffp-contract=off (no FMA contraction: the Rust
 * reference computes `acc += w * x` as a separate multiply and add).
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>

#define Q4O_OK 0
#define Q4O_EINVAL -1

/* ------------------------------------------------------------------ bf16 */

/* f32 -> bf16 bits, round-to-nearest-even.  crates/xnpu-cli/src/main.rs:338-343 */
uint16_t q4o_f32_to_bf16(float x)
{
    uint32_t b;
    memcpy(&b, &x, 4);
    uint32_t bias = 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)((b + bias) >> 16); /* wrapping add, as in the reference */
}

/* bf16 bits -> f32 (exact widening).  crates/xnpu-cli/src/main.rs:663-665 */
float q4o_bf16_to_f32(uint16_t v)
{
    uint32_t b = (uint32_t)v << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* Sign-extend a 4-bit two's-complement nibble: `((nib as i8) << 4) >> 4`,
 * crates/xnpu-cli/src/main.rs:3120. */
static inline int sext4(unsigned nib)
{
    return (int)((int8_t)(uint8_t)(nib << 4) >> 4);
}

/* The reference's dequant rule: w = RNE_bf16(f32(q) * f32(scale_bf16)),
 * crates/xnpu-cli/src/main.rs:3121 (`f32_to_bf16(q as f32 * sf)`). */
uint16_t q4o_dequant_one(int q, uint16_t scale_bits)
{
    return q4o_f32_to_bf16((float)q * q4o_bf16_to_f32(scale_bits));
}

/* ------------------------------------------------------- layout L1 (w4gemv2)
 *
 * Rows are split over `cols` columns (rows_per_col = n/cols), each column holds
 * rows_per_col/tsi tiles of tsi rows; a tile is
 *   [tsi*K/2 nibble bytes | tsi*(K/group) bf16 scales]
 * nibble byte rr*(K/2)+p holds k=2p (low) and k=2p+1 (high), two's complement;
 * the scale for (rr, g) sits at nibble_bytes + (rr*K/group + g)*2.
 * crates/xnpu-cli/src/main.rs:2186-2191 (geometry), :2231-2252 (packer),
 * tools/w4_import.py:4-14 (ABI description), size formula main.rs:2597.
 */
static int l1_geom_ok(int n, int k, int group, int tsi, int cols)
{
    if (n <= 0 || k <= 0 || group <= 0 || tsi <= 0 || cols <= 0) return 0;
    if (k % 2 || k % group) return 0;
    if (n % cols) return 0;
    if ((n / cols) % tsi) return 0;
    return 1;
}

size_t q4o_l1_size(int n, int k, int group, int tsi, int cols)
{
    if (!l1_geom_ok(n, k, group, tsi, cols)) return 0;
    size_t tile = (size_t)tsi * (k / 2) + (size_t)tsi * (k / group) * 2;
    return (size_t)cols * (size_t)(n / cols / tsi) * tile;
}

/* Byte offset of the tile holding row i and its local row index.
 * crates/xnpu-cli/src/main.rs:2236-2241 */
static size_t l1_tile_off(int i, int n, int k, int group, int tsi, int cols, int *rr)
{
    size_t tile = (size_t)tsi * (k / 2) + (size_t)tsi * (k / group) * 2;
    int rows_per_col = n / cols;
    int col = i / rows_per_col;
    int r = i % rows_per_col;
    *rr = r % tsi;
    return ((size_t)col * (rows_per_col / tsi) + r / tsi) * tile;
}

/* Pack signed q[n][k] (-8..7) and bf16 scale bits s[n][k/group] into L1.
 * crates/xnpu-cli/src/main.rs:2231-2252 */
int q4o_l1_pack(const int8_t *q, const uint16_t *s, int n, int k, int group,
                int tsi, int cols, uint8_t *out)
{
    if (!l1_geom_ok(n, k, group, tsi, cols)) return Q4O_EINVAL;
    size_t nibble_bytes = (size_t)tsi * k / 2;
    int gpr = k / group;
    memset(out, 0, q4o_l1_size(n, k, group, tsi, cols));
    for (int i = 0; i < n; i++) {
        int rr;
        size_t off = l1_tile_off(i, n, k, group, tsi, cols, &rr);
        const int8_t *qi = q + (size_t)i * k;
        for (int p = 0; p < k / 2; p++)
            out[off + (size_t)rr * (k / 2) + p] =
                (uint8_t)(((uint8_t)qi[2 * p] & 0x0F) | (((uint8_t)qi[2 * p + 1] & 0x0F) << 4));
        for (int g = 0; g < gpr; g++) {
            uint16_t b = s[(size_t)i * gpr + g];
            size_t o = off + nibble_bytes + ((size_t)rr * gpr + g) * 2;
            out[o] = (uint8_t)(b & 0xff);
            out[o + 1] = (uint8_t)(b >> 8);
        }
    }
    return Q4O_OK;
}

/* Unpack L1 to signed q and scale bits (inverse of the packer). */
int q4o_l1_unpack(const uint8_t *pack, int n, int k, int group, int tsi, int cols,
                  int8_t *q, uint16_t *s)
{
    if (!l1_geom_ok(n, k, group, tsi, cols)) return Q4O_EINVAL;
    size_t nibble_bytes = (size_t)tsi * k / 2;
    int gpr = k / group;
    for (int i = 0; i < n; i++) {
        int rr;
        size_t off = l1_tile_off(i, n, k, group, tsi, cols, &rr);
        for (int p = 0; p < k / 2; p++) {
            uint8_t b = pack[off + (size_t)rr * (k / 2) + p];
            q[(size_t)i * k + 2 * p] = (int8_t)sext4(b & 0x0F);
            q[(size_t)i * k + 2 * p + 1] = (int8_t)sext4(b >> 4);
        }
        for (int g = 0; g < gpr; g++) {
            size_t o = off + nibble_bytes + ((size_t)rr * gpr + g) * 2;
            s[(size_t)i * gpr + g] = (uint16_t)(pack[o] | (pack[o + 1] << 8));
        }
    }
    return Q4O_OK;
}

/* Dequantize rows [r0, r1) of an L1 pack to bf16 bits, w[(i-r0)*k + kk]. */
int q4o_l1_dequant_rows(const uint8_t *pack, int n, int k, int group, int tsi, int cols,
                        int r0, int r1, uint16_t *w)
{
    if (!l1_geom_ok(n, k, group, tsi, cols) || r0 < 0 || r1 > n || r0 > r1) return Q4O_EINVAL;
    size_t nibble_bytes = (size_t)tsi * k / 2;
    int gpr = k / group;
    for (int i = r0; i < r1; i++) {
        int rr;
        size_t off = l1_tile_off(i, n, k, group, tsi, cols, &rr);
        uint16_t *wi = w + (size_t)(i - r0) * k;
        for (int kk = 0; kk < k; kk++) {
            uint8_t b = pack[off + (size_t)rr * (k / 2) + kk / 2];
            int qv = sext4((kk & 1) ? (b >> 4) : (b & 0x0F));
            size_t o = off + nibble_bytes + ((size_t)rr * gpr + kk / group) * 2;
            uint16_t sb = (uint16_t)(pack[o] | (pack[o + 1] << 8));
            wi[kk] = q4o_dequant_one(qv, sb);
        }
    }
    return Q4O_OK;
}

/* ------------------------------------------- layout L2 (w4gemvu v4/v5 "Q4NX")
 *
 * Blocks of ELEM=18560 bytes, each 16 rows x 2048 K, 8 logical columns.
 * Block (col, tile t, chunk c) sits at ((col*chunks + c)*t_num + t)*ELEM: the
 * chunk-major order of crates/xnpu-cli/src/main.rs:2928-2942 (block partials
 * of one column follow chunk-major, see w4u_read_c main.rs:3066-3091 and
 * w4u_c_at main.rs:3127-3141).  Inside a block, the nibble of (group g 0..63,
 * k 0..31, row r 0..15) is at byte g*256 + k*8 + r/2, even rows in the low
 * nibble; the bf16 scale at 16384 + (g*16 + r)*2 (main.rs:3097-3125).
 * The u32 words at ELEM-8 / ELEM-4 are the block's self-description; the
 * importer that writes real files (q4nx_import.py) is not shipped, so this
 * restatement writes K at ELEM-8 and the chunk index at ELEM-4 and no reader
 * depends on them.
 */
#define L2_ELEM 18560
#define L2_TILE_K 2048
#define L2_TILE_ROWS 16
#define L2_COLS 8

static int l2_geom_ok(int n, int k)
{
    return n > 0 && k > 0 && k % L2_TILE_K == 0 && n % (L2_COLS * L2_TILE_ROWS) == 0;
}

size_t q4o_l2_size(int n, int k)
{
    if (!l2_geom_ok(n, k)) return 0;
    /* 8 * w4u_blocks(m, k) * ELEM, crates/xnpu-cli/src/main.rs:3930 */
    return (size_t)L2_COLS * (n / L2_COLS / L2_TILE_ROWS) * (k / L2_TILE_K) * L2_ELEM;
}

static size_t l2_block_off(int row, int chunk, int n, int k, int *r)
{
    int chunks = k / L2_TILE_K;
    int t_num = n / L2_COLS / L2_TILE_ROWS;
    int rpc = n / L2_COLS;
    int col = row / rpc;
    int within = row % rpc;
    int t = within / L2_TILE_ROWS;
    *r = within % L2_TILE_ROWS;
    return (((size_t)col * chunks + chunk) * t_num + t) * L2_ELEM;
}

/* Pack signed q[n][k] and bf16 scales s[n][k/32] into L2 (group fixed at 32). */
int q4o_l2_pack(const int8_t *q, const uint16_t *s, int n, int k, uint8_t *out)
{
    if (!l2_geom_ok(n, k)) return Q4O_EINVAL;
    int chunks = k / L2_TILE_K;
    int gpr = k / 32;
    memset(out, 0, q4o_l2_size(n, k));
    for (int row = 0; row < n; row++) {
        for (int c = 0; c < chunks; c++) {
            int r;
            size_t off = l2_block_off(row, c, n, k, &r);
            for (int g = 0; g < 64; g++) {
                for (int kk = 0; kk < 32; kk++) {
                    int kg = c * L2_TILE_K + g * 32 + kk;
                    uint8_t nib = (uint8_t)q[(size_t)row * k + kg] & 0x0F;
                    size_t bo = off + (size_t)g * 256 + kk * 8 + r / 2;
                    if (r % 2 == 0) out[bo] = (uint8_t)((out[bo] & 0xF0) | nib);
                    else out[bo] = (uint8_t)((out[bo] & 0x0F) | (nib << 4));
                }
                uint16_t sb = s[(size_t)row * gpr + c * 64 + g];
                size_t so = off + 16384 + ((size_t)g * 16 + r) * 2;
                out[so] = (uint8_t)(sb & 0xff);
                out[so + 1] = (uint8_t)(sb >> 8);
            }
            /* self-description words: K and chunk index (see header note) */
            uint32_t kw = (uint32_t)k, cw = (uint32_t)c;
            memcpy(out + off + L2_ELEM - 8, &kw, 4);
            memcpy(out + off + L2_ELEM - 4, &cw, 4);
        }
    }
    return Q4O_OK;
}

/* Dequantize rows [r0, r1) of an L2 pack to bf16, chunk-aware generalisation of
 * w4u_row_bf16 (crates/xnpu-cli/src/main.rs:3102-3125). */
int q4o_l2_dequant_rows(const uint8_t *pack, int n, int k, int r0, int r1, uint16_t *w)
{
    if (!l2_geom_ok(n, k) || r0 < 0 || r1 > n || r0 > r1) return Q4O_EINVAL;
    int chunks = k / L2_TILE_K;
    for (int row = r0; row < r1; row++) {
        uint16_t *wr = w + (size_t)(row - r0) * k;
        for (int c = 0; c < chunks; c++) {
            int r;
            size_t off = l2_block_off(row, c, n, k, &r);
            for (int g = 0; g < 64; g++) {
                size_t sb = off + 16384 + ((size_t)g * 16 + r) * 2;
                uint16_t sbits = (uint16_t)(pack[sb] | (pack[sb + 1] << 8));
                for (int kk = 0; kk < 32; kk++) {
                    uint8_t b = pack[off + (size_t)g * 256 + kk * 8 + r / 2];
                    unsigned nib = (r % 2 == 0) ? (b & 0x0F) : (b >> 4);
                    wr[c * L2_TILE_K + g * 32 + kk] = q4o_dequant_one(sext4(nib), sbits);
                }
            }
        }
    }
    return Q4O_OK;
}

/* Literal restatement of w4u_row_bf16 (crates/xnpu-cli/src/main.rs:3102-3125),
 * including its offset formula, which omits the chunk index and is therefore
 * only valid for K=2048.  Kept to show the generalised reader agrees with the
 * reference where the reference is defined. */
int q4o_l2_row_ref(const uint8_t *pack, int m, int k, int row, uint16_t *out)
{
    if (k != 2048 || !l2_geom_ok(m, k) || row < 0 || row >= m) return Q4O_EINVAL;
    const int cols = 8, tr = 16;
    int chunks = k / 2048;
    int t_num = m / cols / tr;
    int col = row / (m / cols);
    int within = row % (m / cols);
    int t = within / tr;
    int r = within % tr;
    size_t off = ((size_t)col * t_num * chunks + t) * L2_ELEM;
    for (int g = 0; g < 64; g++) {
        size_t sb = off + 16384 + ((size_t)g * 16 + r) * 2;
        float sf = q4o_bf16_to_f32((uint16_t)(pack[sb] | (pack[sb + 1] << 8)));
        for (int kk = 0; kk < 32; kk++) {
            uint8_t b = pack[off + (size_t)g * 256 + kk * 8 + r / 2];
            unsigned nib = (r % 2 == 0) ? (b & 0x0F) : (b >> 4);
            int q = sext4(nib);
            out[g * 32 + kk] = q4o_f32_to_bf16((float)q * sf);
        }
    }
    return Q4O_OK;
}

/* --------------------------------------------------------- GEMV reference
 *
 * y[m][i] = sum_k w[i][k] * f32(x[m][k]), accumulated sequentially over k in
 * f32 and returned in f32 BEFORE the final RNE so callers can compare against
 * the unrounded value; q4o_f32_to_bf16 gives the reference's output.
 *   - over a packed layout or q/s planes, w = f32(q) * f32(scale) exactly, with
 *     no bf16 rounding of w: the reference's GEMV host reference,
 *     crates/xnpu-cli/src/main.rs:2287-2296 (`let w = nibble as f32 *
 *     scale; acc += w * bf16_to_f32(x)`);
 *   - over dequantized bf16 weights (q4o_gemv_bf16), w = the bf16 value: the
 *     importer's golden rows, tools/w4_import.py:55-63 (f32 matmul of the
 *     dequantized weights).
 * Rows are independent; threads split rows, each row keeps the reference's
 * sequential order, so the result does not depend on the thread count.
 */
typedef struct {
    int kind; /* 0: dequantized bf16 w; 1: L1 pack; 2: L2 pack; 3: q/s planes */
    const uint16_t *w;
    const int8_t *q;
    const uint16_t *s;
    const uint8_t *pack;
    int n, k, group, tsi, cols;
    const uint16_t *x;
    int m;
    float *y;
    int r0, r1;
} gemv_job;

#define ROW_BATCH 8

/* w = f32(q) * f32(scale), unrounded (main.rs:2289), for one row of a layout. */
static void row_f32(const gemv_job *j, int row, float *out)
{
    int k = j->k;
    switch (j->kind) {
    case 1: {
        int rr;
        size_t off = l1_tile_off(row, j->n, k, j->group, j->tsi, j->cols, &rr);
        size_t nibble_bytes = (size_t)j->tsi * k / 2;
        int gpr = k / j->group;
        for (int kk = 0; kk < k; kk++) {
            uint8_t b = j->pack[off + (size_t)rr * (k / 2) + kk / 2];
            int qv = sext4((kk & 1) ? (b >> 4) : (b & 0x0F));
            size_t o = off + nibble_bytes + ((size_t)rr * gpr + kk / j->group) * 2;
            out[kk] = (float)qv * q4o_bf16_to_f32((uint16_t)(j->pack[o] | (j->pack[o + 1] << 8)));
        }
        break;
    }
    case 2: {
        int chunks = k / L2_TILE_K;
        for (int c = 0; c < chunks; c++) {
            int r;
            size_t off = l2_block_off(row, c, j->n, k, &r);
            for (int g = 0; g < 64; g++) {
                size_t sb = off + 16384 + ((size_t)g * 16 + r) * 2;
                float sf = q4o_bf16_to_f32((uint16_t)(j->pack[sb] | (j->pack[sb + 1] << 8)));
                for (int kk = 0; kk < 32; kk++) {
                    uint8_t b = j->pack[off + (size_t)g * 256 + kk * 8 + r / 2];
                    unsigned nib = (r % 2 == 0) ? (b & 0x0F) : (b >> 4);
                    out[c * L2_TILE_K + g * 32 + kk] = (float)sext4(nib) * sf;
                }
            }
        }
        break;
    }
    default: { /* planes */
        const int8_t *q = j->q + (size_t)row * k;
        const uint16_t *s = j->s + (size_t)row * (k / 32);
        for (int kk = 0; kk < k; kk++) out[kk] = (float)q[kk] * q4o_bf16_to_f32(s[kk / 32]);
    }
    }
}

static void gemv_rows(const gemv_job *j)
{
    int k = j->k;
    /* scratch for rows of f32 weights (kinds 1-3) */
    float *scratch = NULL;
    if (j->kind != 0) {
        scratch = (float *)malloc((size_t)ROW_BATCH * k * sizeof(float));
        if (!scratch) return;
    }
    for (int i0 = j->r0; i0 < j->r1; i0 += ROW_BATCH) {
        int nb = j->r1 - i0 < ROW_BATCH ? j->r1 - i0 : ROW_BATCH;
        if (j->kind != 0)
            for (int b = 0; b < nb; b++) row_f32(j, i0 + b, scratch + (size_t)b * k);
        for (int mm = 0; mm < j->m; mm++) {
            const uint16_t *xm = j->x + (size_t)mm * k;
            float acc[ROW_BATCH] = {0};
            /* rows interleaved only to hide add latency; each row's own sum
             * stays strictly sequential in k */
            for (int kk = 0; kk < k; kk++) {
                float xv = q4o_bf16_to_f32(xm[kk]);
                for (int b = 0; b < nb; b++) {
                    float w = j->kind == 0 ? q4o_bf16_to_f32(j->w[(size_t)(i0 + b) * k + kk])
                                           : scratch[(size_t)b * k + kk];
                    float p = w * xv;
                    acc[b] = acc[b] + p;
                }
            }
            for (int b = 0; b < nb; b++) j->y[(size_t)mm * j->n + i0 + b] = acc[b];
        }
    }
    free(scratch);
}

static void *gemv_thread(void *arg)
{
    gemv_rows((const gemv_job *)arg);
    return NULL;
}

static int run_gemv(gemv_job base, int nthreads)
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > base.n) nthreads = base.n > 0 ? base.n : 1;
    if (nthreads == 1) {
        base.r0 = 0;
        base.r1 = base.n;
        gemv_rows(&base);
        return Q4O_OK;
    }
    pthread_t th[256];
    gemv_job jobs[256];
    int per = (base.n + nthreads - 1) / nthreads;
    per = (per + ROW_BATCH - 1) / ROW_BATCH * ROW_BATCH;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        jobs[t] = base;
        jobs[t].r0 = t * per < base.n ? t * per : base.n;
        jobs[t].r1 = (t + 1) * per < base.n ? (t + 1) * per : base.n;
        if (jobs[t].r0 >= jobs[t].r1) break;
        pthread_create(&th[t], NULL, gemv_thread, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return Q4O_OK;
}

/* y_f32[m][n] from dequantized bf16 weights w[n][k] and bf16 x[m][k]. */
int q4o_gemv_bf16(const uint16_t *w, const uint16_t *x, int m, int n, int k,
                  float *y, int nthreads)
{
    if (m <= 0 || n <= 0 || k <= 0) return Q4O_EINVAL;
    gemv_job j = {0};
    j.kind = 0; j.w = w; j.n = n; j.k = k; j.x = x; j.m = m; j.y = y;
    return run_gemv(j, nthreads);
}

/* Same, dequantizing each row from an L1 pack on the fly (the CPU baseline's
 * path: the reference's host reference over its own packed layout). */
int q4o_gemv_l1(const uint8_t *pack, int n, int k, int group, int tsi, int cols,
                const uint16_t *x, int m, float *y, int nthreads)
{
    if (m <= 0 || !l1_geom_ok(n, k, group, tsi, cols)) return Q4O_EINVAL;
    gemv_job j = {0};
    j.kind = 1; j.pack = pack; j.n = n; j.k = k; j.group = group; j.tsi = tsi;
    j.cols = cols; j.x = x; j.m = m; j.y = y;
    return run_gemv(j, nthreads);
}

/* Same over an L2 pack. */
int q4o_gemv_l2(const uint8_t *pack, int n, int k, const uint16_t *x, int m,
                float *y, int nthreads)
{
    if (m <= 0 || !l2_geom_ok(n, k)) return Q4O_EINVAL;
    gemv_job j = {0};
    j.kind = 2; j.pack = pack; j.n = n; j.k = k; j.x = x; j.m = m; j.y = y;
    return run_gemv(j, nthreads);
}

/* Same over q/s planes: q int8 [n][k] in [-8, 7], scale bits [n][k/32]. */
int q4o_gemv_q(const int8_t *q, const uint16_t *s, int n, int k, const uint16_t *x, int m,
               float *y, int nthreads)
{
    if (m <= 0 || n <= 0 || k <= 0 || k % 32) return Q4O_EINVAL;
    gemv_job j = {0};
    j.kind = 3; j.q = q; j.s = s; j.n = n; j.k = k; j.group = 32; j.x = x; j.m = m; j.y = y;
    return run_gemv(j, nthreads);
}

/* Round a f32 array to bf16 bits (the reference's final narrowing). */
void q4o_round_bf16(const float *y, size_t n, uint16_t *out)
{
    for (size_t i = 0; i < n; i++) out[i] = q4o_f32_to_bf16(y[i]);
}

/* ------------------------------------------------------------ KAT data
 * crates/xnpu-cli/src/main.rs:2225-2229: nibble(i,k) = ((13i+7k)%16)-8,
 * scale(g) = ((g%4)+1)/16, x[k] = (k%7)-3.  Every product and partial sum is
 * exact in f32, so the output is order-independent and bit-exact. */
void q4o_kat_fill(int n, int k, int group, int8_t *q, uint16_t *s, uint16_t *x)
{
    for (int i = 0; i < n; i++)
        for (int kk = 0; kk < k; kk++)
            q[(size_t)i * k + kk] = (int8_t)((int)((13 * (size_t)i + 7 * (size_t)kk) % 16) - 8);
    int gpr = k / group;
    for (int i = 0; i < n; i++)
        for (int g = 0; g < gpr; g++)
            s[(size_t)i * gpr + g] = q4o_f32_to_bf16((float)((g % 4) + 1) / 16.0f);
    for (int kk = 0; kk < k; kk++) x[kk] = q4o_f32_to_bf16((float)((kk % 7) - 3));
}

/* KAT host reference, literally main.rs:2287-2296: w = nibble*scale in f32
 * (no bf16 rounding; exact for this data), acc += w*x, one RNE. */
void q4o_kat_ref(int n, int k, int group, uint16_t *c_out)
{
    for (int i = 0; i < n; i++) {
        float acc = 0.0f;
        for (int kk = 0; kk < k; kk++) {
            float w = (float)((int)((13 * (size_t)i + 7 * (size_t)kk) % 16) - 8) *
                      ((float)((kk / group) % 4 + 1) / 16.0f);
            float xv = q4o_bf16_to_f32(q4o_f32_to_bf16((float)((kk % 7) - 3)));
            float p = w * xv;
            acc = acc + p;
        }
        c_out[i] = q4o_f32_to_bf16(acc);
    }
}

/* ------------------------------------------- W4A8 activation quantizer
 * Per-group-32 symmetric int8: d = RNE_bf16(amax/127), q = clamp(rne(x/d),
 * -127, 127); an all-zero group keeps q=0, d=0.
 * crates/xnpu-cli/src/main.rs:2955-2986 (scalar path). */
int q4o_quantize_x(const uint16_t *x, int k, int8_t *q, uint16_t *d)
{
    if (k % 32) return Q4O_EINVAL;
    int ng = k / 32;
    memset(q, 0, (size_t)k);
    memset(d, 0, (size_t)ng * 2);
    for (int g = 0; g < ng; g++) {
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            float v = fabsf(q4o_bf16_to_f32(x[g * 32 + j]));
            if (v > amax) amax = v;
        }
        if (amax == 0.0f) continue;
        uint16_t db = q4o_f32_to_bf16(amax / 127.0f);
        d[g] = db;
        float df = q4o_bf16_to_f32(db);
        for (int j = 0; j < 32; j++) {
            float v = q4o_bf16_to_f32(x[g * 32 + j]) / df;
            float r = nearbyintf(v); /* default rounding mode: ties-to-even */
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            q[g * 32 + j] = (int8_t)r;
        }
    }
    return Q4O_OK;
}

/* Sum K-chunk partials in f32 then round once: the K=6144 read-back rule of
 * w4u_read_c / w4u_c_at (crates/xnpu-cli/src/main.rs:3066-3091, :3127-3141).
 * parts[c][n] are bf16 bits; out[n] bf16 bits. */
void q4o_sum_chunk_partials(const uint16_t *parts, int chunks, int n, uint16_t *out)
{
    for (int i = 0; i < n; i++) {
        float acc = q4o_bf16_to_f32(parts[i]);
        for (int c = 1; c < chunks; c++) acc += q4o_bf16_to_f32(parts[(size_t)c * n + i]);
        out[i] = q4o_f32_to_bf16(acc);
    }
}

/* ------------------------------------------- W4A8 GEMV (parity mode)
 * The reference's NPU arithmetic for the w4gemvu kernel (int8 activations
 * from q4o_quantize_x, int4 weights; crates/xnpu-cli/src/main.rs:2912-2916:
 * mmul<4,16,16,int8,int4>): per 32-K group an exact int32 dot
 * T = sum q_w * q_x, scaled by the group's weight scale times the group's
 * activation scale and accumulated in f32 over one 2048-K chunk,
 * acc = fma(f32(s_w) * f32(d_x), f32(T), acc); each chunk's partial is
 * rounded to bf16 (the C tensor holds bf16), and the partials are summed in
 * f32 in chunk order (w4u_read_c, main.rs:3066-3091).  The order of the
 * scale products inside the device kernel is not recorded in the reference
 * (its IRON reference.py is not shipped); this restatement fixes it as above.
 * y[m][n] is that f32 sum, before the final bf16 narrowing. */
typedef struct {
    const int8_t *qw; const uint16_t *sw; const int8_t *qx; const uint16_t *dx;
    int n, k, m, r0, r1; float *y;
} w4a8_job;

static void *w4a8_rows(void *arg)
{
    const w4a8_job *j = (const w4a8_job *)arg;
    const int ng = j->k / 32;
    for (int t = 0; t < j->m; t++)
        for (int i = j->r0; i < j->r1; i++) {
            float total = 0.0f;
            for (int c0 = 0; c0 < j->k; c0 += 2048) {
                const int c1 = c0 + 2048 < j->k ? c0 + 2048 : j->k;
                float acc = 0.0f;
                for (int g = c0 / 32; g < c1 / 32; g++) {
                    int32_t T = 0;
                    for (int e = 0; e < 32; e++)
                        T += (int32_t)j->qw[(size_t)i * j->k + g * 32 + e] *
                             (int32_t)j->qx[(size_t)t * j->k + g * 32 + e];
                    const float sd = q4o_bf16_to_f32(j->sw[(size_t)i * ng + g]) *
                                     q4o_bf16_to_f32(j->dx[(size_t)t * ng + g]);
                    acc = fmaf(sd, (float)T, acc);
                }
                const float part = q4o_bf16_to_f32(q4o_f32_to_bf16(acc));
                total = c0 == 0 ? part : total + part;
            }
            j->y[(size_t)t * j->n + i] = total;
        }
    return NULL;
}

int q4o_gemv_w4a8(const int8_t *qw, const uint16_t *sw, int n, int k, const int8_t *qx,
                  const uint16_t *dx, int m, float *y, int nthreads)
{
    if (m <= 0 || n <= 0 || k <= 0 || k % 32) return Q4O_EINVAL;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 64) nthreads = 64;
    if (nthreads > n) nthreads = n;
    pthread_t th[64];
    w4a8_job jobs[64];
    const int per = (n + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        jobs[t] = (w4a8_job){qw, sw, qx, dx, n, k, m, t * per, (t + 1) * per < n ? (t + 1) * per : n, y};
        if (jobs[t].r0 >= jobs[t].r1) break;
        pthread_create(&th[t], NULL, w4a8_rows, &jobs[t]);
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    return Q4O_OK;
}

/* ------------------------------------------------------------------ decode-step glue */

/* RMSNorm of one token: sequential f32 sum of squares, inv = 1 / sqrt(mean +
 * 1e-5), out = RNE_bf16(x * inv * w).  crates/xnpu-cli/src/main.rs:4714-4724 */
void q4o_rms_norm_bf16(const uint16_t *x, const uint16_t *w, int k, float eps, uint16_t *out)
{
    float sum = 0.f;
    for (int i = 0; i < k; i++) {
        const float v = q4o_bf16_to_f32(x[i]);
        sum += v * v;
    }
    const float inv = 1.f / sqrtf(sum / (float)k + eps);
    for (int i = 0; i < k; i++) out[i] = q4o_f32_to_bf16(q4o_bf16_to_f32(x[i]) * inv * q4o_bf16_to_f32(w[i]));
}

/* out = RNE_bf16(a + b).  crates/xnpu-cli/src/main.rs:4726-4730 */
void q4o_add_bf16(const uint16_t *a, const uint16_t *b, size_t n, uint16_t *out)
{
    for (size_t i = 0; i < n; i++) out[i] = q4o_f32_to_bf16(q4o_bf16_to_f32(a[i]) + q4o_bf16_to_f32(b[i]));
}

/* silu(gate) * up over the halves of a fused [gate | up] vector of 2*half
 * values: out[i] = RNE_bf16(g * (1 / (1 + exp(-g))) * u).
 * crates/xnpu-cli/src/main.rs:4732-4745 (its scalar path) */
void q4o_swiglu_bf16(const uint16_t *x, int half, uint16_t *out)
{
    for (int i = 0; i < half; i++) {
        const float g = q4o_bf16_to_f32(x[i]);
        const float u = q4o_bf16_to_f32(x[half + i]);
        out[i] = q4o_f32_to_bf16(g * (1.f / (1.f + expf(-g))) * u);
    }
}

/* Llama rotate-half RoPE tables at one position: inv_freq = base^(-j/64),
 * c[j] = cos(pos * inv), s[j] = sin(pos * inv), j < 64.
 * crates/xnpu-cli/src/main.rs:4817-4827 */
void q4o_rope_table(int pos, float base, float *c, float *s)
{
    for (int j = 0; j < 64; j++) {
        const float inv = powf(base, -(float)j / 64.f);
        const float a = (float)pos * inv;
        c[j] = cosf(a);
        s[j] = sinf(a);
    }
}

/* RoPE on `heads` heads of 128: out[j] = RNE(x1 c - x2 s), out[64+j] =
 * RNE(x2 c + x1 s).  crates/xnpu-cli/src/main.rs:4829-4839 */
void q4o_rope_apply(const uint16_t *x, const float *c, const float *s, int heads, uint16_t *out)
{
    for (int h = 0; h < heads; h++) {
        const int o = h * 128;
        for (int j = 0; j < 64; j++) {
            const float x1 = q4o_bf16_to_f32(x[o + j]);
            const float x2 = q4o_bf16_to_f32(x[o + 64 + j]);
            out[o + j] = q4o_f32_to_bf16(x1 * c[j] - x2 * s[j]);
            out[o + 64 + j] = q4o_f32_to_bf16(x2 * c[j] + x1 * s[j]);
        }
    }
}

/* Per-head RMSNorm over 128 (the q/k norm applied after RoPE), weights [128]
 * shared by every head.  crates/xnpu-cli/src/main.rs:4844-4857 */
void q4o_qk_rms_bf16(const uint16_t *x, int len, const uint16_t *w, uint16_t *out)
{
    for (int h = 0; h < len / 128; h++) {
        const int o = h * 128;
        float sum = 0.f;
        for (int j = 0; j < 128; j++) {
            const float v = q4o_bf16_to_f32(x[o + j]);
            sum += v * v;
        }
        const float inv = 1.f / sqrtf(sum / 128.f + 1e-5f);
        for (int j = 0; j < 128; j++)
            out[o + j] = q4o_f32_to_bf16(q4o_bf16_to_f32(x[o + j]) * inv * q4o_bf16_to_f32(w[j]));
    }
}

/* GQA decode attention for the token at position pos over a bf16 KV cache
 * laid out [nkv][cache_seq][128]: per q-head, scores = (K q) / sqrt(128)
 * summed sequentially over the 128 dims, softmax with the max subtracted,
 * acc = sum_t w_t v_t in ascending t, out = RNE(acc / sum).  The scalar path
 * of crates/xnpu-cli/src/main.rs:4967-5033. */
int q4o_attention_bf16(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, int pos, int cache_seq,
                       int heads, int nkv, uint16_t *out)
{
    if (heads <= 0 || nkv <= 0 || heads % nkv || pos < 0 || pos >= cache_seq) return Q4O_EINVAL;
    const int s = pos + 1, group = heads / nkv;
    float *sc = (float *)malloc(sizeof(float) * (size_t)s);
    if (!sc) return Q4O_EINVAL;
    for (int kv = 0; kv < nkv; kv++) {
        const size_t base = (size_t)kv * cache_seq * 128;
        for (int h = kv * group; h < (kv + 1) * group; h++) {
            const int qo = h * 128;
            float mx = -INFINITY;
            for (int t = 0; t < s; t++) {
                float d = 0.f;
                for (int j = 0; j < 128; j++)
                    d += q4o_bf16_to_f32(kc[base + (size_t)t * 128 + j]) * q4o_bf16_to_f32(q[qo + j]);
                sc[t] = d / sqrtf(128.f);
                mx = fmaxf(mx, sc[t]);
            }
            float sum = 0.f;
            for (int t = 0; t < s; t++) {
                sc[t] = expf(sc[t] - mx);
                sum += sc[t];
            }
            float acc[128];
            for (int j = 0; j < 128; j++) acc[j] = 0.f;
            for (int t = 0; t < s; t++)
                for (int j = 0; j < 128; j++) acc[j] += sc[t] * q4o_bf16_to_f32(vc[base + (size_t)t * 128 + j]);
            for (int j = 0; j < 128; j++) out[qo + j] = q4o_f32_to_bf16(acc[j] / sum);
        }
    }
    free(sc);
    return Q4O_OK;
}
