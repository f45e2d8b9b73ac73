// xq4_layout.h -- the GPU-resident int4 weight layout ("XQ4G") shared by the
// host repacker and the sm_100a kernels.
//
// The reference stores int4 weights in layouts built for AIE tiles: L1 (tiles
// of tsi rows, per-row nibble runs then per-row scales; crates/xnpu-cli/src/
// main.rs:2186-2252) and L2 (16-row x 2048-K blocks, group-major nibbles,
// transposed scales; main.rs:2912-2949, :3097-3125).  Neither suits a GPU warp:
// the GPU wants each lane's 16-byte load to hold exactly the nibbles one
// tensor-core fragment consumes, and the scales for those nibbles next to them
// so one stream feeds both.  XQ4G is that layout.
//
//   Rows padded to NP = ceil(n/16)*16, K padded to KP = ceil(k/64)*64
//   (k must be a multiple of 32).  NB = NP/16 row blocks, KC = KP/64 chunks.
//   Unit (rb, kc) = 16 rows x 64 K (two 32-K scale groups), UNIT_BYTES = 576,
//   at (rb*KC + kc)*576:
//     [0, 512)   codes.  Lane l (g = l>>2, t = l&3) owns bytes [16l, 16l+16):
//                rows g and g+8 of the block, K offsets 8t..8t+7 of each of
//                the chunk's two groups, as 4 little-endian u32 words.  Word
//                j = 2G + H is the mma.m16n8k16 A fragment of K step j, which
//                covers group G (0/1), half H (0/1).  Within word j, nibble s
//                and nibble s+4 (s = 0..3) hold one consecutive-K pair:
//                  s=0: row g,   k = 32G + 8t + 4H + 0, +1   (A reg 0)
//                  s=1: row g+8, k = 32G + 8t + 4H + 0, +1   (A reg 1)
//                  s=2: row g,   k = 32G + 8t + 4H + 2, +3   (A reg 2)
//                  s=3: row g+8, k = 32G + 8t + 4H + 2, +3   (A reg 3)
//                Nibble value = q + 8.  The MMA's K slots 2t,2t+1 / 2t+8,2t+9
//                are thus bound to actual K 32G+8t+4H+{0,1} / {2,3}: every K
//                step stays inside one scale group (so a group's scale can be
//                applied to the step's result), and the matching B fragment of
//                lane (g, t) is the 8 contiguous bytes x[tok][32G+8t+4H ..+4],
//                i.e. one 16-byte run per group.  (A dot product does not
//                depend on the order of K.)
//     [512, 576) scales, bf16.  Row pair g (rows g, g+8) owns the 8 bytes at
//                512 + 8g: [s(g, grp0), s(g+8, grp0), s(g, grp1), s(g+8, grp1)].
//   Padding rows / K: code 8 (q = 0) and scale 0, so every padded weight is +0.
//
// With the "128 + code" bf16 bit trick, (word >> 4s) & 0x000F000F | 0x43004300
// yields a bf16x2 pair (128+code_lo, 128+code_hi) = (q_lo+136, q_hi+136),
// exactly.
#pragma once
#include <stdint.h>
#include <stddef.h>

#define XQ4G_ROWS 16
#define XQ4G_KCHUNK 64
#define XQ4G_GROUP 32
#define XQ4G_CODE_BYTES 512
#define XQ4G_UNIT_BYTES 576

static inline int xq4g_nb(int n) { return (n + XQ4G_ROWS - 1) / XQ4G_ROWS; }
static inline int xq4g_kc(int k) { return (k + XQ4G_KCHUNK - 1) / XQ4G_KCHUNK; }
static inline size_t xq4g_bytes(int n, int k)
{
    return (size_t)xq4g_nb(n) * (size_t)xq4g_kc(k) * XQ4G_UNIT_BYTES;
}

// Position of weight (row r16 within the 16-row block, k64 within the 64-K
// chunk) inside its unit: byte offset of its u32 word and nibble index 0..7.
static inline void xq4g_locate(int r16, int k64, int *byte_off, int *nib)
{
    int G = k64 >> 5;          // scale group within the chunk
    int kg = k64 & 31;         // K within the group
    int t = kg >> 3;           // lane & 3
    int H = (kg >> 2) & 1;     // half of the group covered by the K step
    int pr = (kg >> 1) & 1;    // second pair of the step's four K -> s += 2
    int odd = kg & 1;          // odd K -> high nibble (s + 4)
    int g = r16 & 7;
    int rhi = r16 >> 3;        // row g+8 -> s += 1
    int lane = g * 4 + t;
    int j = 2 * G + H;
    *byte_off = lane * 16 + j * 4;
    *nib = pr * 2 + rhi + 4 * odd;
}

// Byte offset of the scale of (row r16, group grp 0/1) inside its unit.
static inline int xq4g_scale_off(int r16, int grp)
{
    return XQ4G_CODE_BYTES + 8 * (r16 & 7) + 4 * grp + 2 * (r16 >> 3);
}
