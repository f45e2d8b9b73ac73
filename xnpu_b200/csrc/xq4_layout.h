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
//   Unit (rb, kc) = 16 rows x 64 K, UNIT_BYTES = 576, at (rb*KC + kc)*576:
//     [0, 512)   codes.  Lane l (g = l>>2, t = l&3) owns bytes [16l, 16l+16):
//                rows g and g+8 of the block, K offsets [16t, 16t+16) of the
//                chunk, as 4 little-endian u32 words.  Word j, nibble s and
//                nibble s+4 (s = 0..3) hold one consecutive-K pair:
//                  s=0: row g,   k = 16t+4j+0, +1   (mma.m16n8k16 A reg 0)
//                  s=1: row g+8, k = 16t+4j+0, +1   (A reg 1)
//                  s=2: row g,   k = 16t+4j+2, +3   (A reg 2)
//                  s=3: row g+8, k = 16t+4j+2, +3   (A reg 3)
//                Nibble value = q + 8.  Word j is the A fragment of K step j:
//                the MMA's K slots 2t,2t+1 / 2t+8,2t+9 are bound to actual
//                K 16t+4j+{0,1} / {2,3}, so the matching B fragment of lane
//                (g, t) is the 8 contiguous bytes x[tok][16t+4j .. +4] and a
//                lane's activation slice for the whole chunk is 32 contiguous
//                bytes.  (A dot product does not depend on the order of K.)
//     [512, 576) scales, bf16.  Row pair g (rows g, g+8) owns the 8 bytes at
//                512 + 8g: [s(g, grp0), s(g+8, grp0), s(g, grp1), s(g+8, grp1)]
//                with grp0/grp1 the chunk's first/second 32-K group; lane
//                (g, t) needs only the u32 at 512 + 8g + 4(t>>1).
//   Padding rows / K: code 8 (q = 0) and scale 0, so every padded weight is +0.
//
// With the "128 + code" bf16 bit trick, (word >> 4s) & 0x000F000F | 0x43004300
// yields a bf16x2 pair (128+code_lo, 128+code_hi); subtracting 136 gives q
// exactly, and one bf16x2 multiply by the scale gives RNE_bf16(q * s): the
// reference's dequantized value, bit for bit.
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
    int t = k64 >> 4;          // lane & 3
    int j = (k64 >> 2) & 3;    // word (K step)
    int pr = (k64 >> 1) & 1;   // second pair of the word's four K -> s += 2
    int odd = k64 & 1;         // odd K -> high nibble (s + 4)
    int g = r16 & 7;
    int rhi = r16 >> 3;        // row g+8 -> s += 1
    int lane = g * 4 + t;
    *byte_off = lane * 16 + j * 4;
    *nib = pr * 2 + rhi + 4 * odd;
}

// Byte offset of the scale of (row r16, group grp 0/1) inside its unit.
static inline int xq4g_scale_off(int r16, int grp)
{
    return XQ4G_CODE_BYTES + 8 * (r16 & 7) + 4 * grp + 2 * (r16 >> 3);
}
