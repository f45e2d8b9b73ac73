// repack.cpp -- offline repacker: the reference's int4 layouts -> XQ4G.
//
// Inputs are the layouts the reference writes and reads:
//   L1     w4gemv2 tiles (crates/xnpu-cli/src/main.rs:2186-2252,
//          tools/w4_import.py:4-14; size check main.rs:2597)
//   L2     w4gemvu v4/v5 16x2048 blocks, chunk-major (main.rs:2912-2949,
//          :3097-3125, :3127-3141)
//   PLANES row-major codes + scales (signed or zero-point-8 codes, bf16 or
//          fp16 scales), for weights that come from elsewhere.
// Output: XQ4G (xq4_layout.h).  The repacker moves nibbles and scale bits
// without arithmetic, so the dequantized values RNE_bf16(q*s) of the output
// are those of the input, bit for bit.
#include <cstdint>
#include <cstring>
#include <cstdio>
#include <string>
#include <thread>
#include <vector>
#include <algorithm>

#include "xq4_layout.h"
#include "xq4_internal.h"

namespace {

constexpr int kL2Elem = 18560;   // W4U_ELEM, crates/xnpu-cli/src/main.rs:2927
constexpr int kL2TileK = 2048;   // W4U_TILE_K, main.rs:2929
constexpr int kL2TileRows = 16;  // W4U_TILE_ROWS, main.rs:2930
constexpr int kL2Cols = 8;

// fp16 bits -> bf16 bits when the value is exactly representable, else -1.
int fp16_to_bf16_exact(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    int exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t f;
    if (exp == 0x1f) {
        f = sign | 0x7f800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            f = sign;
        } else {  // subnormal fp16: normalise
            int e = -14;
            while (!(man & 0x400)) { man <<= 1; e--; }
            man &= 0x3ff;
            f = sign | ((uint32_t)(e + 127) << 23) | (man << 13);
        }
    } else {
        f = sign | ((uint32_t)(exp - 15 + 127) << 23) | (man << 13);
    }
    if (f & 0xffffu) return -1;  // needs more than bf16's 8 significant bits
    return (int)(f >> 16);
}

struct Source {
    const uint8_t *src;
    size_t len;
    xq4_layout_desc d;

    // Fill codes[0..cnt) (unsigned, q+8) for row `row`, K [k0, k0+cnt).
    void codes(int row, int k0, int cnt, uint8_t *out) const
    {
        switch (d.layout) {
        case XQ4_LAYOUT_L1: {
            int rows_per_col = d.n / d.cols;
            int col = row / rows_per_col, r = row % rows_per_col, rr = r % d.tsi;
            size_t tile = (size_t)d.tsi * (d.k / 2) + (size_t)d.tsi * (d.k / d.group) * 2;
            size_t off = ((size_t)col * (rows_per_col / d.tsi) + r / d.tsi) * tile +
                         (size_t)rr * (d.k / 2);
            for (int i = 0; i < cnt; i++) {
                int kk = k0 + i;
                uint8_t b = src[off + kk / 2];
                uint8_t nib = (kk & 1) ? (b >> 4) : (b & 0x0F);
                out[i] = nib ^ 8;  // two's complement -> q + 8
            }
            break;
        }
        case XQ4_LAYOUT_L2: {
            int chunks = d.k / kL2TileK, t_num = d.n / kL2Cols / kL2TileRows;
            int rpc = d.n / kL2Cols;
            int col = row / rpc, within = row % rpc;
            int t = within / kL2TileRows, r = within % kL2TileRows;
            for (int i = 0; i < cnt; i++) {
                int kk = k0 + i;
                int c = kk / kL2TileK, kc = kk % kL2TileK;
                size_t off = (((size_t)col * chunks + c) * t_num + t) * kL2Elem;
                uint8_t b = src[off + (size_t)(kc / 32) * 256 + (kc % 32) * 8 + r / 2];
                uint8_t nib = (r % 2 == 0) ? (b & 0x0F) : (b >> 4);
                out[i] = nib ^ 8;
            }
            break;
        }
        default: {  // PLANES
            const uint8_t *rowp = src + (size_t)row * (d.k / 2);
            for (int i = 0; i < cnt; i++) {
                int kk = k0 + i;
                uint8_t b = rowp[kk / 2];
                uint8_t nib = (kk & 1) ? (b >> 4) : (b & 0x0F);
                out[i] = d.code_format == XQ4_CODE_S4 ? (uint8_t)(nib ^ 8) : nib;
            }
        }
        }
    }

    // bf16 bits of the scale of (row, group g); -1 if not representable.
    int scale(int row, int g) const
    {
        switch (d.layout) {
        case XQ4_LAYOUT_L1: {
            int rows_per_col = d.n / d.cols;
            int col = row / rows_per_col, r = row % rows_per_col, rr = r % d.tsi;
            int gpr = d.k / d.group;
            size_t tile = (size_t)d.tsi * (d.k / 2) + (size_t)d.tsi * gpr * 2;
            size_t off = ((size_t)col * (rows_per_col / d.tsi) + r / d.tsi) * tile +
                         (size_t)d.tsi * (d.k / 2) + ((size_t)rr * gpr + g) * 2;
            return src[off] | (src[off + 1] << 8);
        }
        case XQ4_LAYOUT_L2: {
            int chunks = d.k / kL2TileK, t_num = d.n / kL2Cols / kL2TileRows;
            int rpc = d.n / kL2Cols;
            int col = row / rpc, within = row % rpc;
            int t = within / kL2TileRows, r = within % kL2TileRows;
            int c = g / 64, gl = g % 64;
            size_t off = (((size_t)col * chunks + c) * t_num + t) * kL2Elem + 16384 +
                         ((size_t)gl * 16 + r) * 2;
            return src[off] | (src[off + 1] << 8);
        }
        default: {
            size_t off = d.scale_offset + ((size_t)row * (d.k / d.group) + g) * 2;
            uint16_t v = (uint16_t)(src[off] | (src[off + 1] << 8));
            return d.scale_dtype == XQ4_SCALE_FP16 ? fp16_to_bf16_exact(v) : v;
        }
        }
    }
};

size_t source_bytes(const xq4_layout_desc &d)
{
    switch (d.layout) {
    case XQ4_LAYOUT_L1: {
        size_t tile = (size_t)d.tsi * (d.k / 2) + (size_t)d.tsi * (d.k / d.group) * 2;
        return (size_t)d.cols * (size_t)(d.n / d.cols / d.tsi) * tile;
    }
    case XQ4_LAYOUT_L2:
        return (size_t)kL2Cols * (d.n / kL2Cols / kL2TileRows) * (d.k / kL2TileK) * kL2Elem;
    default:
        return d.scale_offset + (size_t)d.n * (d.k / d.group) * 2;
    }
}

}  // namespace

// Validate a layout descriptor against the source length; fills row range.
int xq4_check_desc(const xq4_layout_desc *desc, size_t src_len, int *r0, int *r1)
{
    if (!desc) return xq4_fail(XQ4_EINVAL, "layout desc is NULL");
    const xq4_layout_desc &d = *desc;
    if (d.n <= 0 || d.k <= 0) return xq4_fail(XQ4_EINVAL, "n and k must be positive (n=%d k=%d)", d.n, d.k);
    if (d.group != 32) return xq4_fail(XQ4_EINVAL, "group must be 32 (got %d)", d.group);
    if (d.k % 32) return xq4_fail(XQ4_EINVAL, "k must be a multiple of 32 (got %d)", d.k);
    switch (d.layout) {
    case XQ4_LAYOUT_L1:
        if (d.tsi <= 0 || d.cols <= 0 || d.n % d.cols || (d.n / d.cols) % d.tsi)
            return xq4_fail(XQ4_EINVAL, "L1 geometry: n=%d must split into cols=%d x tiles of tsi=%d rows",
                            d.n, d.cols, d.tsi);
        break;
    case XQ4_LAYOUT_L2:
        if (d.k % kL2TileK || d.n % (kL2Cols * kL2TileRows))
            return xq4_fail(XQ4_EINVAL, "L2 geometry: k=%d must be a multiple of 2048 and n=%d of 128",
                            d.k, d.n);
        break;
    case XQ4_LAYOUT_PLANES:
        if (d.code_format != XQ4_CODE_S4 && d.code_format != XQ4_CODE_U4_ZP8)
            return xq4_fail(XQ4_EINVAL, "unknown code_format %d", d.code_format);
        if (d.scale_dtype != XQ4_SCALE_BF16 && d.scale_dtype != XQ4_SCALE_FP16)
            return xq4_fail(XQ4_EINVAL, "unknown scale_dtype %d", d.scale_dtype);
        if (d.scale_offset < (size_t)d.n * (d.k / 2))
            return xq4_fail(XQ4_EINVAL, "scale plane (offset %zu) overlaps the code plane (%zu bytes)",
                            d.scale_offset, (size_t)d.n * (d.k / 2));
        break;
    default:
        return xq4_fail(XQ4_EINVAL, "unknown layout %d", d.layout);
    }
    size_t need = source_bytes(d);
    if (src_len < need)
        return xq4_fail(XQ4_EINVAL, "source is %zu bytes, layout needs %zu (stale import?)", src_len, need);
    int a = d.row_begin, b = d.row_end;
    if (a == 0 && b == 0) b = d.n;
    if (a < 0 || b > d.n || a >= b)
        return xq4_fail(XQ4_EINVAL, "row range [%d, %d) outside [0, %d)", a, b, d.n);
    *r0 = a;
    *r1 = b;
    return XQ4_OK;
}

// Repack rows [r0, r1) of src into XQ4G at dst (xq4g_bytes(r1-r0, k) bytes).
int xq4_repack_rows(const void *src, size_t src_len, const xq4_layout_desc *desc, int r0, int r1,
                    uint8_t *dst)
{
    Source s{(const uint8_t *)src, src_len, *desc};
    const int n = r1 - r0, k = desc->k;
    const int NB = xq4g_nb(n), KC = xq4g_kc(k);
    // placement of the 16x64 weights of a unit (thread-safe static init)
    struct Pos { int byte[16][64], nib[16][64]; };
    static const Pos pos = [] {
        Pos p;
        for (int r = 0; r < 16; r++)
            for (int kk = 0; kk < 64; kk++) xq4g_locate(r, kk, &p.byte[r][kk], &p.nib[r][kk]);
        return p;
    }();
    unsigned hw = std::thread::hardware_concurrency();
    int nth = (int)std::min<unsigned>(hw ? hw : 1, 64);
    nth = std::max(1, std::min(nth, NB));
    std::vector<int> fail(nth, 0);
    auto work = [&](int tid) {
        uint8_t codes[64];
        for (int rb = tid; rb < NB; rb += nth) {
            for (int kc = 0; kc < KC; kc++) {
                uint8_t *u = dst + ((size_t)rb * KC + kc) * XQ4G_UNIT_BYTES;
                uint32_t words[128];
                for (int i = 0; i < 128; i++) words[i] = 0x88888888u;  // q = 0 padding
                uint16_t sc[16][2] = {};
                for (int r = 0; r < 16; r++) {
                    int row = rb * 16 + r;
                    if (row >= n) break;
                    int kvalid = std::min(64, k - kc * 64);
                    s.codes(r0 + row, kc * 64, kvalid, codes);
                    for (int kk = 0; kk < kvalid; kk++) {
                        int w = pos.byte[r][kk] / 4, nb = pos.nib[r][kk] * 4;
                        words[w] = (words[w] & ~(0xFu << nb)) | ((uint32_t)codes[kk] << nb);
                    }
                    for (int grp = 0; grp < 2; grp++) {
                        int g = kc * 2 + grp;
                        if (g * 32 >= k) break;
                        int v = s.scale(r0 + row, g);
                        if (v < 0) { fail[tid] = 1; v = 0; }
                        sc[r][grp] = (uint16_t)v;
                    }
                }
                memcpy(u, words, XQ4G_CODE_BYTES);
                for (int r = 0; r < 16; r++)
                    for (int grp = 0; grp < 2; grp++) {
                        int o = xq4g_scale_off(r, grp);
                        u[o] = (uint8_t)(sc[r][grp] & 0xff);
                        u[o + 1] = (uint8_t)(sc[r][grp] >> 8);
                    }
            }
        }
    };
    if (nth == 1) {
        work(0);
    } else {
        std::vector<std::thread> th;
        for (int t = 0; t < nth; t++) th.emplace_back(work, t);
        for (auto &t : th) t.join();
    }
    for (int f : fail)
        if (f) return xq4_fail(XQ4_EINVAL, "an fp16 scale is not exactly representable in bf16");
    return XQ4_OK;
}

extern "C" size_t xq4_gpu_layout_bytes(int n, int k)
{
    if (n <= 0 || k <= 0 || k % 32) return 0;
    return xq4g_bytes(n, k);
}

extern "C" int xq4_repack_host(const void *src, size_t src_len, const xq4_layout_desc *desc,
                               void *dst, size_t dst_len)
{
    xq4_clear_error();
    if (!src || !dst) return xq4_fail(XQ4_EINVAL, "src/dst is NULL");
    int r0, r1;
    int rc = xq4_check_desc(desc, src_len, &r0, &r1);
    if (rc) return rc;
    size_t need = xq4g_bytes(r1 - r0, desc->k);
    if (dst_len < need) return xq4_fail(XQ4_EINVAL, "dst is %zu bytes, need %zu", dst_len, need);
    return xq4_repack_rows(src, src_len, desc, r0, r1, (uint8_t *)dst);
}
