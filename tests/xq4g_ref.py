"""Numpy decoder of the XQ4G GPU layout, written from its specification in
xnpu_b200/csrc/xq4_layout.h (test helper, independent of the C++ repacker)."""
import numpy as np

UNIT = 576


def decode(img, n, k):
    """XQ4G image -> (q int8 [n, k], scale bits uint16 [n, k//32],
    q of the padded image, scales of the padded image)."""
    nb, kc = -(-n // 16), -(-k // 64)
    u = np.frombuffer(np.asarray(img, dtype=np.uint8).tobytes()[: nb * kc * UNIT], dtype=np.uint8)
    u = u.reshape(nb, kc, UNIT)
    words = u[:, :, :512].copy().view("<u4").reshape(nb, kc, 32, 4)  # [rb, kc, lane, j]
    q = np.zeros((nb * 16, kc * 64), dtype=np.int8)
    lane = np.arange(32)
    g, t = lane // 4, lane % 4
    rb = np.arange(nb)[:, None, None]
    ch = np.arange(kc)[None, :, None]
    for j in range(4):
        G, H = j >> 1, j & 1  # word j: scale group G, half H
        w = words[:, :, :, j]
        for s in range(4):
            for odd in range(2):
                nib = ((w >> np.uint32(4 * (s + 4 * odd))) & np.uint32(0xF)).astype(np.int16) - 8
                rows = rb * 16 + (g + 8 * (s & 1))[None, None, :]
                cols = ch * 64 + (32 * G + 8 * t + 4 * H + 2 * (s >> 1) + odd)[None, None, :]
                q[np.broadcast_to(rows, nib.shape), np.broadcast_to(cols, nib.shape)] = nib
    sc = u[:, :, 512:576].copy().view("<u2").reshape(nb, kc, 8, 2, 2)  # [rb, kc, g, grp, rhi]
    s_full = np.zeros((nb * 16, kc * 2), dtype=np.uint16)
    for gg in range(8):
        for grp in range(2):
            for rhi in range(2):
                r = (np.arange(nb) * 16 + gg + 8 * rhi)[:, None]
                c = (np.arange(kc) * 2 + grp)[None, :]
                s_full[r, c] = sc[:, :, gg, grp, rhi]
    return q[:n, :k], s_full[:n, : k // 32], q, s_full
