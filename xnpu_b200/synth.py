"""Seeded synthetic inputs for the int4 path (no datasets or checkpoints).

Distributions (the benchmark configurations of the int4 decode/prefill path):
  * codes: uniform integers in [0, 15], q = code - 8 (zero point 8).  Stored as
    the reference's two's-complement nibble q & 0xF == code ^ 8, two per byte,
    low nibble first along K (tools/w4_import.py:4-6).  A uniformly random byte
    holds two independent uniform codes, so the packed code plane is drawn as
    random bytes.
  * scales: |N(0, 0.02)| / 7.5 in f32, rounded RNE to bf16, clamped to >= 2^-14;
    such a value is exactly representable in both bf16 (the reference layout's
    scale type) and fp16, so both readings agree bit for bit.
  * activations: N(0, 1) in f32 rounded RNE to bf16.
Each tensor has its own numpy Generator(PCG64(seed)).
"""
import numpy as np

SCALE_MIN_BF16 = 0x3880  # 2**-14


def f32_to_bf16_bits(a):
    """RNE f32 -> bf16 bits, the bit trick of crates/xnpu-cli/src/main.rs:338-343."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def synth_codes(n, k, seed):
    """Packed signed-nibble code plane [n, k//2] (uint8): the raw 64-bit
    outputs of PCG64(seed), as little-endian bytes."""
    nbytes = n * (k // 2)
    words = np.random.PCG64(seed).random_raw(-(-nbytes // 8))
    return words.astype("<u8").view(np.uint8)[:nbytes].reshape(n, k // 2)


def synth_scales(n, k, seed, group=32):
    """bf16 scale bits [n, k//group]."""
    rng = np.random.Generator(np.random.PCG64(seed + 0x9E3779B1))
    s = np.abs(rng.standard_normal(n * (k // group), dtype=np.float32) * np.float32(0.02)) / np.float32(7.5)
    bits = f32_to_bf16_bits(s)
    bits = np.maximum(bits, np.uint16(SCALE_MIN_BF16))  # positive bf16 order == bit order
    return bits.reshape(n, k // group)


def synth_x(m, k, seed):
    """bf16 activation bits [m, k]."""
    rng = np.random.Generator(np.random.PCG64(seed + 0x7F4A7C15))
    return f32_to_bf16_bits(rng.standard_normal(m * k, dtype=np.float32)).reshape(m, k)


def planes_bytes(codes, scales):
    """The PLANES import image: code plane then scale plane (little-endian)."""
    return np.concatenate([codes.reshape(-1), scales.astype("<u2").reshape(-1).view(np.uint8)])


def unpack_codes_signed(codes):
    """[n, k//2] packed nibbles -> int8 q [n, k]."""
    lo = (codes & 0x0F).astype(np.int8)
    hi = (codes >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo).astype(np.int8)
    hi = np.where(hi >= 8, hi - 16, hi).astype(np.int8)
    q = np.empty((codes.shape[0], codes.shape[1] * 2), dtype=np.int8)
    q[:, 0::2] = lo
    q[:, 1::2] = hi
    return q


def pack_codes_signed(q):
    """int8 q [n, k] in [-8, 7] -> packed nibbles [n, k//2]."""
    u = (np.asarray(q, dtype=np.int8).astype(np.uint8) & 0x0F)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)
