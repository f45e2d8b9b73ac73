"""Offline w4 importer: safetensors -> group-32 symmetric int4 -> L1 tiles.

The B200 counterpart of the reference's tools/w4_import.py (:1-134): read a
model's decode projections from a .safetensors file, quantize each fused
projection to signed int4 per 32-wide group with a bf16 scale, pack it in the
L1 tile layout (the w4gemv2 ABI that xq4_weight_import reads with
XQ4_LAYOUT_L1), and write one .bin per layer and fused shape, a meta.json and
one golden spot-check file per shape in the reference's raw format
(tools/w4_import.py:66-76).

Quantization rule.  The reference calls IRON's quantize_and_pack
(w4gemv2/reference.py, not part of the reference tree, so its exact rounding
is not available here: parity unpinned).  This module restates the rule its
docstring names (tools/w4_import.py:4-6): per row and 32-wide group,
scale = amax / 7 rounded to bf16 (round to nearest even), q = round-half-even
(w / scale) clamped to [-8, 7], stored as two's-complement nibbles; an
all-zero group gets scale 0 and q = 0.

Layout L1 (crates/xnpu-cli/src/main.rs:2186-2191, :2231-2252): the n rows are
split over `cols` columns of n/cols rows, each column into tiles of `tsi`
rows; a tile is [tsi*k/2 nibble bytes | tsi*(k/32) bf16 scales], nibble byte
rr*(k/2)+p holding k = 2p in the low nibble and 2p+1 in the high nibble, the
scale of (row rr, group g) at nibble_bytes + (rr*(k/32) + g)*2; tiles are
stored column by column.

Run:  python -m xnpu_b200.importer --model model.safetensors --out build/w4 --layers 0 1
"""
import argparse
import json
import struct
import sys
from pathlib import Path

import numpy as np

GROUP = 32

# Fused decode projections of a Llama-style layer: name -> (parts, tsi).
# The parts are concatenated along the rows in this order (the reference's
# SHAPES table, tools/w4_import.py:48-53); tsi as the reference's fixtures.
LLAMA_SHAPES = {
    "qkv": ((("self_attn", "q_proj"), ("self_attn", "k_proj"), ("self_attn", "v_proj")), 16),
    "o": ((("self_attn", "o_proj"),), 16),
    "gateup": ((("mlp", "gate_proj"), ("mlp", "up_proj")), 16),
    "down": ((("mlp", "down_proj"),), 4),
}

_ST_DTYPES = {"BF16": (2, "bf16"), "F16": (2, np.float16), "F32": (4, np.float32)}


# ------------------------------------------------------------------ safetensors
class SafeTensors:
    """Minimal reader of the .safetensors format (u64 header length, JSON
    header of {name: {dtype, shape, data_offsets}}, raw little-endian data)."""

    def __init__(self, path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            self.header = json.loads(f.read(hlen))
        self.base = 8 + hlen
        self.header.pop("__metadata__", None)

    def names(self):
        return list(self.header)

    def shape(self, name):
        return tuple(self.header[name]["shape"])

    def get_f32(self, name):
        """The tensor as float32 (bf16 and f16 widen exactly)."""
        h = self.header[name]
        if h["dtype"] not in _ST_DTYPES:
            raise ValueError(f"{name}: dtype {h['dtype']} not supported")
        size, kind = _ST_DTYPES[h["dtype"]]
        b0, b1 = h["data_offsets"]
        raw = np.fromfile(self.path, dtype=np.uint8, count=b1 - b0, offset=self.base + b0)
        if kind == "bf16":
            a = (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            a = raw.view(np.dtype(kind).newbyteorder("<")).astype(np.float32)
        return a.reshape(h["shape"])


def write_safetensors(path, tensors):
    """Write {name: (dtype, array)} with dtype "BF16" (uint16 bit array),
    "F16" or "F32" -- for tests and for round trips."""
    header, blobs, off = {}, [], 0
    for name, (dtype, arr) in tensors.items():
        arr = np.ascontiguousarray(arr)
        raw = arr.astype("<u2" if dtype == "BF16" else ("<f2" if dtype == "F16" else "<f4")).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


# ------------------------------------------------------------------ bf16 / quantization
def f32_to_bf16_bits(a):
    """Round to nearest even f32 -> bf16 (crates/xnpu-cli/src/main.rs:338-343)."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def quantize_group32(w):
    """w: float32 [n, k] (k a multiple of 32) -> (q int8 [n, k] in [-8, 7],
    scale bf16 bits uint16 [n, k/32])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if k % GROUP:
        raise ValueError(f"k = {k} is not a multiple of {GROUP}")
    g = w.reshape(n, k // GROUP, GROUP)
    amax = np.abs(g).max(axis=2)
    s_bits = f32_to_bf16_bits(amax / np.float32(7.0))
    s = bf16_bits_to_f32(s_bits)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(s[:, :, None] > 0, g / s[:, :, None], np.float32(0.0))
    q = np.clip(np.rint(r), -8, 7).astype(np.int8)
    return q.reshape(n, k), s_bits


def dequant_f32(q, s_bits):
    """q * scale in f32 (exact), [n, k]."""
    n, k = q.shape
    s = bf16_bits_to_f32(s_bits)
    return (q.reshape(n, k // GROUP, GROUP).astype(np.float32) * s[:, :, None]).reshape(n, k)


# ------------------------------------------------------------------ L1 tiles
def l1_bytes(n, k, tsi, cols=8):
    rows_per_col = n // cols
    return cols * (rows_per_col // tsi) * (tsi * (k // 2) + tsi * (k // GROUP) * 2)


def pack_l1(q, s_bits, tsi, cols=8):
    """Signed codes [n, k] and scale bits [n, k/32] -> L1 tile bytes."""
    n, k = q.shape
    if n % cols or (n // cols) % tsi or k % GROUP:
        raise ValueError(f"{n}x{k} does not tile with cols={cols}, tsi={tsi}")
    u = (q.astype(np.int16) & 0xF).astype(np.uint8)
    nib = (u[:, 0::2] | (u[:, 1::2] << 4)).reshape(n // tsi, tsi * (k // 2))  # tiles in row order
    sc = np.ascontiguousarray(s_bits, dtype="<u2").view(np.uint8).reshape(n // tsi, tsi * (k // GROUP) * 2)
    # row order of tiles = column-major order (column c holds rows [c*n/cols, (c+1)*n/cols))
    return np.concatenate([nib, sc], axis=1).tobytes()


# ------------------------------------------------------------------ golden spot checks
def spot_rows(n, k, q, s_bits, x_bits):
    """Rows {0, 1, n/2, n-2, n-1}: f32 dot of the dequantized weights with x,
    one bf16 rounding (tools/w4_import.py:55-63)."""
    rows = sorted({0, 1, n // 2, n - 2, n - 1})
    w = dequant_f32(q[rows], s_bits[rows])
    x = bf16_bits_to_f32(x_bits)
    return rows, f32_to_bf16_bits((w @ x).astype(np.float32))


def write_golden(path, k, rows, ref_bits, x_bits):
    """u32 nrows, u32 K, rows u32[nrows], x bits u16[K], ref bits u16[nrows]
    (tools/w4_import.py:66-76)."""
    buf = struct.pack("<II", len(rows), k)
    buf += np.asarray(rows, dtype="<u4").tobytes()
    buf += np.ascontiguousarray(x_bits, dtype="<u2").tobytes()
    buf += np.ascontiguousarray(ref_bits, dtype="<u2").tobytes()
    Path(path).write_bytes(buf)


def read_golden(path):
    b = Path(path).read_bytes()
    nrows, k = struct.unpack_from("<II", b, 0)
    o = 8
    rows = np.frombuffer(b, dtype="<u4", count=nrows, offset=o)
    o += 4 * nrows
    x = np.frombuffer(b, dtype="<u2", count=k, offset=o)
    o += 2 * k
    ref = np.frombuffer(b, dtype="<u2", count=nrows, offset=o)
    return rows, x, ref


def golden_x(k):
    """The deterministic activation x[k] = (k % 7) - 3 (exact in bf16)."""
    return f32_to_bf16_bits((np.arange(k) % 7 - 3).astype(np.float32))


# ------------------------------------------------------------------ the import
def interleave_rows(a, b):
    """Rows a0, b0, a1, b1, ...: a gate/up projection whose SwiGLU a GEMV
    epilogue can apply within one 16-row block (both halves of a pair in
    neighbouring rows)."""
    if a.shape != b.shape:
        raise ValueError("gate and up differ in shape")
    out = np.empty((2 * a.shape[0], a.shape[1]), dtype=a.dtype)
    out[0::2], out[1::2] = a, b
    return out


def import_layers(model, out, layers=None, shapes=LLAMA_SHAPES, cols=8, prefix="model.layers", log=print,
                  interleave_gateup=False):
    st = SafeTensors(model)
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    if layers is None:
        idx = {int(nm.split(".")[2]) for nm in st.names() if nm.startswith(prefix + ".")}
        layers = sorted(idx)
    meta = {"group_size": GROUP, "cols": cols, "layers": list(layers), "shapes": {},
            "quantizer": "symmetric amax/7 per 32-wide group, bf16 scale (RNE), q = rint(w/s) in [-8, 7]",
            "gateup_rows": "interleaved (gate_i, up_i)" if interleave_gateup else "gate then up"}
    total = 0
    for li, n_layer in enumerate(layers):
        for shape, (parts, tsi) in shapes.items():
            mats = [st.get_f32(f"{prefix}.{n_layer}.{blk}.{p}.weight") for blk, p in parts]
            k = mats[0].shape[1]
            if any(m.ndim != 2 or m.shape[1] != k for m in mats):
                raise ValueError(f"layer {n_layer} {shape}: parts disagree on K")
            if interleave_gateup and shape == "gateup":
                w = interleave_rows(*mats)
            else:
                w = np.concatenate(mats, axis=0)
            n = w.shape[0]
            q, s = quantize_group32(w)
            packed = pack_l1(q, s, tsi, cols)
            (out / f"layer{n_layer:02d}_{shape}.bin").write_bytes(packed)
            total += len(packed)
            if li == 0:
                meta["shapes"][shape] = {"M": n, "K": k, "tsi": tsi, "bytes": len(packed)}
                xb = golden_x(k)
                rows, ref = spot_rows(n, k, q, s, xb)
                write_golden(out / f"golden_{shape}.bin", k, rows, ref, xb)
        log(f"layer {n_layer}: {len(shapes)} shapes written")
    (out / "meta.json").write_text(json.dumps(meta, indent=1))
    log(f"done: {len(layers)} layers, {total / 1e6:.1f} MB, golden spot checks for layer {layers[0]}")
    return meta


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", required=True, help=".safetensors file")
    ap.add_argument("--out", required=True)
    ap.add_argument("--layers", type=int, nargs="*", default=None, help="layer indices (default: all)")
    ap.add_argument("--cols", type=int, default=8)
    ap.add_argument("--interleave-gateup", action="store_true",
                    help="write gateup rows as gate_i, up_i pairs (for a chain op's fused SwiGLU)")
    args = ap.parse_args(argv)
    import_layers(args.model, args.out, args.layers, cols=args.cols, interleave_gateup=args.interleave_gateup)
    return 0


if __name__ == "__main__":
    sys.exit(main())
