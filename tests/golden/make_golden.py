"""Generate the committed golden fixtures for the int4 path.

Usage: python tests/golden/make_golden.py <reference source tree>

Run where the reference source is mounted, giving its root as the one
required argument; the fixtures it writes are committed and the tests never
read the reference at run time.

1. golden_<shape>.bin -- produced by the REFERENCE'S OWN functions
   ``spot_rows`` and ``write_golden`` (tools/w4_import.py:55-76), taken out of
   the reference source with ``ast`` and executed here (the module itself
   cannot be imported: at import time it loads an external packer that the
   reference does not ship).  Their input ``w_dequant`` is RNE_bf16(q * s) of
   seeded synthetic codes/scales (torch arithmetic, independent of the C
   oracle).  The file format is the reference's: u32 nrows, u32 K,
   rows u32[nrows], x bits u16[K], ref bits u16[nrows].  Shapes are the
   reference's SHAPES table (tools/w4_import.py:47-52, read from the source)
   plus the 8B-shaped projections of the decode benchmark.
2. kat_<n>x<k>.bin -- the bit-exact known-answer test of run-w4gemv
   (crates/xnpu-cli/src/main.rs:2164-2299): nibble ((13i+7k)%16)-8, scale
   ((g%4)+1)/16, x (k%7)-3.  The expected output is computed with exact
   rational arithmetic (fractions.Fraction), so it does not depend on any
   floating-point implementation: u32 n, u32 K, ref bits u16[n].
3. l1_small.bin / l2_small.bin -- reference layouts of a small seeded matrix,
   written by pure-Python transliterations of the reference packers
   (main.rs:2231-2252 for L1; the L2 geometry of main.rs:2912-2949 /
   :3097-3125), independent of the C oracle, with their q/s planes.
4. manifest.json -- seeds and shapes of every fixture.
"""
import ast
import json
import struct
import sys
from fractions import Fraction
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = None  # the reference source tree, the required command-line argument
sys.path.insert(0, str(HERE.parent.parent))
from xnpu_b200 import synth  # noqa: E402


def load_reference_functions():
    """Exec only the needed defs/assignments of tools/w4_import.py."""
    src = (REF / "tools" / "w4_import.py").read_text()
    tree = ast.parse(src)
    keep = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in ("spot_rows", "write_golden"):
            keep.append(node)
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "SHAPES" for t in node.targets):
            keep.append(node)
    mod = ast.Module(body=keep, type_ignores=[])
    ns = {"np": np, "torch": torch}
    exec(compile(mod, str(REF / "tools" / "w4_import.py"), "exec"), ns)
    return ns["spot_rows"], ns["write_golden"], ns["SHAPES"]


def q_and_s(n, k, seed):
    codes = synth.synth_codes(n, k, seed)
    scales = synth.synth_scales(n, k, seed)
    return synth.unpack_codes_signed(codes), scales


def w_dequant_torch(q, s):
    qt = torch.from_numpy(q.astype(np.float32))
    st = torch.from_numpy(s.astype(np.int32) << 16).view(torch.float32)
    prod = qt * st.repeat_interleave(32, dim=1)
    return prod.to(torch.bfloat16)  # torch's f32 -> bf16 cast rounds RNE


def kat_expected(n, k, group=32):
    """Exact sums: sum_k nib*(g%4+1)*x / 16 as an integer numerator (int64),
    then one exact conversion (checked with Fraction) and one RNE to bf16."""
    i = np.arange(n, dtype=np.int64)[:, None]
    kk = np.arange(k, dtype=np.int64)[None, :]
    nib = (13 * i + 7 * kk) % 16 - 8
    num = (nib * ((kk // group) % 4 + 1) * ((kk % 7) - 3)).sum(axis=1)
    out = np.empty(n, dtype=np.uint16)
    for r in range(n):
        acc = Fraction(int(num[r]), 16)
        f = np.float32(float(acc))
        assert Fraction(float(f)) == acc, "KAT value not exact in f32"
        out[r] = synth.f32_to_bf16_bits(np.array([f], dtype=np.float32))[0]
    return out


def l1_pack_py(q, s, tsi, cols):
    """Transliteration of the L1 packer, crates/xnpu-cli/src/main.rs:2231-2252."""
    m, k = q.shape
    group = 32
    tile_bytes = tsi * (k // 2) + tsi * (k // group) * 2
    out = bytearray(cols * (m // cols // tsi) * tile_bytes)
    rows_per_col = m // cols
    nibble_bytes = tsi * k // 2
    for i in range(m):
        col, r = divmod(i, rows_per_col)
        off = (col * (rows_per_col // tsi) + r // tsi) * tile_bytes
        rr = r % tsi
        for p in range(k // 2):
            out[off + rr * (k // 2) + p] = (int(q[i, 2 * p]) & 0xF) | ((int(q[i, 2 * p + 1]) & 0xF) << 4)
        for g in range(k // group):
            o = off + nibble_bytes + (rr * (k // group) + g) * 2
            out[o:o + 2] = struct.pack("<H", int(s[i, g]))
    return bytes(out)


def l2_pack_py(q, s):
    """L2 blocks: (col, tile, chunk) at ((col*chunks + c)*t_num + t)*18560;
    nibble (g, kk, r) at g*256 + kk*8 + r//2 (even r low); scale at
    16384 + (g*16 + r)*2; K and chunk words at ELEM-8 / ELEM-4."""
    m, k = q.shape
    elem, chunks, t_num, rpc = 18560, k // 2048, m // 8 // 16, m // 8
    out = bytearray(8 * t_num * chunks * elem)
    for row in range(m):
        col, within = divmod(row, rpc)
        t, r = divmod(within, 16)
        for c in range(chunks):
            off = ((col * chunks + c) * t_num + t) * elem
            for g in range(64):
                for kk in range(32):
                    nib = int(q[row, c * 2048 + g * 32 + kk]) & 0xF
                    bo = off + g * 256 + kk * 8 + r // 2
                    out[bo] = (out[bo] & 0xF0) | nib if r % 2 == 0 else (out[bo] & 0x0F) | (nib << 4)
                so = off + 16384 + (g * 16 + r) * 2
                out[so:so + 2] = struct.pack("<H", int(s[row, c * 64 + g]))
            out[off + elem - 8:off + elem] = struct.pack("<II", k, c)
    return bytes(out)


def main():
    global REF
    if len(sys.argv) != 2 or not (Path(sys.argv[1]) / "tools" / "w4_import.py").is_file():
        sys.exit("usage: make_golden.py <reference source tree (holding tools/w4_import.py)>")
    REF = Path(sys.argv[1])
    spot_rows, write_golden, shapes = load_reference_functions()
    manifest = {"golden": {}, "kat": {}, "layouts": {}}
    golden_shapes = {name: (m, k, tsi) for name, (_parts, m, k, tsi) in shapes.items()}
    golden_shapes.update({
        "b8_qkv": (6144, 4096, 16), "b8_o": (4096, 4096, 16), "b8_gate": (14336, 4096, 16),
        "b8_down": (4096, 14336, 4),
    })
    for i, (name, (m, k, tsi)) in enumerate(sorted(golden_shapes.items())):
        seed = 1000 + i
        q, s = q_and_s(m, k, seed)
        w = w_dequant_torch(q, s)
        x = (torch.arange(k) % 7 - 3).to(torch.bfloat16)  # tools/w4_import.py:93-95
        rows, ref = spot_rows(m, k, w, x)
        write_golden(HERE, name, k, rows, ref, x.view(torch.uint16).numpy())
        manifest["golden"][name] = {"m": m, "k": k, "tsi": tsi, "seed": seed, "rows": rows}
        print(f"golden_{name}.bin rows {rows}")
    for n, k in [(2048, 2048), (256, 4096), (128, 14336)]:
        ref = kat_expected(n, k)
        (HERE / f"kat_{n}x{k}.bin").write_bytes(struct.pack("<II", n, k) + ref.astype("<u2").tobytes())
        manifest["kat"][f"{n}x{k}"] = {"n": n, "k": k}
        print(f"kat_{n}x{k}.bin")
    # small reference-layout images (and their planes) for layout tests
    m, k, seed = 128, 4096, 77
    q, s = q_and_s(m, k, seed)
    (HERE / "l1_small.bin").write_bytes(l1_pack_py(q, s, tsi=16, cols=8))
    (HERE / "l2_small.bin").write_bytes(l2_pack_py(q, s))
    manifest["layouts"] = {"m": m, "k": k, "seed": seed, "l1": {"tsi": 16, "cols": 8}}
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("manifest.json")


if __name__ == "__main__":
    main()
