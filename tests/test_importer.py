"""The offline w4 importer (xnpu_b200/importer.py).

CPU: the quantizer rule, the L1 packer against the oracle's packer
(crates/xnpu-cli/src/main.rs:2231-2252) byte for byte, and a synthetic
two-layer safetensors model imported end to end (files, sizes, the codes and
scales read back by the oracle's L1 unpacker, golden spot checks against the
oracle's GEMV over the packed tiles).  GPU: the written .bin imported through
xq4_weight_import (L1) and run by the GEMV, checked against the golden rows
at the reference's tier |g - w| <= 0.01 + 0.01 |w| (main.rs:2705-2714).
"""
import json

import numpy as np
import pytest

from oracle import oracle as O
from xnpu_b200 import importer as I


def _rng(seed):
    return np.random.default_rng(seed)


def test_quantize_rule():
    w = _rng(1).normal(0, 0.05, size=(64, 256)).astype(np.float32)
    w[3, 32:64] = 0.0  # an all-zero group
    q, s = I.quantize_group32(w)
    assert q.dtype == np.int8 and q.min() >= -8 and q.max() <= 7
    amax = np.abs(w.reshape(64, 8, 32)).max(axis=2)
    assert np.array_equal(s, I.f32_to_bf16_bits(amax / np.float32(7)))
    assert s[3, 1] == 0 and not q[3, 32:64].any()
    sf = I.bf16_bits_to_f32(s)
    err = np.abs(I.dequant_f32(q, s) - w).reshape(64, 8, 32)
    assert (err <= sf[:, :, None] * 0.5 + 1e-12).all()  # round to nearest, nothing clipped


def test_f32_to_bf16_matches_oracle():
    a = _rng(2).normal(0, 3, size=4096).astype(np.float32)
    a[:4] = [0.0, -0.0, 1.00390625, 1.01171875]  # exact ties round to even
    want = np.array([O.f32_to_bf16(float(v)) for v in a], dtype=np.uint16)
    assert np.array_equal(I.f32_to_bf16_bits(a), want)


@pytest.mark.parametrize("n,k,tsi", [(128, 256, 16), (64, 512, 4), (384, 96, 16)])
def test_pack_l1_matches_oracle(n, k, tsi):
    rng = _rng(n + k)
    q = rng.integers(-8, 8, size=(n, k)).astype(np.int8)
    s = rng.integers(0, 1 << 15, size=(n, k // 32)).astype(np.uint16)
    got = I.pack_l1(q, s, tsi)
    assert len(got) == I.l1_bytes(n, k, tsi) == O.l1_size(n, k, tsi)
    assert got == O.l1_pack(q, s, tsi).tobytes()


def _tiny_model(path, layers=2, hidden=256, kv=64, inter=512, seed=3):
    rng = _rng(seed)
    t = {}
    for n in range(layers):
        def put(name, rows, cols):
            w = rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)
            t[f"model.layers.{n}.{name}.weight"] = ("BF16", I.f32_to_bf16_bits(w))
        put("self_attn.q_proj", hidden, hidden)
        put("self_attn.k_proj", kv, hidden)
        put("self_attn.v_proj", kv, hidden)
        put("self_attn.o_proj", hidden, hidden)
        put("mlp.gate_proj", inter, hidden)
        put("mlp.up_proj", inter, hidden)
        put("mlp.down_proj", hidden, inter)
    t["model.embed_tokens.weight"] = ("F32", rng.normal(size=(16, hidden)).astype(np.float32))
    I.write_safetensors(path, t)
    return t


def test_import_end_to_end(tmp_path):
    model = tmp_path / "tiny.safetensors"
    tensors = _tiny_model(model)
    out = tmp_path / "w4"
    meta = I.import_layers(model, out, log=lambda *_: None)
    assert meta["layers"] == [0, 1]
    assert json.loads((out / "meta.json").read_text())["shapes"]["qkv"]["M"] == 384
    for layer in (0, 1):
        for shape, (parts, tsi) in I.LLAMA_SHAPES.items():
            mats = [I.bf16_bits_to_f32(tensors[f"model.layers.{layer}.{b}.{p}.weight"][1]) for b, p in parts]
            w = np.concatenate(mats, axis=0)
            n, k = w.shape
            blob = np.fromfile(out / f"layer{layer:02d}_{shape}.bin", dtype=np.uint8)
            assert blob.size == O.l1_size(n, k, tsi)
            q, s = O.l1_unpack(blob, n, k, tsi)
            q_ref, s_ref = I.quantize_group32(w)
            assert np.array_equal(q, q_ref) and np.array_equal(s, s_ref), (layer, shape)
            if layer == 0:
                rows, x, ref = I.read_golden(out / f"golden_{shape}.bin")
                assert list(rows) == sorted({0, 1, n // 2, n - 2, n - 1})
                assert np.array_equal(x, I.golden_x(k))
                y = O.gemv_l1(blob, n, k, tsi, x.reshape(1, k))[0]
                g = I.bf16_bits_to_f32(ref)
                assert (np.abs(g - y[rows]) <= 0.01 + 0.01 * np.abs(y[rows])).all(), shape


def test_import_interleaved_gateup(tmp_path):
    model = tmp_path / "tiny.safetensors"
    tensors = _tiny_model(model, layers=1)
    out = tmp_path / "w4"
    meta = I.import_layers(model, out, log=lambda *_: None, interleave_gateup=True)
    assert meta["gateup_rows"].startswith("interleaved")
    g = I.bf16_bits_to_f32(tensors["model.layers.0.mlp.gate_proj.weight"][1])
    u = I.bf16_bits_to_f32(tensors["model.layers.0.mlp.up_proj.weight"][1])
    n, k = 2 * g.shape[0], g.shape[1]
    q, s = O.l1_unpack(np.fromfile(out / "layer00_gateup.bin", dtype=np.uint8), n, k, 16)
    qg, sg = I.quantize_group32(g)
    qu, su = I.quantize_group32(u)
    assert np.array_equal(q[0::2], qg) and np.array_equal(q[1::2], qu)
    assert np.array_equal(s[0::2], sg) and np.array_equal(s[1::2], su)


def test_safetensors_reader_dtypes(tmp_path):
    a = _rng(4).normal(size=(3, 5)).astype(np.float32)
    path = tmp_path / "d.safetensors"
    I.write_safetensors(path, {"f32": ("F32", a), "f16": ("F16", a.astype(np.float16)),
                               "bf16": ("BF16", I.f32_to_bf16_bits(a))})
    st = I.SafeTensors(path)
    assert np.array_equal(st.get_f32("f32"), a)
    assert np.array_equal(st.get_f32("f16"), a.astype(np.float16).astype(np.float32))
    assert np.array_equal(st.get_f32("bf16"), I.bf16_bits_to_f32(I.f32_to_bf16_bits(a)))


@pytest.mark.gpu
def test_imported_l1_on_gpu(dev, tmp_path):
    """The importer's .bin through xq4_weight_import (L1) and the GEMV, at
    the golden rows' tier and the GEMV parity bars against the oracle."""
    import torch
    from xnpu_b200 import hal
    from test_gpu_kernels import assert_parity, from_dev_bf16, to_dev_u16
    model = tmp_path / "tiny.safetensors"
    _tiny_model(model, layers=1, hidden=512, kv=128, inter=1024, seed=5)
    out = tmp_path / "w4"
    meta = I.import_layers(model, out, log=lambda *_: None)
    for shape, info in meta["shapes"].items():
        n, k, tsi = info["M"], info["K"], info["tsi"]
        blob = (out / f"layer00_{shape}.bin").read_bytes()
        w = hal.Weight.import_(dev, blob, hal.layout_desc(hal.XQ4_LAYOUT_L1, n, k, tsi=tsi, cols=8))
        rows, x, ref = I.read_golden(out / f"golden_{shape}.bin")
        y = from_dev_bf16(hal.linear(w, to_dev_u16(x.reshape(1, k))))[0]
        got, g = I.bf16_bits_to_f32(y[rows]), I.bf16_bits_to_f32(ref)
        assert (np.abs(got - g) <= 0.01 + 0.01 * np.abs(g)).all(), shape
        want = O.gemv_l1(np.frombuffer(blob, dtype=np.uint8), n, k, tsi, x.reshape(1, k))
        assert_parity(y.reshape(1, n), want, f"imported {shape}")
        w.destroy()
        torch.cuda.synchronize()


def test_importer_command_line(tmp_path):
    model = tmp_path / "tiny.safetensors"
    _tiny_model(model, layers=2)
    out = tmp_path / "w4"
    assert I.main(["--model", str(model), "--out", str(out), "--layers", "1", "--interleave-gateup"]) == 0
    meta = json.loads((out / "meta.json").read_text())
    assert meta["layers"] == [1] and meta["gateup_rows"].startswith("interleaved")
    assert sorted(p.name for p in out.iterdir()) == sorted(
        ["meta.json"] + [f"layer01_{s}.bin" for s in I.LLAMA_SHAPES] + [f"golden_{s}.bin" for s in I.LLAMA_SHAPES])
