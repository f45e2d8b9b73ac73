"""The CPU oracle against the reference's known answers and golden vectors.

The oracle (oracle/q4nx_oracle.c) restates the reference's host arithmetic;
these tests pin it before it is trusted as the checker of the GPU path.
"""
import json
import struct

import numpy as np
import pytest

from oracle import oracle as O
from xnpu_b200 import synth


# ---------------------------------------------------------------- bf16 helpers
def test_bf16_round_trip_and_rne():
    """f32_to_bf16 is RNE (crates/xnpu-cli/src/main.rs:338-343)."""
    assert O.f32_to_bf16(1.0) == 0x3F80
    assert O.bf16_to_f32(0x3F80) == 1.0
    # halfway cases round to even
    one_plus_half_ulp = np.array([0x3F808000], dtype=np.uint32).view(np.float32)[0]
    assert O.f32_to_bf16(float(one_plus_half_ulp)) == 0x3F80
    three_halves = np.array([0x3F818000], dtype=np.uint32).view(np.float32)[0]
    assert O.f32_to_bf16(float(three_halves)) == 0x3F82
    rng = np.random.default_rng(0)
    v = rng.standard_normal(4096).astype(np.float32) * 100
    ref = synth.f32_to_bf16_bits(v)
    got = np.array([O.f32_to_bf16(float(a)) for a in v], dtype=np.uint16)
    assert np.array_equal(ref, got)
    import torch
    tb = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ref, tb)


def test_dequant_rule_sign_extend():
    """w = RNE_bf16(sext4(nib) * s) for every nibble (main.rs:3117-3121)."""
    s = O.f32_to_bf16(0.013)
    for q in range(-8, 8):
        w = O.dequant_one(q, s)
        assert w == O.f32_to_bf16(q * O.bf16_to_f32(s))


# ---------------------------------------------------------------- KAT
@pytest.mark.parametrize("n,k", [(2048, 2048), (256, 4096), (128, 14336)])
def test_kat_matches_exact_answer(golden_dir, n, k):
    """The oracle's restatement of run-w4gemv's host reference equals the
    exactly-computed KAT answer bit for bit (main.rs:2164-2299)."""
    raw = (golden_dir / f"kat_{n}x{k}.bin").read_bytes()
    hn, hk = struct.unpack_from("<II", raw)
    assert (hn, hk) == (n, k)
    expect = np.frombuffer(raw, dtype="<u2", offset=8)
    assert np.array_equal(O.kat_ref(n, k), expect)
    # the general GEMV path over the KAT planes gives the same bits
    q, s, x = O.kat_fill(n, k)
    w = O.dequant_planes(q, s)
    y = O.gemv_bf16(w, x[None, :])
    assert np.array_equal(O.round_bf16(y)[0], expect)


def test_kat_through_l1_pack(golden_dir):
    """KAT data through the reference's L1 layout (tsi=1, 4 columns: the
    run-w4gemv default fixture geometry, main.rs:319-321)."""
    n = k = 2048
    q, s, x = O.kat_fill(n, k)
    pack = O.l1_pack(q, s, tsi=1, cols=4)
    assert pack.size == O.l1_size(n, k, tsi=1, cols=4) == n * (k // 2 + k // 32 * 2)
    y = O.gemv_l1(pack, n, k, 1, x[None, :], cols=4)
    expect = np.frombuffer((golden_dir / "kat_2048x2048.bin").read_bytes(), dtype="<u2", offset=8)
    assert np.array_equal(O.round_bf16(y)[0], expect)


# ---------------------------------------------------------------- layouts
def _small_planes(golden_dir):
    man = json.loads((golden_dir / "manifest.json").read_text())["layouts"]
    m, k, seed = man["m"], man["k"], man["seed"]
    q = synth.unpack_codes_signed(synth.synth_codes(m, k, seed))
    s = synth.synth_scales(m, k, seed)
    return m, k, q, s, man


def test_l1_pack_matches_fixture(golden_dir):
    """C L1 packer == the Python transliteration that wrote l1_small.bin."""
    m, k, q, s, man = _small_planes(golden_dir)
    pack = O.l1_pack(q, s, tsi=man["l1"]["tsi"], cols=man["l1"]["cols"])
    assert pack.tobytes() == (golden_dir / "l1_small.bin").read_bytes()
    q2, s2 = O.l1_unpack(pack, m, k, man["l1"]["tsi"], man["l1"]["cols"])
    assert np.array_equal(q2, q) and np.array_equal(s2, s)


def test_l2_pack_matches_fixture(golden_dir):
    m, k, q, s, _ = _small_planes(golden_dir)
    pack = O.l2_pack(q, s)
    assert pack.tobytes() == (golden_dir / "l2_small.bin").read_bytes()
    w = O.l2_dequant(pack, m, k)
    assert np.array_equal(w, O.dequant_planes(q, s))


def test_l2_general_reader_agrees_with_reference_row_reader():
    """For K=2048 (where the reference's w4u_row_bf16 is defined) the
    chunk-aware reader equals the literal restatement row by row."""
    m, k = 256, 2048
    q = synth.unpack_codes_signed(synth.synth_codes(m, k, 5))
    s = synth.synth_scales(m, k, 5)
    pack = O.l2_pack(q, s)
    w = O.l2_dequant(pack, m, k)
    for row in (0, 1, 15, 16, 31, 32, 127, 128, 200, 255):
        assert np.array_equal(O.l2_row_ref(pack, m, k, row), w[row])


def test_gemv_same_over_every_layout():
    """The reference's GEMV (w = q*s unrounded, main.rs:2287-2296) gives the
    same bits over q/s planes, the L1 pack and the L2 pack, and differs from
    the bf16-weight form only by the weights' rounding."""
    m, k = 128, 4096
    q = synth.unpack_codes_signed(synth.synth_codes(m, k, 31))
    s = synth.synth_scales(m, k, 31)
    x = synth.synth_x(3, k, 31)
    yq = O.gemv_q(q, s, x)
    assert np.array_equal(yq, O.gemv_l1(O.l1_pack(q, s, tsi=16), m, k, 16, x))
    assert np.array_equal(yq, O.gemv_l2(O.l2_pack(q, s), m, k, x))
    yb = O.gemv_bf16(O.dequant_planes(q, s), x)
    assert np.abs(yq - yb).max() < 1e-2 * np.abs(yq).max()
    # one thread or eight: same bits (rows are independent)
    assert np.array_equal(yq, O.gemv_q(q, s, x, nthreads=1))


def test_l1_dequant_equals_planes():
    m, k = 128, 6144
    q = synth.unpack_codes_signed(synth.synth_codes(m, k, 9))
    s = synth.synth_scales(m, k, 9)
    for tsi in (4, 16):
        pack = O.l1_pack(q, s, tsi=tsi)
        assert np.array_equal(O.l1_dequant(pack, m, k, tsi), O.dequant_planes(q, s))


def test_layout_size_formulas():
    """Size checks of the reference: L1 main.rs:2597, L2 8*blocks*ELEM (:3930)."""
    for (m, k, tsi) in [(2560, 2048, 16), (2048, 2048, 16), (12288, 2048, 16), (2048, 6144, 4)]:
        expect = 8 * (m // 8) * (tsi * (k // 2) + tsi * (k // 32) * 2) // tsi
        assert O.l1_size(m, k, tsi) == expect
    assert O.l2_size(121088, 2048) == 8 * (121088 // 8 // 16) * 18560
    assert O.l2_size(2048, 6144) == 8 * (2048 // 8 // 16) * 3 * 18560


# ---------------------------------------------------------------- goldens
def _read_golden(path):
    raw = path.read_bytes()
    nrows, k = struct.unpack_from("<II", raw)
    assert len(raw) == 8 + 4 * nrows + 2 * k + 2 * nrows  # main.rs:2475
    rows = np.frombuffer(raw, dtype="<u4", count=nrows, offset=8)
    x = np.frombuffer(raw, dtype="<u2", count=k, offset=8 + 4 * nrows)
    ref = np.frombuffer(raw, dtype="<u2", count=nrows, offset=8 + 4 * nrows + 2 * k)
    return rows, x, ref


def golden_cases(golden_dir):
    man = json.loads((golden_dir / "manifest.json").read_text())["golden"]
    return sorted(man.items())


def test_oracle_matches_reference_goldens(golden_dir):
    """Goldens written by the reference's spot_rows/write_golden; the oracle's
    sequential-f32 GEMV over the L1 pack matches within the reference's own
    tolerance |g - w| <= 0.01 + 0.01|w| (main.rs:2705-2714)."""
    for name, meta in golden_cases(golden_dir):
        rows, x, ref = _read_golden(golden_dir / f"golden_{name}.bin")
        assert list(rows) == meta["rows"]
        m, k, tsi, seed = meta["m"], meta["k"], meta["tsi"], meta["seed"]
        assert np.array_equal(x, synth.f32_to_bf16_bits((np.arange(k) % 7 - 3).astype(np.float32)))
        q = synth.unpack_codes_signed(synth.synth_codes(m, k, seed))
        s = synth.synth_scales(m, k, seed)
        pack = O.l1_pack(q, s, tsi=tsi)
        got = np.zeros(len(rows), dtype=np.float32)
        w = O.l1_dequant(pack, m, k, tsi)
        y = O.gemv_bf16(w[rows], x[None, :])[0]
        got = synth.bf16_bits_to_f32(O.round_bf16(y))
        want = synth.bf16_bits_to_f32(ref)
        err = np.abs(got - want)
        assert np.all(err <= 0.01 + 0.01 * np.abs(want)), (name, err.max())
        # and it is the same value up to one bf16 rounding step
        assert np.all(np.abs(got.view(np.int32) - want.view(np.int32)) <= 1 << 16), name


# ---------------------------------------------------------------- W4A8 quantizer
def test_quantize_x_semantics():
    """Per-group-32 int8 quantizer (main.rs:2955-2986): d = bf16(amax/127),
    q = clamp(rne(x/d)), zero group -> q=0, d=0."""
    rng = np.random.default_rng(3)
    x = synth.f32_to_bf16_bits(rng.standard_normal(4096).astype(np.float32))
    x[64:96] = 0  # an all-zero group
    q, d = O.quantize_x(x)
    xf = synth.bf16_bits_to_f32(x).reshape(-1, 32)
    amax = np.abs(xf).max(axis=1)
    d_ref = np.where(amax > 0, synth.f32_to_bf16_bits((amax / np.float32(127.0)).astype(np.float32)), 0)
    assert np.array_equal(d, d_ref.astype(np.uint16))
    df = synth.bf16_bits_to_f32(d)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(df[:, None] > 0, np.rint(xf / df[:, None]), 0)
    assert np.array_equal(q.reshape(-1, 32), np.clip(r, -127, 127).astype(np.int8))
    assert np.all(q[64:96] == 0) and d[2] == 0


def test_chunk_partial_sum_rule():
    """K=6144 read-back: f32 sum of bf16 chunk partials, one RNE (main.rs:3080-3086)."""
    parts = synth.f32_to_bf16_bits(np.array([[1.0, 2.5], [0.00390625, -2.5], [1.0, 0.0]], dtype=np.float32))
    out = synth.bf16_bits_to_f32(O.sum_chunk_partials(parts))
    # 1 + 2^-8 + 1 = 2.00390625 in f32; 2^-8 is below half a bf16 ulp at 2
    assert out.tolist() == [2.0, 0.0]


def _bf(v):
    """f32 values -> bf16 bits (RNE), independent of the oracle."""
    b = np.asarray(v, dtype=np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def _f(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_glue_restatements():
    """rms_norm_bf16 / add_bf16 / swiglu_bf16 (crates/xnpu-cli/src/main.rs:
    4714-4745) against a direct numpy transcription with the reference's
    operation order: a sequential f32 sum of squares, (x * inv) * w, one
    RNE per output."""
    rng = np.random.default_rng(7)
    k = 512
    x = _bf(rng.normal(0, 2, size=(3, k)))
    w = _bf(rng.normal(1, 0.1, size=k))
    got = O.rms_norm(x, w, eps=1e-5)
    for t in range(3):
        s = np.float32(0)
        for v in _f(x[t]):
            s = np.float32(s + np.float32(v * v))
        inv = np.float32(1) / np.sqrt(np.float32(s / np.float32(k) + np.float32(1e-5)))
        want = _bf((_f(x[t]) * inv).astype(np.float32) * _f(w))
        assert np.array_equal(got[t], want), t
    a, b = _bf(rng.normal(size=1000)), _bf(rng.normal(size=1000))
    assert np.array_equal(O.add_bf16(a, b), _bf(_f(a) + _f(b)))
    gu = _bf(rng.normal(0, 3, size=(2, 64)))
    g, u = _f(gu[:, :32]), _f(gu[:, 32:])
    sig = (np.float32(1) / (np.float32(1) + np.exp(-g).astype(np.float32))).astype(np.float32)
    want = _bf((g * sig).astype(np.float32) * u)
    d = np.abs(O.swiglu(gu).astype(np.int32) - want.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() < 0.05  # numpy's exp and libm's may differ in the last f32 bit


def test_rope_and_qk_norm_restatements():
    """rope_table / rope_apply / qk_rms_bf16 (main.rs:4817-4857)."""
    c, s = O.rope_table(0)
    assert np.all(c == 1) and np.all(s == 0)
    rng = np.random.default_rng(11)
    x = _bf(rng.normal(0, 2, size=4 * 128))
    assert np.array_equal(O.rope_apply(x, c, s), x)  # position 0: identity
    pos, base = 37, 10000.0
    c, s = O.rope_table(pos, base)
    j = np.arange(64, dtype=np.float64)
    a = pos * base ** (-j / 64)
    assert np.allclose(c, np.cos(a), rtol=0, atol=2e-6) and np.allclose(s, np.sin(a), rtol=0, atol=2e-6)
    got = O.rope_apply(x, c, s).reshape(4, 128)
    xf = _f(x).reshape(4, 128)
    x1, x2 = xf[:, :64], xf[:, 64:]
    want = np.concatenate([_bf((x1 * c).astype(np.float32) - (x2 * s).astype(np.float32)),
                           _bf((x2 * c).astype(np.float32) + (x1 * s).astype(np.float32))], axis=1)
    assert np.array_equal(got, want)
    w = _bf(rng.normal(1, 0.1, size=128))
    got = O.qk_rms(x, w).reshape(4, 128)
    for h in range(4):
        acc = np.float32(0)
        for v in xf[h]:
            acc = np.float32(acc + np.float32(v * v))
        inv = np.float32(1) / np.sqrt(np.float32(acc / np.float32(128) + np.float32(1e-5)))
        assert np.array_equal(got[h], _bf((xf[h] * inv).astype(np.float32) * _f(w))), h


def test_attention_restatement():
    """attention_bf16 (main.rs:4967-5033): one position returns its V row;
    a longer context agrees with a float64 softmax to the bf16 grain."""
    rng = np.random.default_rng(12)
    heads, nkv, seq = 8, 2, 40
    q = _bf(rng.normal(size=heads * 128))
    kc = _bf(rng.normal(size=(nkv, seq, 128)))
    vc = _bf(rng.normal(size=(nkv, seq, 128)))
    out0 = O.attention(q, kc, vc, 0, seq, heads, nkv).reshape(heads, 128)
    for h in range(heads):
        assert np.array_equal(out0[h], vc[h // (heads // nkv), 0]), h
    pos = 29
    out = _f(O.attention(q, kc, vc, pos, seq, heads, nkv)).reshape(heads, 128).astype(np.float64)
    qf, kf, vf = _f(q).reshape(heads, 128), _f(kc), _f(vc)
    for h in range(heads):
        kv = h // (heads // nkv)
        sc = kf[kv, :pos + 1].astype(np.float64) @ qf[h].astype(np.float64) / np.sqrt(128.0)
        p = np.exp(sc - sc.max())
        ref = (p / p.sum()) @ vf[kv, :pos + 1].astype(np.float64)
        assert np.all(np.abs(out[h] - ref) <= 2.0 ** -7 * np.abs(ref) + 1e-6), h
