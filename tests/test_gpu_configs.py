"""GPU parity at the exact shape of every benchmark configuration of the int4
path, every output checked.

  * config 0: one decode GEMV, m = 1, 4096 -> 4096, imported from the
    reference's L1 tile layout (tools/w4_import.py:4-14);
  * config 1: one 8B-shaped layer (qkv 4096->6144, o 4096->4096, gate and up
    4096->14336, down 14336->4096) at m = 1, as one chain launch (the
    benchmark's step kernel) and as single ops;
  * config 2: the gate projection 4096 -> 14336 at m in {1, 2, 4, 8, 16, 32,
    64} through xq4_linear's routing (the decode GEMV below m = 25, the
    tcgen05 GEMM from m = 25);
  * config 3: prefill m = 2048, 4096 -> 14336: every output against a torch
    fp32 matmul of the bit-exact dequantized weights, and a row subset
    against the oracle itself;
  * config 4: lm_head 4096 -> 128256 with f32 logits, every logit against the
    oracle, plus the reference's logit gate (argmax equal, top-8 overlap,
    rel_rms < 0.05; crates/xnpu-cli/src/main.rs:4059-4097).

Dequantization is checked bit-exact on every weight of every shape.  Bars are
those of tests/parity.py; the GEMM's own oracle is the bf16-weight GEMV over
the dequantized weights, and against the unrounded-weight GEMV
(main.rs:2287-2296) it must lie within the bound that rounding each weight to
bf16 allows (as in test_gpu_gemm.py).
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_parity as assert_parity_f32, rel_metrics
from test_gpu_kernels import assert_parity, from_dev_bf16, import_planes, to_dev_u16
from xnpu_b200 import hal, synth

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 8
GEMM_MIN_M = 25  # xq4_linear's routing (XQ4_GEMM_MIN_M in xq4_internal.h)


def make(n, k, seed):
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, seed))
    s = synth.synth_scales(n, k, seed)
    return q, s


def dequant_bit_exact(w, q, s, rows_per_slice=8192):
    """Every weight of the GPU's dequant op equals the oracle's RNE_bf16(q*s),
    compared in row slices to bound host memory."""
    d = hal.dequant(w)
    n = q.shape[0]
    for r0 in range(0, n, rows_per_slice):
        r1 = min(n, r0 + rows_per_slice)
        got = d[r0:r1].cpu().view(torch.int16).numpy().view(np.uint16)
        if not np.array_equal(got, O.dequant_planes(q[r0:r1], s[r0:r1])):
            return False
    del d
    return True


def within_rounding_bound(got, q, s, x):
    """GEMM outputs (bf16-rounded weights) against the unrounded-weight GEMV:
    rounding each weight moves it by at most 2^-9 relative, so outputs may
    differ by 2^-9 * sum|w||x| plus both sides' final rounding."""
    yq = O.gemv_q(q, s, x, nthreads=THREADS)
    absx = (np.asarray(x, dtype=np.uint16) & 0x7FFF).astype(np.uint16)
    bound = O.gemv_q(np.abs(q).astype(np.int8), s, absx, nthreads=THREADS)
    return bool(np.all(np.abs(got - yq) <= 2.0 ** -9 * bound * 1.01 + 2.0 ** -8 * np.abs(yq)))


# ------------------------------------------------------------------ config 0
def test_config0_single_gemv_l1(dev):
    n, k = 4096, 4096
    q, s = make(n, k, 10)
    x = synth.synth_x(1, k, 11)
    pack = O.l1_pack(q, s, tsi=16)
    w = hal.Weight.import_(dev, pack, hal.layout_desc(hal.XQ4_LAYOUT_L1, n, k, tsi=16, cols=8))
    assert np.array_equal(from_dev_bf16(hal.dequant(w)), O.l1_dequant(pack, n, k, 16))
    y = from_dev_bf16(hal.linear(w, to_dev_u16(x)))
    # the reference's GEMV over its own L1 bytes (main.rs:2287-2296)
    assert_parity(y, O.gemv_l1(pack, n, k, 16, x, nthreads=THREADS), "config 0 4096x4096 m=1")
    # back-to-back launches give the same bits
    y2 = from_dev_bf16(hal.linear(w, to_dev_u16(x)))
    assert np.array_equal(y, y2)
    w.destroy()


# ------------------------------------------------------------------ config 1
LAYER = [("qkv", 6144, 4096), ("o", 4096, 4096), ("gate", 14336, 4096), ("up", 14336, 4096),
         ("down", 4096, 14336)]


def test_config1_layer_every_output(dev):
    ws, xs, qs, ops, ys = [], [], [], [], []
    for i, (name, n, k) in enumerate(LAYER):
        q, s = make(n, k, 20 + i)
        w = import_planes(dev, q, s)
        assert dequant_bit_exact(w, q, s), name
        x = synth.synth_x(1, k, 30 + i)
        xd = to_dev_u16(x)
        y = torch.full((1, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        ws.append(w)
        xs.append((x, xd))
        qs.append((q, s))
        ys.append(y)
        ops.append((w, xd.data_ptr(), y.data_ptr(), 1, 0, 0))
    chain = hal.Chain(dev, ops)
    chain.run()
    torch.cuda.synchronize()
    for (name, n, k), (q, s), (x, xd), y, w in zip(LAYER, qs, xs, ys, ws):
        ref = O.gemv_q(q, s, x, nthreads=THREADS)
        assert_parity(from_dev_bf16(y), ref, f"config 1 chain {name}")
        assert_parity(from_dev_bf16(hal.linear(w, xd)), ref, f"config 1 single {name}")
    assert dev.fault() == 0
    chain.destroy()
    for w in ws:
        w.destroy()


# ------------------------------------------------------------------ config 2
@pytest.fixture(scope="module")
def gate(dev):
    n, k = 14336, 4096
    q, s = make(n, k, 40)
    w = import_planes(dev, q, s)
    assert dequant_bit_exact(w, q, s)
    yield q, s, w
    w.destroy()


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16, 32, 64])
def test_config2_gate_batch_sweep(dev, gate, m):
    q, s, w = gate
    x = synth.synth_x(m, 4096, 41 + m)
    y = from_dev_bf16(hal.linear(w, to_dev_u16(x)))
    if m < GEMM_MIN_M:
        ref = O.gemv_q(q, s, x, nthreads=THREADS)
    else:
        ref = O.gemv_bf16(O.dequant_planes(q, s), x, nthreads=THREADS)
        assert within_rounding_bound(synth.bf16_bits_to_f32(y), q, s, x), f"m={m}"
    assert_parity(y, ref, f"config 2 gate m={m}")
    assert dev.fault() == 0


# ------------------------------------------------------------------ config 3
def test_config3_prefill_2048x4096x14336(dev, gate):
    q, s, w = gate
    m, n = 2048, q.shape[0]
    x = synth.synth_x(m, 4096, 50)
    xd = to_dev_u16(x)
    y = hal.linear(w, xd, out_dtype=torch.float32)
    ref = xd.float() @ hal.dequant(w).float().t()  # fp32 matmul of the bit-exact weights
    torch.cuda.synchronize()
    got, want = y.cpu().numpy(), ref.cpu().numpy()
    # f32 outputs: the tensor cores add each K=16 step's products before the
    # f32 accumulate, so the order (and last-bit rounding) differs from a
    # sequential sum; the bars of the f32 GEMM test (5e-3 floored)
    max_rel, mae, raw = rel_metrics(got, want, "config 3 f32 vs torch fp32")
    assert max_rel <= 5e-3 and mae <= 1e-5, (max_rel, mae, raw)
    yb = from_dev_bf16(hal.linear(w, xd))
    rows = np.arange(0, n, 97)
    assert_parity(yb[:, rows], O.gemv_bf16(O.dequant_planes(q[rows], s[rows]), x, nthreads=THREADS),
                  "config 3 bf16 vs oracle (row subset)")
    assert within_rounding_bound(synth.bf16_bits_to_f32(yb[:, rows]), q[rows], s[rows], x)
    assert dev.fault() == 0


# ------------------------------------------------------------------ config 4
def test_config4_lm_head_logits(dev):
    n, k = 128256, 4096
    q, s = make(n, k, 60)
    w = import_planes(dev, q, s)
    assert dequant_bit_exact(w, q, s)
    x = synth.synth_x(1, k, 61)
    y = hal.linear(w, to_dev_u16(x), out_dtype=torch.float32).cpu().numpy()
    ref = O.gemv_q(q, s, x, nthreads=THREADS)
    assert_parity_f32(y, ref, "config 4 lm_head f32 logits")
    # the reference's logit gate (main.rs:4059-4097)
    assert int(np.argmax(y[0])) == int(np.argmax(ref[0]))
    top = len(set(np.argsort(-y[0])[:8].tolist()) & set(np.argsort(-ref[0])[:8].tolist()))
    assert top == 8, top
    rel_rms = float(np.sqrt(np.mean((y - ref) ** 2)) / max(np.sqrt(np.mean(ref ** 2)), 1e-9))
    assert rel_rms < 0.05, rel_rms
    assert dev.fault() == 0
    w.destroy()
