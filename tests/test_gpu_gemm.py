"""GPU parity of the tcgen05 dequant-GEMM (m >= 25) through the C ABI.

The GEMM multiplies x by the dequantized weights RNE_bf16(q * s) (the
reference's dequant, main.rs:3097-3125) with f32 accumulation, so its own
oracle is the bf16-weight GEMV over the oracle's dequantized weights
(q4o_gemv_bf16); against the unrounded-weight GEMV of main.rs:2287-2296 the
outputs must lie within the bound that weight rounding allows.  Bars:
bit-exact on the KAT fixtures (exact arithmetic in any order); max relative
error <= 1e-2 with the floored denominator and mean absolute error <= 1e-3 on
seeded synthetic data (the rationale is in test_gpu_kernels.py), 5e-3 for f32
outputs; at prefill sizes a plain torch fp32 matmul of the bit-exact
dequantized weights covers every output.  xq4_linear runs the GEMM from
m = GEMM_MIN_M on; below it the GEMV (unrounded weights, the formula of
main.rs:2287-2296), whose oracle is the unrounded-weight GEMV.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from xnpu_b200 import hal, synth
from test_gpu_kernels import (MAE, MAX_REL, assert_parity, from_dev_bf16, import_planes, rel_metrics,
                              row_subset, to_dev_u16)

pytestmark = pytest.mark.gpu

GEMM_MIN_M = 25  # xq4_linear's routing (XQ4_GEMM_MIN_M in xq4_internal.h)


def oracle_for(q, s, x, rows, m):
    """The oracle of the path xq4_linear takes for m tokens."""
    if m < GEMM_MIN_M:
        return O.gemv_q(q[rows], s[rows], x)
    return O.gemv_bf16(O.dequant_planes(q[rows], s[rows]), x)


def make(n, k, seed):
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, seed))
    s = synth.synth_scales(n, k, seed)
    return q, s


@pytest.mark.parametrize("m", [16, 64, 300])
def test_gemm_kat_bit_exact(dev, golden_dir, m):
    n, k = 256, 4096
    expect = np.frombuffer((golden_dir / f"kat_{n}x{k}.bin").read_bytes(), dtype="<u2", offset=8)
    q, s, x = O.kat_fill(n, k)
    w = import_planes(dev, q, s)
    y = from_dev_bf16(hal.linear(w, to_dev_u16(np.repeat(x[None, :], m, axis=0))))
    bad = [t for t in range(m) if not np.array_equal(y[t], expect)]
    assert not bad, f"tokens {bad[:8]} differ"


@pytest.mark.parametrize("m", [16, 17, 32, 48, 64, 100, 128, 255, 256, 300])
def test_gemm_parity_batch_sweep(dev, m):
    """4096 -> 4096 projection over the batched-decode / short-prefill sizes."""
    n, k = 4096, 4096
    q, s = make(n, k, 900)
    x = synth.synth_x(m, k, 901 + m)
    w = import_planes(dev, q, s)
    y = from_dev_bf16(hal.linear(w, to_dev_u16(x)))
    rows = row_subset(n, limit=768)
    assert_parity(y[:, rows], oracle_for(q, s, x, rows, m), f"m={m}")
    # Against the unrounded-weight GEMV (main.rs:2287-2296): rounding each
    # weight to bf16 moves it by at most 2^-9 relative, so the outputs may
    # differ by 2^-9 * sum|w||x| (plus both sides' final bf16 rounding and
    # f32 summation, 2^-8 * |y| + 2^-8 * 2^-9 * sum|w||x| covers them).
    yq = O.gemv_q(q[rows], s[rows], x)
    absx = (np.asarray(x, dtype=np.uint16) & 0x7FFF).astype(np.uint16)
    bound = O.gemv_q(np.abs(q[rows]).astype(np.int8), s[rows], absx)
    got = synth.bf16_bits_to_f32(y[:, rows])
    assert np.all(np.abs(got - yq) <= 2.0 ** -9 * bound * 1.01 + 2.0 ** -8 * np.abs(yq)), f"m={m}"


@pytest.mark.parametrize("n,k,m", [(17, 96, 16), (17, 96, 25), (333, 160, 40), (4100, 4128, 33),
                                   (130, 14336, 20), (130, 14336, 28), (14336, 4096, 64), (4096, 14336, 24),
                                   (4096, 14336, 25)])
def test_gemm_parity_ragged_and_8b_shapes(dev, n, k, m):
    """Ragged features (not a multiple of the 128-feature tile), K with a
    half chunk (k % 64 == 32), ragged token counts, and the 8B-shaped
    gate/down projections."""
    q, s = make(n, k, 950 + n)
    x = synth.synth_x(m, k, 951 + n)
    w = import_planes(dev, q, s)
    y = from_dev_bf16(hal.linear(w, to_dev_u16(x)))
    rows = row_subset(n, limit=768)
    assert_parity(y[:, rows], oracle_for(q, s, x, rows, m), f"{n}x{k} m={m}")


def test_gemm_f32_output(dev):
    n, k, m = 1024, 4096, 32
    q, s = make(n, k, 960)
    x = synth.synth_x(m, k, 961)
    w = import_planes(dev, q, s)
    y = hal.linear(w, to_dev_u16(x), out_dtype=torch.float32).cpu().numpy()
    ref = O.gemv_bf16(O.dequant_planes(q, s), x)
    # the tensor cores add each K=16 step's products before the f32
    # accumulate, so the order (and last-bit rounding) differs from a
    # sequential sum: ~1e-5 of rms, at most 5e-3 of the floored denominator
    max_rel, mae, raw = rel_metrics(y, ref)
    rel_rms = np.sqrt(np.mean((y - ref) ** 2)) / np.sqrt(np.mean(ref ** 2))
    assert max_rel <= 5e-3 and mae <= 1e-5 and rel_rms < 1e-4, (max_rel, mae, raw, rel_rms)


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 2048), (14336, 4096, 512), (14336, 4096, 600)])
def test_gemm_prefill_vs_torch_fp32(dev, n, k, m):
    """Prefill sizes: every output against a torch fp32 matmul of the GPU's
    dequantized weights (bit-exact to the oracle's, tested above), and a row
    subset against the oracle itself.  14336 x 4096 at m = 600 is 336 tiles
    of 128 x 256 (the last token tile ragged): two whole waves through the
    persistent kernel (two tiles per CTA, both accumulator halves) and 40
    tiles with K split over clusters of 3, on a 148-SM B200."""
    q, s = make(n, k, 970 + m)
    x = synth.synth_x(m, k, 971 + m)
    w = import_planes(dev, q, s)
    xd = to_dev_u16(x)
    y = hal.linear(w, xd, out_dtype=torch.float32)
    wd = hal.dequant(w)
    ref = (xd.float() @ wd.float().t())
    torch.cuda.synchronize()
    err = (y - ref).abs()
    floor = 1e-2 * ref.pow(2).mean().sqrt()
    max_rel = (err / torch.maximum(ref.abs(), floor)).max().item()
    assert max_rel <= 5e-3 and err.mean().item() <= 1e-5, max_rel
    rows = np.arange(0, n, max(1, n // 96))
    yb = from_dev_bf16(hal.linear(w, xd))
    assert_parity(yb[:, rows], O.gemv_bf16(O.dequant_planes(q[rows], s[rows]), x), f"{n}x{k} m={m}")


def test_gemm_deterministic(dev):
    """Two runs of the same GEMM give the same bits."""
    n, k, m = 2048, 4096, 200
    q, s = make(n, k, 980)
    w = import_planes(dev, q, s)
    xd = to_dev_u16(synth.synth_x(m, k, 981))
    a = from_dev_bf16(hal.linear(w, xd))
    b = from_dev_bf16(hal.linear(w, xd))
    assert np.array_equal(a, b)


def test_gemm_no_fault_flag(dev):
    """No bounded wait ran out in any kernel so far."""
    n, k, m = 512, 4096, 64
    q, s = make(n, k, 990)
    w = import_planes(dev, q, s)
    hal.linear(w, to_dev_u16(synth.synth_x(m, k, 991)))
    torch.cuda.synchronize()
    assert dev.fault() == 0
