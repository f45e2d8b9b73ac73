"""W4A8 parity mode on the GPU: the reference's NPU numerics.

* quantize: bit-exact q and d against the oracle's restatement of
  w4u_quantize_x (crates/xnpu-cli/src/main.rs:2955-2986), on normal data and
  on the edge groups (all zero, one huge value, subnormal-sized values,
  negative zeros).
* GEMV: against the oracle's W4A8 restatement (exact int32 group dots, f32
  scale products, bf16 per 2048-K chunk partial, f32 sum of partials,
  main.rs:2912-2916, :3066-3091): the group dots are exact on both sides and
  only the f32 summation order inside a chunk differs, so an output may move
  by one bf16 ulp of each chunk partial (the bound is computed from the
  oracle's partials), MAE <= 1e-3, and at least 90 % of the outputs must
  match bit for bit.
* Against the bf16-activation reference (the reference's own golden check
  of its W4A8 device output, main.rs:2705-2714): |g - w| <= 0.01 + 0.01|w|.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from xnpu_b200 import hal, synth
from test_gpu_kernels import from_dev_bf16, import_planes, rel_metrics, to_dev_u16

pytestmark = pytest.mark.gpu


def quantize_ref(x):
    qs, ds = zip(*(O.quantize_x(x[t]) for t in range(x.shape[0])))
    return np.stack(qs), np.stack(ds)


@pytest.mark.parametrize("m,k", [(1, 4096), (3, 14336), (8, 2048), (2, 160)])
def test_quantize_bit_exact(dev, m, k):
    rng = np.random.default_rng(500 + m)
    xf = rng.standard_normal((m, k)).astype(np.float32)
    xf[0, :32] = 0.0                       # all-zero group
    xf[0, 32:64] = -0.0                    # negative zeros
    if k >= 128:
        xf[0, 64] = 3.0e38                 # one huge value in a group
        xf[0, 96:128] *= 1e-38             # tiny magnitudes
    x = synth.f32_to_bf16_bits(xf)
    q, d = hal.quantize_x(to_dev_u16(x))
    qr, dr = quantize_ref(x)
    assert np.array_equal(q.cpu().numpy(), qr)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), dr)


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 1), (14336, 4096, 3), (4096, 14336, 8), (333, 160, 2),
                                   (2048, 6144, 11)])
def test_w4a8_parity(dev, n, k, m):
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, 510 + n))
    s = synth.synth_scales(n, k, 510 + n)
    x = synth.synth_x(m, k, 511 + m)
    w = import_planes(dev, q, s)
    qx, dx = hal.quantize_x(to_dev_u16(x))
    y = from_dev_bf16(hal.linear_w4a8(w, qx, dx))
    qxr, dxr = quantize_ref(x)
    ref = O.gemv_w4a8(q, s, qxr, dxr)
    got = synth.bf16_bits_to_f32(y)
    ref_b = synth.bf16_bits_to_f32(O.round_bf16(ref))
    # Each 2048-K chunk partial is a bf16 value: a different f32 summation
    # order inside a chunk can move a partial by one bf16 ulp (2^-8 of its
    # magnitude), so outputs may differ by 2^-8 * sum|partial| plus one final
    # rounding.  The partials come from the oracle run on each chunk alone.
    partial_abs = np.zeros_like(ref)
    for c0 in range(0, k, 2048):
        c1 = min(k, c0 + 2048)
        partial_abs += np.abs(O.gemv_w4a8(q[:, c0:c1], s[:, c0 // 32:c1 // 32], qxr[:, c0:c1], dxr[:, c0 // 32:c1 // 32]))
    assert np.all(np.abs(got - ref_b) <= 2.0 ** -8 * partial_abs + 2.0 ** -8 * np.abs(ref_b)), f"w4a8 {n}x{k} m={m}"
    max_rel, mae, raw = rel_metrics(got, ref_b)
    assert mae <= 1e-3, mae
    same = np.mean(y == O.round_bf16(ref))
    assert same >= 0.9, f"only {same:.3f} of the outputs match the oracle bit for bit"
    yf = hal.linear_w4a8(w, qx, dx, out_dtype=torch.float32).cpu().numpy()
    assert np.all(np.abs(yf - ref) <= 2.0 ** -8 * partial_abs + 1e-6 * np.abs(ref))


def test_w4a8_within_the_golden_tier_of_the_bf16_reference(dev):
    """The reference checks its W4A8 NPU output against bf16-activation
    goldens with |g - w| <= 0.01 + 0.01|w| (main.rs:2705-2714)."""
    n, k = 2048, 2048
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, 520))
    s = synth.synth_scales(n, k, 520)
    x = synth.synth_x(1, k, 521)
    w = import_planes(dev, q, s)
    qx, dx = hal.quantize_x(to_dev_u16(x))
    g = synth.bf16_bits_to_f32(from_dev_bf16(hal.linear_w4a8(w, qx, dx))[0])
    ref = synth.bf16_bits_to_f32(O.round_bf16(O.gemv_q(q, s, x))[0])
    assert np.all(np.abs(g - ref) <= 0.01 + 0.01 * np.abs(ref))
