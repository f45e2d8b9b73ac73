"""GPU: W4A8 chain ops (xq4_chain_op.w4a8), the reference's NPU numerics
inside the GEMV chain, and the fused rms -> int8 quant -> W4A8 GEMV of the
reference's M9/P18 pairs (crates/xnpu-cli/src/main.rs:7802-7815).

  * A W4A8 op of a chain gives, bit for bit, what xq4_quantize_x followed by
    xq4_linear_w4a8 gives on the same activation: the chain's prep quantizes
    with the same formula, and per row block the chain runs the same integer
    MMAs, scale products, 2048-K chunk roundings and partial sums in the same
    order (several shapes: whole and partial 2048-K chunks, a K tail of half
    a chunk, ragged rows, 1 to 8 tokens, bf16 and f32 outputs, next to fp16
    ops and an op that waits for a W4A8 op's output).
  * With the RMSNorm fused in front (the prep normalises, then quantizes):
    the prep sums the squares in its own fixed order (per-thread sums over
    runs of 8, a butterfly per warp, the warps in order), which this test
    restates exactly on the CPU; from that
    normalised activation the oracle quantizes (w4u_quantize_x) and runs its
    W4A8 GEMV, and the chain's output must meet the bound of
    test_gpu_w4a8.py (one bf16 ulp of each 2048-K chunk partial, at least
    90 % bit-identical).  Against the reference's sequential sum of squares
    it is within the parity bars of tests/parity.py.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import rel_metrics
from test_gpu_kernels import from_dev_bf16, import_planes, to_dev_u16
from xnpu_b200 import hal, synth

pytestmark = pytest.mark.gpu

SHAPES = [  # (n, k, m, f32)
    (4096, 4096, 1, False),
    (14336, 4096, 3, False),
    (4096, 14336, 1, True),     # 7 whole 2048-K chunks
    (2048, 6144, 8, False),
    (333, 160, 2, False),       # a partial chunk, ragged rows
    (1040, 4128, 5, True),      # K tail of half a 64-K chunk
]


def _bits(t):
    return t.view(torch.int32 if t.dtype == torch.float32 else torch.int16)


def test_w4a8_chain_ops_match_the_single_op(dev):
    ws, ops, refs = [], [], []
    for i, (n, k, m, f32) in enumerate(SHAPES):
        q = synth.unpack_codes_signed(synth.synth_codes(n, k, 800 + i))
        s = synth.synth_scales(n, k, 800 + i)
        w = import_planes(dev, q, s)
        xd = to_dev_u16(synth.synth_x(m, k, 810 + i))
        dt = torch.float32 if f32 else torch.bfloat16
        y = torch.full((m, n), float("nan"), dtype=dt, device="cuda")
        qx, dx = hal.quantize_x(xd)
        refs.append(hal.linear_w4a8(w, qx, dx, out_dtype=dt))
        ws.append((w, xd, y))
        ops.append((w, xd.data_ptr(), y.data_ptr(), m, 1 if f32 else 0, 0, None, {"w4a8": True}))
    # an fp16 op beside them, and a bf16-path op reading op 0's output
    n, k = 2048, 4096
    wq = import_planes(dev, synth.unpack_codes_signed(synth.synth_codes(n, k, 820)), synth.synth_scales(n, k, 820))
    x16 = to_dev_u16(synth.synth_x(1, k, 821))
    y16 = torch.empty((1, n), dtype=torch.bfloat16, device="cuda")
    wd = import_planes(dev, synth.unpack_codes_signed(synth.synth_codes(512, 4096, 822)),
                       synth.synth_scales(512, 4096, 822))
    yd = torch.empty((1, 512), dtype=torch.bfloat16, device="cuda")
    ops.insert(1, (wq, x16.data_ptr(), y16.data_ptr(), 1, 0, 0))
    ops.append((wd, ws[0][2].data_ptr(), yd.data_ptr(), 1, 0, 1))
    chain = hal.Chain(dev, ops)
    for rep in range(2):
        for _, _, y in ws:
            y.fill_(float("nan"))
        chain.run()
        torch.cuda.synchronize()
        for (n, k, m, f32), (w, xd, y), ref in zip(SHAPES, ws, refs):
            assert torch.equal(_bits(y), _bits(ref)), (rep, (n, k, m, f32))
    # the op after the wait read op 0's complete output
    yr = hal.linear(wd, ws[0][2])
    assert torch.equal(_bits(yd), _bits(yr))
    assert dev.fault() == 0
    chain.destroy()


def prep_rms_norm(x_bits, w_bits, eps=1e-5):
    """The chain prep's RMSNorm, operation for operation in f32: thread i of
    256 sums the squares of its runs of 8 activations (runs i, i + 256, ...,
    each run's values in order), a butterfly (xor 16, 8, 4, 2, 1) adds each
    warp's 32 sums, the 8 warp sums are added in warp order; inv = 1 /
    sqrt(ss / k + eps), out = RNE_bf16((x * inv) * w)."""
    x = synth.bf16_bits_to_f32(x_bits).astype(np.float32)
    w = synth.bf16_bits_to_f32(w_bits).astype(np.float32)
    m, k = x.shape
    out = np.empty_like(x_bits)
    f32 = np.float32
    runs = k // 8
    for t in range(m):
        ss = np.zeros(256, dtype=np.float32)
        for r0 in range(0, runs, 256):
            idx = np.arange(r0, min(runs, r0 + 256))
            for e in range(8):
                v = x[t, 8 * idx + e]
                ss[idx - r0] = (ss[idx - r0] + (v * v).astype(np.float32)).astype(np.float32)
        ws = ss.reshape(8, 32)
        for o in (16, 8, 4, 2, 1):
            ws = (ws + ws[:, np.arange(32) ^ o]).astype(np.float32)
        tot = f32(0.0)
        for i in range(8):
            tot = f32(tot + ws[i, 0])
        inv = f32(1.0) / np.sqrt(f32(f32(tot) / f32(k)) + f32(eps))
        out[t] = synth.f32_to_bf16_bits(((x[t] * inv).astype(np.float32) * w).astype(np.float32))
    return out


def w4a8_bound_ok(got, ref, q, s, qxr, dxr, k):
    """test_gpu_w4a8.py's bound: one bf16 ulp of each 2048-K chunk partial
    plus the final rounding."""
    partial_abs = np.zeros_like(ref)
    for c0 in range(0, k, 2048):
        c1 = min(k, c0 + 2048)
        partial_abs += np.abs(O.gemv_w4a8(q[:, c0:c1], s[:, c0 // 32:c1 // 32], qxr[:, c0:c1],
                                          dxr[:, c0 // 32:c1 // 32]))
    ref_b = synth.bf16_bits_to_f32(O.round_bf16(ref))
    return bool(np.all(np.abs(got - ref_b) <= 2.0 ** -8 * partial_abs + 2.0 ** -8 * np.abs(ref_b)))


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 1), (14336, 4096, 2), (4096, 14336, 1)])
def test_fused_rms_quant_w4a8(dev, n, k, m):
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, 830 + m))
    s = synth.synth_scales(n, k, 830 + m)
    w = import_planes(dev, q, s)
    x = synth.synth_x(m, k, 831 + m)
    rng = np.random.default_rng(832)
    nw = synth.f32_to_bf16_bits((1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32))
    xd, nwd = to_dev_u16(x), to_dev_u16(nw[None, :])
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    chain = hal.Chain(dev, [(w, xd.data_ptr(), y.data_ptr(), m, 0, 0, None,
                             {"w4a8": True, "norm_w": nwd.data_ptr(), "eps": 1e-5})])
    chain.run()
    torch.cuda.synchronize()
    got_bits = from_dev_bf16(y)
    got = synth.bf16_bits_to_f32(got_bits)
    # exact: from the prep's own normalisation
    xn = prep_rms_norm(x, nw)
    qs, ds = zip(*(O.quantize_x(xn[t]) for t in range(m)))
    qxr, dxr = np.stack(qs), np.stack(ds)
    ref = O.gemv_w4a8(q, s, qxr, dxr)
    assert w4a8_bound_ok(got, ref, q, s, qxr, dxr, k), f"{n}x{k} m={m}"
    same = float(np.mean(got_bits == O.round_bf16(ref)))
    assert same >= 0.9, same
    # against the reference's own order of the sum of squares: the parity bars
    xr = O.rms_norm(x, nw)
    qs, ds = zip(*(O.quantize_x(xr[t]) for t in range(m)))
    ref2 = O.gemv_w4a8(q, s, np.stack(qs), np.stack(ds))
    max_rel, mae, _ = rel_metrics(got, synth.bf16_bits_to_f32(O.round_bf16(ref2)),
                                  f"fused rms+quant+w4a8 {n}x{k} m={m}")
    assert mae <= 1e-3, mae
    assert dev.fault() == 0
    chain.destroy()
