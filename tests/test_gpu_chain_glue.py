"""GPU: decode-step glue fused into chain ops (RMSNorm in the activation
prep, SwiGLU and residual-add epilogues), against the oracle's restatement
of the reference's glue (crates/xnpu-cli/src/main.rs:4714-4745).

Bars:
  * the epilogues themselves: the residual add bit-exact against add_bf16 of
    the GPU's own unfused GEMV output; SwiGLU against swiglu_bf16 of the
    GPU's own unfused gate/up outputs, bit-exact except where CUDA's expf and
    the C library's differ in the last bit (at most 1 bf16 ulp, on under
    0.5 % of the outputs);
  * RMSNorm + GEMV against the oracle (rms_norm_bf16, then the GEMV).  The
    reference sums the squares sequentially, the GPU in a fixed tree order,
    so 1/rms may differ in its last f32 bit and a normalised activation that
    lies at a bf16 rounding tie may round one ulp the other way (about one
    element per token).  The bar is that bound: |y - ref| <= 2^-8 *
    sum_k |w_k| |xn_k| (one ulp of every activation) + 2^-8 |ref| (the
    output's own rounding), plus mean absolute error <= 1e-3;
  * the rest of the block from the GPU's own norm-GEMV output: SwiGLU and
    the residual add as above, so the whole block is pinned step by step;
  * two runs give the same bits; no fault bit; bad combinations rejected.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from xnpu_b200 import hal, synth
from test_gpu_kernels import from_dev_bf16, import_planes, to_dev_u16
from test_gpu_chain import _raw

pytestmark = pytest.mark.gpu

HID, INTER, M = 4096, 14336, 2


def _w(n, k, seed):
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, seed))
    s = synth.synth_scales(n, k, seed)
    return q, s


def _gamma(k, seed):
    rng = np.random.default_rng(seed)
    return synth.f32_to_bf16_bits(rng.normal(1.0, 0.1, size=k).astype(np.float32))


def _assert_norm_bound(got, q, s, xn, what):
    """GPU output (f32 values) of a GEMV over RMS-normalised activations
    against the oracle: within one bf16 ulp of every normalised activation
    plus the output's rounding (see the module docstring)."""
    ref = O.gemv_q(q, s, xn)
    absx = (np.asarray(xn, dtype=np.uint16) & 0x7FFF).astype(np.uint16)
    bound = O.gemv_q(np.abs(q).astype(np.int8), s, absx)
    err = np.abs(np.asarray(got, dtype=np.float64) - ref)
    assert np.all(err <= 2.0 ** -8 * bound * 1.01 + 2.0 ** -8 * np.abs(ref)), what
    assert err.mean() <= 1e-3, (what, err.mean())


def _ulp_dist(a, b):
    """Distance in bf16 units in the last place between same-sign values."""
    a = np.asarray(a, dtype=np.uint16).astype(np.int32)
    b = np.asarray(b, dtype=np.uint16).astype(np.int32)
    same_sign = (a >> 15) == (b >> 15)
    return np.where(same_sign, np.abs(a - b), 1 << 16)


def test_ffn_block_chain(dev):
    h = synth.synth_x(M, HID, 4242)
    gamma = _gamma(HID, 4243)
    qgu, sgu = _w(2 * INTER, HID, 4244)   # rows alternate gate_i, up_i
    qd, sd = _w(HID, INTER, 4245)
    wgu, wd = import_planes(dev, qgu, sgu), import_planes(dev, qd, sd)
    hd, gd = to_dev_u16(h), to_dev_u16(gamma.reshape(1, HID))
    act = torch.empty((M, INTER), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((M, HID), dtype=torch.bfloat16, device="cuda")
    g_plain = torch.empty((M, 2 * INTER), dtype=torch.bfloat16, device="cuda")

    ffn = hal.Chain(dev, [
        (wgu, hd.data_ptr(), act.data_ptr(), M, 0, 0, {"norm_w": gd.data_ptr(), "eps": 1e-5, "swiglu": True}),
        (wd, act.data_ptr(), out.data_ptr(), M, 0, 1, {"residual": hd.data_ptr()}),
    ])
    plain = hal.Chain(dev, [(wgu, hd.data_ptr(), g_plain.data_ptr(), M, 0, 0, {"norm_w": gd.data_ptr()})])
    runs = []
    for _ in range(2):
        act.fill_(float("nan"))
        out.fill_(float("nan"))
        ffn.run()
        torch.cuda.synchronize()
        runs.append((from_dev_bf16(act).copy(), from_dev_bf16(out).copy()))
    assert np.array_equal(runs[0][0], runs[1][0]) and np.array_equal(runs[0][1], runs[1][1])
    plain.run()
    torch.cuda.synchronize()
    assert dev.fault() == 0
    a_gpu, o_gpu = runs[0]

    # SwiGLU epilogue: the reference's swiglu of the same GEMV outputs
    g = from_dev_bf16(g_plain)
    want_act = O.swiglu(np.concatenate([g[:, 0::2], g[:, 1::2]], axis=1))
    d = _ulp_dist(a_gpu, want_act)
    assert d.max() <= 1 and (d > 0).mean() < 5e-3, (int(d.max()), float((d > 0).mean()))

    # residual epilogue: add_bf16 of the down GEMV (same bf16 path, single op)
    y_down = from_dev_bf16(_raw(wd, act, M, HID, False))
    assert np.array_equal(o_gpu, O.add_bf16(h, y_down))

    # RMSNorm + GEMV against the oracle (rms_norm_bf16, then the GEMV)
    xn = O.rms_norm(h, gamma)
    rows = np.unique(np.concatenate([np.arange(512), np.arange(2 * INTER - 512, 2 * INTER)]))
    _assert_norm_bound(synth.bf16_bits_to_f32(g[:, rows]), qgu[rows], sgu[rows], xn, "rmsnorm -> gateup")
    ffn.destroy()
    plain.destroy()


def test_norm_op_f32(dev):
    """RMSNorm in the prep feeding an f32-output op (a qkv-like projection)."""
    n, k, m = 6144, 4096, 3
    x = synth.synth_x(m, k, 4250)
    gamma = _gamma(k, 4251)
    q, s = _w(n, k, 4252)
    w = import_planes(dev, q, s)
    xd, gd = to_dev_u16(x), to_dev_u16(gamma.reshape(1, k))
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ch = hal.Chain(dev, [(w, xd.data_ptr(), y.data_ptr(), m, 1, 0, {"norm_w": gd.data_ptr(), "eps": 1e-6})])
    ch.run()
    torch.cuda.synchronize()
    rows = np.arange(0, n, 5)
    _assert_norm_bound(y.cpu().numpy()[:, rows], q[rows], s[rows], O.rms_norm(x, gamma, eps=1e-6), "rmsnorm f32")
    assert dev.fault() == 0
    ch.destroy()


def test_glue_rejections(dev):
    q, s = _w(64, 64, 4260)
    w = import_planes(dev, q, s)
    qo, so = _w(63, 64, 4261)
    w_odd = import_planes(dev, qo, so)
    x = to_dev_u16(synth.synth_x(1, 64, 4262))
    y = torch.empty((1, 64), dtype=torch.float32, device="cuda")
    y2 = torch.empty((1, 64), dtype=torch.bfloat16, device="cuda")
    bad = [
        [(w, x.data_ptr(), y.data_ptr(), 1, 1, 0, {"residual": x.data_ptr()})],          # residual into f32
        [(w_odd, x.data_ptr(), y2.data_ptr(), 1, 0, 0, {"swiglu": True})],               # odd rows
        [(w, x.data_ptr(), y2.data_ptr(), 1, 0, 0, {"swiglu": True, "residual": x.data_ptr()})],
        [(w, x.data_ptr(), y2.data_ptr(), 1, 0, 0),                                     # norm of a chain output
         (w, y2.data_ptr(), y.data_ptr(), 1, 1, 1, {"norm_w": x.data_ptr()})],
    ]
    for ops in bad:
        with pytest.raises(hal.Xq4Error):
            hal.Chain(dev, ops)
