"""GPU: one decode step of a Llama-shaped model through xnpu_b200.decode
(three GEMV chains and the attention kernel per layer) against the oracle's
restatement of the reference's decode layer (crates/xnpu-cli/src/main.rs:
8114-8337: rms_norm, qkv, rope, q/k norm, attention, o, residual, rms_norm,
gate/up, SwiGLU, down, residual).

  * Stage by stage on one layer: every intermediate the step leaves on the
    device is checked against the oracle applied to the GPU's own input of
    that stage -- the appended k/v rows bit-exact, the rest within the
    parity bars (tests/parity.py);
  * end to end, two layers over three consecutive tokens: the residual stream
    after each token against the oracle's composition.  The stages' last-bit
    differences (one bf16 ulp here and there, each within the bars above)
    compound through the softmax, the norms and the residual adds, so the
    end-to-end bound is stated against the stream's scale: mean absolute
    error <= 1e-3 x RMS and maximum absolute error <= 2^-5 x max |x|.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_parity, rel_metrics
from test_gpu_kernels import from_dev_bf16, to_dev_u16
from xnpu_b200 import decode, synth

pytestmark = pytest.mark.gpu

HID, HEADS, NKV, INTER, CACHE = 1024, 8, 2, 2048, 64


def planes(n, k, seed):
    return synth.unpack_codes_signed(synth.synth_codes(n, k, seed)), synth.synth_scales(n, k, seed)


def bits(t):
    return from_dev_bf16(t).reshape(-1)


def f32(b):
    return synth.bf16_bits_to_f32(np.asarray(b, dtype=np.uint16))


def gemv(w, x):
    return O.round_bf16(O.gemv_q(w[0], w[1], np.asarray(x, dtype=np.uint16).reshape(1, -1)))[0]


def swiglu_interleaved(gu):
    """The reference's swiglu_bf16 on a fused [gate | up] vector; the
    device's gate/up rows alternate gate_i, up_i."""
    return O.swiglu(np.concatenate([gu[0::2], gu[1::2]]))[0]


def host_weights(seed):
    return {"qkv": planes((HEADS + 2 * NKV) * 128, HID, seed), "o": planes(HID, HEADS * 128, seed + 1),
            "gateup": planes(2 * INTER, HID, seed + 2), "down": planes(HID, INTER, seed + 3)}


def oracle_layer(hw, ln1, ln2, qkn, x, kc, vc, pos, base):
    xn = O.rms_norm(x, ln1)[0]
    qkv = gemv(hw["qkv"], xn)
    q, k, v = qkv[:HEADS * 128], qkv[HEADS * 128:(HEADS + NKV) * 128], qkv[(HEADS + NKV) * 128:]
    c, s = O.rope_table(pos, base)
    q, k = O.rope_apply(q, c, s), O.rope_apply(k, c, s)
    if qkn is not None:
        q, k = O.qk_rms(q, qkn[0]), O.qk_rms(k, qkn[1])
    kc[:, pos, :] = k.reshape(NKV, 128)
    vc[:, pos, :] = v.reshape(NKV, 128)
    attn = O.attention(q, kc, vc, pos, CACHE, HEADS, NKV)
    h1 = O.add_bf16(x, gemv(hw["o"], attn))
    sw = swiglu_interleaved(gemv(hw["gateup"], O.rms_norm(h1, ln2)[0]))
    return O.add_bf16(h1, gemv(hw["down"], sw))


@pytest.mark.parametrize("qk_norm", [False, True])
def test_decode_layer_stage_by_stage(dev, qk_norm):
    base = 500000.0
    lw = decode.synth_layer(dev, HID, HEADS, NKV, INTER, 500, qk_norm=qk_norm)
    hw = host_weights(500)
    step = decode.DecodeStep(dev, [lw], HID, HEADS, NKV, CACHE, rope_base=base)
    rng = np.random.default_rng(501)
    kc = synth.f32_to_bf16_bits(rng.standard_normal((NKV, CACHE, 128)).astype(np.float32))
    vc = synth.f32_to_bf16_bits(rng.standard_normal((NKV, CACHE, 128)).astype(np.float32))
    x0 = synth.synth_x(1, HID, 502)[0]
    pos = 37
    step.k_cache[0].copy_(to_dev_u16(kc))
    step.v_cache[0].copy_(to_dev_u16(vc))
    step.x.copy_(to_dev_u16(x0[None, :]))
    step.pos.fill_(pos)
    step.run()
    torch.cuda.synchronize()
    ln1, ln2 = bits(lw.ln1), bits(lw.ln2)
    qkn = None if lw.qk_norm is None else from_dev_bf16(lw.qk_norm)
    # qkv of the normalised residual stream
    g_qkv = bits(step.qkv)
    assert_parity(f32(g_qkv), f32(gemv(hw["qkv"], O.rms_norm(x0, ln1)[0])), "qkv (fused RMSNorm)")
    # the appended cache rows, from the GPU's qkv: bit-exact
    q, k, v = g_qkv[:HEADS * 128], g_qkv[HEADS * 128:(HEADS + NKV) * 128], g_qkv[(HEADS + NKV) * 128:]
    c, s = O.rope_table(pos, base)
    q, k = O.rope_apply(q, c, s), O.rope_apply(k, c, s)
    if qkn is not None:
        q, k = O.qk_rms(q, qkn[0]), O.qk_rms(k, qkn[1])
    kc[:, pos, :] = k.reshape(NKV, 128)
    vc[:, pos, :] = v.reshape(NKV, 128)
    assert np.array_equal(from_dev_bf16(step.k_cache[0]), kc)
    assert np.array_equal(from_dev_bf16(step.v_cache[0]), vc)
    g_attn = bits(step.attn_out)
    assert_parity(f32(g_attn), f32(O.attention(q, kc, vc, pos, CACHE, HEADS, NKV)), "attention")
    g_h1 = bits(step.h1)
    assert_parity(f32(g_h1), f32(O.add_bf16(x0, gemv(hw["o"], g_attn))), "o + residual")
    g_inter = bits(step.inter)
    assert_parity(f32(g_inter), f32(swiglu_interleaved(gemv(hw["gateup"], O.rms_norm(g_h1, ln2)[0]))),
                  "gate/up (fused RMSNorm) + SwiGLU")
    assert_parity(f32(bits(step.x)), f32(O.add_bf16(g_h1, gemv(hw["down"], g_inter))), "down + residual")
    assert dev.fault() == 0
    step.destroy()
    lw.destroy()


def test_decode_two_layers_three_tokens(dev):
    base = 10000.0
    lws = [decode.synth_layer(dev, HID, HEADS, NKV, INTER, 600 + 10 * i, qk_norm=True) for i in range(2)]
    hws = [host_weights(600 + 10 * i) for i in range(2)]
    step = decode.DecodeStep(dev, lws, HID, HEADS, NKV, CACHE, rope_base=base)
    caches = [(np.zeros((NKV, CACHE, 128), np.uint16), np.zeros((NKV, CACHE, 128), np.uint16)) for _ in lws]
    x = synth.synth_x(1, HID, 603)[0]
    step.x.copy_(to_dev_u16(x[None, :]))
    for pos in range(3):
        step.run()
        torch.cuda.synchronize()
        for li, (lw, hw) in enumerate(zip(lws, hws)):
            x = oracle_layer(hw, bits(lw.ln1), bits(lw.ln2), from_dev_bf16(lw.qk_norm), x, caches[li][0],
                             caches[li][1], pos, base)
        got, want = f32(bits(step.x)).astype(np.float64), f32(x).astype(np.float64)
        rel_metrics(got, want, f"two layers, token {pos}")
        err = np.abs(got - want)
        rms, top = float(np.sqrt(np.mean(want ** 2))), float(np.abs(want).max())
        assert err.mean() <= 1e-3 * rms and err.max() <= 2.0 ** -5 * top, (pos, err.mean(), err.max(), rms, top)
        step.advance()
        x = bits(step.x)  # the next token's input is the GPU's state (the oracle follows it stage by stage)
    assert dev.fault() == 0
    step.destroy()
    for lw in lws:
        lw.destroy()
