"""GPU: decode attention of one token (xq4_attn_decode) against the oracle's
restatement of the reference's decode glue: rope_table + rope_apply
(crates/xnpu-cli/src/main.rs:4817-4839), qk_rms_bf16 (main.rs:4844-4857)
and attention_bf16 (main.rs:4967-5033).

Bars:
  * the k and v rows the kernel appends to the caches are bit-exact (the RoPE
    table is the reference's f32 formula computed on the host; RoPE and the
    norm use the reference's operation order), and no other cache row
    changes;
  * the attention output is within the parity bars of tests/parity.py
    against the oracle's output, and at least 90 % of it bit-identical: the
    kernel splits the positions over CTAs and merges the splits, and uses
    CUDA's expf, so f32 sums are reordered.
Shapes: Llama-3-8B attention (32 q heads over 8 kv heads, 4096-position
caches) with and without the q/k norm, at positions across split edges;
4 q heads over 1 kv head; and three consecutive tokens, each reading the
previous tokens' appended rows.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from parity import assert_parity
from test_gpu_kernels import from_dev_bf16, to_dev_u16
from xnpu_b200 import hal, synth

pytestmark = pytest.mark.gpu


def _case(heads, nkv, cache_seq, pos, seed, norm):
    rng = np.random.default_rng(seed)
    qkv = synth.f32_to_bf16_bits(rng.standard_normal((heads + 2 * nkv) * 128).astype(np.float32))
    kc = synth.f32_to_bf16_bits(rng.standard_normal((nkv, cache_seq, 128)).astype(np.float32))
    vc = synth.f32_to_bf16_bits(rng.standard_normal((nkv, cache_seq, 128)).astype(np.float32))
    w = synth.f32_to_bf16_bits((1.0 + 0.1 * rng.standard_normal((2, 128))).astype(np.float32)) if norm else None
    return qkv, kc, vc, w


def _oracle(qkv, kc, vc, w, heads, nkv, cache_seq, pos, base):
    q, k, v = qkv[:heads * 128], qkv[heads * 128:(heads + nkv) * 128], qkv[(heads + nkv) * 128:]
    if base > 0:
        c, s = O.rope_table(pos, base)
        q, k = O.rope_apply(q, c, s), O.rope_apply(k, c, s)
    if w is not None:
        q, k = O.qk_rms(q, w[0]), O.qk_rms(k, w[1])
    kc, vc = kc.copy(), vc.copy()
    kc[:, pos, :] = k.reshape(nkv, 128)
    vc[:, pos, :] = v.reshape(nkv, 128)
    return O.attention(q, kc, vc, pos, cache_seq, heads, nkv), kc, vc


def _run(dev, attn, qkv, kc, vc, w, pos):
    kd, vd = to_dev_u16(kc), to_dev_u16(vc)
    pd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    wd = None if w is None else to_dev_u16(w)
    out = attn.decode(to_dev_u16(qkv), kd, vd, pd, q_norm=None if wd is None else wd[0],
                      k_norm=None if wd is None else wd[1])
    torch.cuda.synchronize()
    return from_dev_bf16(out), from_dev_bf16(kd), from_dev_bf16(vd)


def _check(got, want, got_kc, want_kc, got_vc, want_vc, what):
    assert np.array_equal(got_kc, want_kc), f"{what}: k cache"
    assert np.array_equal(got_vc, want_vc), f"{what}: v cache"
    assert_parity(synth.bf16_bits_to_f32(got), synth.bf16_bits_to_f32(want), what)
    same = float(np.mean(got == want))
    assert same >= 0.9, (what, same)


@pytest.mark.parametrize("pos", [0, 1, 31, 32, 110, 111, 1000, 4095])
@pytest.mark.parametrize("norm", [False, True])
def test_attention_llama8b_shape(dev, pos, norm):
    heads, nkv, cache_seq, base = 32, 8, 4096, 500000.0
    attn = hal.Attention(dev, heads, nkv, cache_seq, base)
    qkv, kc, vc, w = _case(heads, nkv, cache_seq, pos, 100 + pos, norm)
    got, gk, gv = _run(dev, attn, qkv, kc, vc, w, pos)
    want, wk, wv = _oracle(qkv, kc, vc, w, heads, nkv, cache_seq, pos, base)
    _check(got, want, gk, wk, gv, wv, f"pos={pos} norm={norm}")
    assert dev.fault() == 0
    attn.destroy()


def test_attention_group_of_four_no_rope(dev):
    heads, nkv, cache_seq, pos = 4, 1, 300, 257
    attn = hal.Attention(dev, heads, nkv, cache_seq, 0.0)
    qkv, kc, vc, w = _case(heads, nkv, cache_seq, pos, 7, True)
    got, gk, gv = _run(dev, attn, qkv, kc, vc, w, pos)
    want, wk, wv = _oracle(qkv, kc, vc, w, heads, nkv, cache_seq, pos, 0.0)
    _check(got, want, gk, wk, gv, wv, "4 over 1, no rope")
    attn.destroy()


def test_attention_consecutive_tokens(dev):
    """Three tokens in a row on one cache: each step appends its k/v and
    attends over every earlier token's appended row."""
    heads, nkv, cache_seq, base = 32, 8, 512, 10000.0
    attn = hal.Attention(dev, heads, nkv, cache_seq, base)
    rng = np.random.default_rng(3)
    kc = np.zeros((nkv, cache_seq, 128), dtype=np.uint16)
    vc = np.zeros((nkv, cache_seq, 128), dtype=np.uint16)
    kd, vd = to_dev_u16(kc), to_dev_u16(vc)
    pd = torch.zeros(1, dtype=torch.int32, device="cuda")
    w = synth.f32_to_bf16_bits((1.0 + 0.1 * rng.standard_normal((2, 128))).astype(np.float32))
    wd = to_dev_u16(w)
    for pos in range(3):
        qkv = synth.f32_to_bf16_bits(rng.standard_normal((heads + 2 * nkv) * 128).astype(np.float32))
        pd.fill_(pos)
        out = attn.decode(to_dev_u16(qkv), kd, vd, pd, q_norm=wd[0], k_norm=wd[1])
        torch.cuda.synchronize()
        want, kc, vc = _oracle(qkv, kc, vc, w, heads, nkv, cache_seq, pos, base)
        _check(from_dev_bf16(out), want, from_dev_bf16(kd), kc, from_dev_bf16(vd), vc, f"token {pos}")
    assert dev.fault() == 0
    attn.destroy()


def test_attention_position_outside_the_cache(dev):
    """A device-resident position past the cache is refused by the kernel:
    nothing is written and fault bit 0x20 is raised."""
    heads, nkv, cache_seq = 8, 2, 64
    attn = hal.Attention(dev, heads, nkv, cache_seq, 10000.0)
    qkv, kc, vc, _ = _case(heads, nkv, cache_seq, 0, 9, False)
    kd, vd = to_dev_u16(kc), to_dev_u16(vc)
    out = torch.full((heads * 128,), 7.0, dtype=torch.bfloat16, device="cuda")
    for bad in (cache_seq, -1):
        attn.decode(to_dev_u16(qkv), kd, vd, torch.tensor([bad], dtype=torch.int32, device="cuda"), out=out)
        torch.cuda.synchronize()
        assert dev.fault() == 0x20
    assert np.array_equal(from_dev_bf16(kd), kc) and np.array_equal(from_dev_bf16(vd), vc)
    assert bool((out == 7.0).all())
    attn.destroy()


def test_attention_handles_of_different_sizes(dev):
    """A handle created after a larger one (a smaller shared-memory plan) must
    leave the larger one's launches valid: the kernel's shared-memory limit is
    one per-device attribute, raised by creates and never lowered."""
    heads, nkv, base = 32, 8, 500000.0
    big = hal.Attention(dev, heads, nkv, 4096, base)
    small = hal.Attention(dev, heads, nkv, 64, base)
    for attn, cache_seq, pos in ((big, 4096, 1000), (small, 64, 40), (big, 4096, 4095)):
        qkv, kc, vc, w = _case(heads, nkv, cache_seq, pos, 200 + pos, True)
        got, gk, gv = _run(dev, attn, qkv, kc, vc, w, pos)
        want, wk, wv = _oracle(qkv, kc, vc, w, heads, nkv, cache_seq, pos, base)
        _check(got, want, gk, wk, gv, wv, f"cache {cache_seq} pos={pos}")
    assert dev.fault() == 0
    small.destroy()
    big.destroy()
