"""One decode step of a Llama-shaped transformer over int4 weights: the
reference's decode layer loop (crates/xnpu-cli/src/main.rs:8114-8337) on the
device.

Per layer, as the reference orders it:

    xn = rms_norm(x, ln1)                       main.rs:8121
    qkv = W_qkv xn                              main.rs:8122
    q, k = rope(q), rope(k); q/k norm           main.rs:8132-8143
    append k, v to the cache; attn = GQA(q)     main.rs:8230
    x = x + W_o attn                            main.rs:8320-8325
    xn = rms_norm(x, ln2)                       main.rs:8326
    x = x + W_down swiglu(W_gateup xn)          main.rs:8327-8337

runs as three GEMV chains and one attention launch (six launches with the
8B shapes: chains 1 and 3 launch a prep kernel for their RMSNorm first):

  * chain 1: qkv, with the RMSNorm fused into the chain's activation prep;
  * attention: RoPE, q/k norm, KV-cache append and attention (xq4_attn_decode);
  * chain 2: o with the residual add in its epilogue;
  * chain 3: gate/up with the RMSNorm in the prep and SwiGLU in the epilogue
    (rows interleaved gate_i, up_i), then down, which waits for it, with the
    residual add in its epilogue.

The token's position lives in device memory, so a captured CUDA graph of the
step replays as the position advances (``advance`` bumps it on the device).
There is no host fallback: every launch goes through libxq4.
"""
import numpy as np

from . import hal, synth

# The library's fp16-path threshold (XQ4_XH_MIN_CHUNKS, 16-row x 64-K chunks):
# a chain activation whose readers stream fewer chunks gets no prep launch.
XH_MIN_CHUNKS = 98304


class DecodeLayerWeights:
    """One layer's weights on the device: int4 qkv, o, gate/up (interleaved
    rows gate_i, up_i) and down, bf16 RMSNorm weights ln1 and ln2, optional
    bf16 q/k norm weights [2][128]."""

    def __init__(self, qkv, o, gateup, down, ln1, ln2, qk_norm=None):
        self.qkv, self.o, self.gateup, self.down = qkv, o, gateup, down
        self.ln1, self.ln2, self.qk_norm = ln1, ln2, qk_norm

    def destroy(self):
        for w in (self.qkv, self.o, self.gateup, self.down):
            w.destroy()


class DecodeStep:
    """Buffers, KV caches, chains and attention objects of a decode step over
    `layers` (a list of DecodeLayerWeights), batch 1.

    hidden: model width (the o and down rows, the qkv / gateup K); heads, nkv:
    attention heads (head dim 128); cache_seq: positions of every layer's KV
    cache; rope_base: RoPE base (0 = none); eps: the RMSNorm epsilon; comm,
    world: the communicator over which every layer's gate/up rows are
    sharded (its SwiGLU intermediate gathered inside the chain), or None."""

    def __init__(self, dev, layers, hidden, heads, nkv, cache_seq, rope_base=500000.0, eps=1e-5, comm=None,
                 world=1):
        import torch
        self.dev, self.layers = dev, layers
        self.hidden, self.heads, self.nkv, self.cache_seq = hidden, heads, nkv, cache_seq
        dv = f"cuda:{dev.ordinal}"
        n_qkv = (heads + 2 * nkv) * 128
        inter = layers[0].gateup.n // 2 * world  # gate/up rows sharded over `world` ranks of `comm`
        self.x = torch.zeros((1, hidden), dtype=torch.bfloat16, device=dv)        # the residual stream
        self.h1 = torch.zeros((1, hidden), dtype=torch.bfloat16, device=dv)       # after attention's residual add
        self.qkv = torch.zeros((1, n_qkv), dtype=torch.bfloat16, device=dv)
        self.attn_out = torch.zeros((1, heads * 128), dtype=torch.bfloat16, device=dv)
        self.inter = torch.zeros((1, inter), dtype=torch.bfloat16, device=dv)     # SwiGLU intermediate
        self.pos = torch.zeros(1, dtype=torch.int32, device=dv)
        self.k_cache = [torch.zeros((nkv, cache_seq, 128), dtype=torch.bfloat16, device=dv) for _ in layers]
        self.v_cache = [torch.zeros((nkv, cache_seq, 128), dtype=torch.bfloat16, device=dv) for _ in layers]
        self.attn = hal.Attention(dev, heads, nkv, cache_seq, rope_base)
        p = lambda t: t.data_ptr()  # noqa: E731
        self.chains = []
        for lw in layers:
            c1 = hal.Chain(dev, [(lw.qkv, p(self.x), p(self.qkv), 1, 0, 0, None,
                                  {"norm_w": p(lw.ln1), "eps": eps})])
            c2 = hal.Chain(dev, [(lw.o, p(self.attn_out), p(self.h1), 1, 0, 0, None, {"residual": p(self.x)})])
            c3 = hal.Chain(dev, [(lw.gateup, p(self.h1), p(self.inter), 1, 0, 0, comm,
                                  {"norm_w": p(lw.ln2), "eps": eps, "swiglu": True}),
                                 (lw.down, p(self.inter), p(self.x), 1, 0, 1, None, {"residual": p(self.h1)})])
            self.chains.append((c1, c2, c3))
        # per layer: chains 1 and 3 (each with its prep, their RMSNorm), the
        # attention kernel, chain 2 (its prep only when the o projection streams
        # at least XH_MIN_CHUNKS chunks: below that the library keeps the bf16
        # path and launches no prep)
        o_chunks = (hidden + 15) // 16 * ((heads * 128 + 63) // 64)
        self.launches_per_step = (5 + (2 if o_chunks >= XH_MIN_CHUNKS else 1)) * len(layers)

    def run(self, stream=None):
        """One token through every layer: x (the residual stream) in, x out;
        the position is read from ``pos`` on the device."""
        for li, (c1, c2, c3) in enumerate(self.chains):
            lw = self.layers[li]
            c1.run(stream)
            qn = kn = None
            if lw.qk_norm is not None:
                qn, kn = lw.qk_norm[0], lw.qk_norm[1]
            self.attn.decode(self.qkv[0], self.k_cache[li], self.v_cache[li], self.pos, out=self.attn_out[0],
                             q_norm=qn, k_norm=kn, stream=stream)
            c2.run(stream)
            c3.run(stream)

    def advance(self, stream=None):
        """Next position, on the device (graph-replay friendly)."""
        import torch
        if stream is not None:
            with torch.cuda.stream(stream):
                self.pos.add_(1)
        else:
            self.pos.add_(1)

    def destroy(self):
        for cs in self.chains:
            for c in cs:
                c.destroy()
        self.chains = []
        self.attn.destroy()


def synth_layer(dev, hidden, heads, nkv, inter, seed, qk_norm=False, shard=None):
    """Seeded random-init weights of one layer (the synthetic distributions of
    xnpu_b200.synth; RMSNorm weights 1 + N(0, 0.02)).  shard = (rank, world)
    imports only the rank's rows of the gate/up projection."""
    import torch

    def imp(n, k, s, rows=None):
        src = synth.planes_bytes(synth.synth_codes(n, k, s), synth.synth_scales(n, k, s))
        r0, r1 = rows or (0, 0)
        return hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=r0, row_end=r1))

    rng = np.random.default_rng(seed)

    def norm_w(n):
        w = synth.f32_to_bf16_bits((1.0 + 0.02 * rng.standard_normal(n)).astype(np.float32))
        return torch.from_numpy(w.view(np.int16)).to(f"cuda:{dev.ordinal}").view(torch.bfloat16)

    rows = None
    if shard is not None:
        rank, world = shard
        rows = (rank * 2 * inter // world, (rank + 1) * 2 * inter // world)
    return DecodeLayerWeights(imp((heads + 2 * nkv) * 128, hidden, seed), imp(hidden, heads * 128, seed + 1),
                              imp(2 * inter, hidden, seed + 2, rows), imp(hidden, inter, seed + 3),
                              norm_w(hidden), norm_w(hidden),
                              norm_w(256).view(2, 128) if qk_norm else None)
