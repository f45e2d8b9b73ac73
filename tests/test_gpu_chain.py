"""GPU: a chain of GEMV ops run as one persistent kernel (xq4_chain_*).

An op whose activation no op of the chain writes runs the fp16 path from an
image prepared once per run when the activation's readers stream at least
the single-op GEMV's threshold of chunks (else the bf16 path, as that GEMV);
an op that reads an earlier op's output runs the bf16 path.  Bars:
  * every op within the GEMV parity bars against the oracle (8B decode
    shapes, ragged n and K tails with k % 64 == 32, m = 1, 3, 8, bf16 / f32
    outputs), and bit-identical to the single-op GEMV, which takes the same
    path (fp16 for the large matrices at m <= 5 and k = 4096, bf16 below the
    threshold);
  * bf16-path ops (wait_prev, x = the previous op's y written in the same
    launch): bit-identical to the single-op GEMV run on the same input;
  * repeated runs (the completion counters reset) and the device-queue
    submit give the same bits; no fault bit is raised.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from xnpu_b200 import hal, lib, synth
from xnpu_b200._lib import check
from test_gpu_kernels import assert_parity, from_dev_bf16, import_planes, rel_metrics, to_dev_u16

pytestmark = pytest.mark.gpu


def _op_inputs(n, k, m, seed):
    q = synth.unpack_codes_signed(synth.synth_codes(n, k, seed))
    s = synth.synth_scales(n, k, seed)
    x = synth.synth_x(m, k, seed + 1)
    return q, s, x


def _raw(w, xd, m, n, f32):
    y = torch.empty((m, n), dtype=torch.float32 if f32 else torch.bfloat16, device="cuda")
    check(lib().xq4_linear_raw(w.handle, xd.data_ptr(), y.data_ptr(), m, 1 if f32 else 0,
                               torch.cuda.current_stream().cuda_stream))
    return y


def _bits(t):
    return t.view(torch.int32 if t.dtype == torch.float32 else torch.int16)


SHAPES = [  # (n, k, m, f32)
    (6144, 4096, 1, False),    # qkv
    (4096, 4096, 1, False),    # o
    (14336, 4096, 1, False),   # gate
    (4096, 14336, 1, False),   # down
    (333, 160, 3, False),      # ragged rows, partial stage
    (4100, 4128, 8, True),     # K tail (k % 64 == 32), f32 out
    (17, 96, 8, False),        # fewer row blocks than CTAs
    (2048, 2048, 3, True),
    (28672, 4096, 3, True),    # the single-op GEMV's fp16 path too: bit-identical
    (28672, 4096, 1, False),
]
# Every op reads its own activation: the two 28672 x 4096 ops stream enough
# chunks for the fp16 path, in the chain and in xq4_linear_raw alike; the
# others stay below the threshold and run the bf16 path in both.  So every
# op's output is bit-identical to the single-op GEMV's.
RAW_SAME = set(range(10))


def _oracle_rows(n):
    if n <= 1536:
        return np.arange(n)
    return np.unique(np.concatenate([np.arange(512), np.arange(n - 512, n)]))


def test_chain_matches_single_ops(dev):
    ws, ops, refs, oracle = [], [], [], []
    for i, (n, k, m, f32) in enumerate(SHAPES):
        q, s, x = _op_inputs(n, k, m, 900 + i)
        w = import_planes(dev, q, s)
        xd = to_dev_u16(x)
        y = torch.full((m, n), float("nan"), dtype=torch.float32 if f32 else torch.bfloat16, device="cuda")
        ws.append((w, xd, y))
        ops.append((w, xd.data_ptr(), y.data_ptr(), m, 1 if f32 else 0, i % 2))
        refs.append(_raw(w, xd, m, n, f32) if i in RAW_SAME else None)
        rows = _oracle_rows(n)
        oracle.append((rows, O.gemv_q(q[rows], s[rows], x)))
    chain = hal.Chain(dev, ops)
    first = None
    for rep in range(3):
        for _, _, y in ws:
            y.fill_(float("nan"))
        if rep < 2:
            chain.run()
        else:
            hal.timeline_wait(dev, chain.submit(), 10_000_000_000)
        torch.cuda.synchronize()
        bits = [_bits(y).clone() for _, _, y in ws]
        if first is None:
            first = bits
        for i, (b, f) in enumerate(zip(bits, first)):
            assert torch.equal(b, f), (rep, SHAPES[i], "runs differ")
        for i, ((w, xd, y), ref) in enumerate(zip(ws, refs)):
            if ref is not None:
                assert torch.equal(_bits(y), _bits(ref)), (rep, SHAPES[i])
    assert dev.fault() == 0
    for (n, k, m, f32), (_, _, y), (rows, ref) in zip(SHAPES, ws, oracle):
        if f32:
            max_rel, mae, _ = rel_metrics(y.cpu().numpy()[:, rows], ref)
            assert max_rel <= 1e-2 and mae <= 1e-3, ((n, k, m), max_rel, mae)
        else:
            assert_parity(from_dev_bf16(y)[:, rows], ref, f"chain {n}x{k} m={m}")
    chain.destroy()


def test_chain_dependent_ops(dev):
    """o -> gate -> down with each op reading the previous op's output (the
    wait_prev barrier inside the launch): the first op (external x, fp16
    path) against the oracle, the others (bf16 path) bit-identical to the
    single-op GEMV on the chain's own upstream output."""
    m = 2
    dims = [(4096, 4096), (14336, 4096), (4096, 14336)]  # (n, k); k of op i = n of op i-1
    x0h = synth.synth_x(m, 4096, 77)
    x0 = to_dev_u16(x0h)
    ws, ys, qs = [], [], []
    for i, (n, k) in enumerate(dims):
        q, s, _ = _op_inputs(n, k, 1, 950 + i)
        qs.append((q, s))
        ws.append(import_planes(dev, q, s))
        ys.append(torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda"))
    ops = []
    for i, (w, y) in enumerate(zip(ws, ys)):
        xp = x0.data_ptr() if i == 0 else ys[i - 1].data_ptr()
        ops.append((w, xp, y.data_ptr(), m, 0, 1))
    chain = hal.Chain(dev, ops)
    for rep in range(2):
        for y in ys:
            y.fill_(float("nan"))
        chain.run()
        torch.cuda.synchronize()
        rows = _oracle_rows(dims[0][0])
        q, s = qs[0]
        assert_parity(from_dev_bf16(ys[0])[:, rows], O.gemv_q(q[rows], s[rows], x0h), f"rep {rep} op 0")
        for i in (1, 2):
            ref = _raw(ws[i], ys[i - 1], m, dims[i][0], False)
            assert torch.equal(_bits(ys[i]), _bits(ref)), (rep, i)
    assert dev.fault() == 0
    chain.destroy()


def test_chain_sparse_segments(dev):
    """Segments that few CTAs visit: a 32-row op (2 row blocks, so 2 CTAs)
    between two large ones, a 4096-row op over K = 32 after it, and an op
    that reads the first op's output two segments later (complete through
    the waits of the segments between). Every waiting op bit-identical to the
    single-op GEMV on the chain's own upstream output, twice in a row (the
    segment counters are left zeroed for the next launch)."""
    m = 3
    specs = [(4096, 4096, None), (32, 4096, 0), (4096, 32, 1), (2048, 4096, 0), (17, 2048, 3)]  # (n, k, x from op)
    x0h = synth.synth_x(m, 4096, 91)
    x0 = to_dev_u16(x0h)
    ws, ys, qs = [], [], []
    for i, (n, k, _) in enumerate(specs):
        q, s, _ = _op_inputs(n, k, 1, 970 + i)
        qs.append((q, s))
        ws.append(import_planes(dev, q, s))
        ys.append(torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda"))
    ops = []
    for i, (w, y, (_, _, src)) in enumerate(zip(ws, ys, specs)):
        xp = x0.data_ptr() if src is None else ys[src].data_ptr()
        ops.append((w, xp, y.data_ptr(), m, 0, 0 if i == 0 else 1))
    chain = hal.Chain(dev, ops)
    for rep in range(2):
        for y in ys:
            y.fill_(float("nan"))
        chain.run()
        torch.cuda.synchronize()
        rows = _oracle_rows(specs[0][0])
        q, s = qs[0]
        assert_parity(from_dev_bf16(ys[0])[:, rows], O.gemv_q(q[rows], s[rows], x0h), f"rep {rep} op 0")
        for i in range(1, len(specs)):
            ref = _raw(ws[i], ys[specs[i][2]], m, specs[i][0], False)
            assert torch.equal(_bits(ys[i]), _bits(ref)), (rep, i)
    assert dev.fault() == 0
    chain.destroy()


def test_chain_decode_set(dev):
    """Four layers of the 8B decode set (qkv, o, gateup, down) with fixed
    activations, every op after the previous (the decode step's order): the
    gateups bit-identical to the single-op fp16 path, the rest against the
    oracle."""
    shapes = [(6144, 4096), (4096, 4096), (28672, 4096), (4096, 14336)]
    xh = {k: synth.synth_x(1, k, 60 + k % 7) for k in (4096, 14336)}
    xs = {k: to_dev_u16(v) for k, v in xh.items()}
    ops, outs, refs = [], [], []
    for layer in range(4):
        for j, (n, k) in enumerate(shapes):
            q, s, _ = _op_inputs(n, k, 1, 1000 + 4 * layer + j)
            w = import_planes(dev, q, s)
            y = torch.empty((1, n), dtype=torch.bfloat16, device="cuda")
            ops.append((w, xs[k].data_ptr(), y.data_ptr(), 1, 0, 1))
            outs.append(y)
            if j == 2:
                refs.append(("raw", None, _raw(w, xs[k], 1, n, False)))
            else:
                rows = np.unique(np.concatenate([np.arange(256), np.arange(n - 256, n)]))
                refs.append(("oracle", rows, O.gemv_q(q[rows], s[rows], xh[k])))
    chain = hal.Chain(dev, ops)
    chain.run()
    torch.cuda.synchronize()
    for i, (y, (kind, rows, r)) in enumerate(zip(outs, refs)):
        if kind == "raw":
            assert torch.equal(_bits(y), _bits(r)), i
        else:
            assert_parity(from_dev_bf16(y)[:, rows], r, f"chain op {i}")
    assert dev.fault() == 0
    chain.destroy()


def test_chain_rejects_bad_ops(dev):
    q, s, x = _op_inputs(64, 64, 1, 5)
    w = import_planes(dev, q, s)
    xd = to_dev_u16(x)
    y = torch.empty((9, 64), dtype=torch.bfloat16, device="cuda")
    for op in [(w, xd.data_ptr(), y.data_ptr(), 9, 0, 0),        # m > 8
               (w, xd.data_ptr() + 2, y.data_ptr(), 1, 0, 0),    # x not 16-byte aligned
               (w, xd.data_ptr(), y.data_ptr() + 2, 1, 1, 0),    # f32 y not 4-byte aligned
               (w, xd.data_ptr(), y.data_ptr(), 1, 7, 0)]:       # unknown out_dtype
        with pytest.raises(hal.Xq4Error):
            hal.Chain(dev, [op])
    h = ctypes.c_void_p()
    assert lib().xq4_chain_create(dev.handle, None, 0, ctypes.byref(h)) != 0


def test_chain_refused_when_its_grid_cannot_be_resident():
    """The chain's CTAs wait for one another, so chain create refuses a device
    that cannot hold its whole grid at once: emulated with the diagnostic
    override of the occupancy figure (one CTA per SM), in a child process."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    code = (
        "import sys, torch, numpy as np\n"
        f"sys.path.insert(0, {str(root)!r})\n"
        "from xnpu_b200 import hal, synth, _lib\n"
        "dev = hal.Device.open(0)\n"
        "src = synth.planes_bytes(synth.synth_codes(256, 4096, 5), synth.synth_scales(256, 4096, 5))\n"
        "w = hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, 256, 4096))\n"
        "x = torch.zeros((1, 4096), dtype=torch.bfloat16, device='cuda')\n"
        "y = torch.zeros((1, 256), dtype=torch.bfloat16, device='cuda')\n"
        "try:\n"
        "    hal.Chain(dev, [(w, x.data_ptr(), y.data_ptr(), 1, 0, 0)])\n"
        "    print('created')\n"
        "except _lib.Xq4Error as e:\n"
        "    print('status', e.status)\n"
    )
    env = dict(os.environ, XQ4_RESIDENT_CTAS_PER_SM="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert f"status {6}" in r.stdout, r.stdout  # XQ4_ENOTSUP
    env["XQ4_RESIDENT_CTAS_PER_SM"] = ""  # the real occupancy: two CTAs per SM fit
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert "created" in r.stdout, (r.stdout, r.stderr[-2000:])
