"""Column (N) sharded linear on two GPUs.

Two processes (one per GPU) import their row shard of one matrix, run the
shard's GEMV (m < 25) or GEMM (m >= 25), all-gather the slices with NCCL
(xq4_linear_sharded) and must both hold the full output, within the parity
bars of the single-GPU tests against the oracle over the full matrix.  The
same call without a workspace (xq4_linear_sharded_noalloc, its gather staged
in the library's fixed scratch array) must give the identical bits.  For
m < 16 the same call with the gather fused into the GEMV over peer memory
(xq4_linear_sharded_fused) must give the identical bits on both ranks, twice
in a row, with no fault bit raised.

A chain with column-sharded ops (a gate/up projection with its SwiGLU
epilogue, whose 1-per-pair intermediate is gathered; an f32 projection; a
replicated op; and an op that waits for the gathered intermediate and reads
it) must give, on both ranks and in two runs, the bits of the same chain run
unsharded on the full weights.

A fused call that only one rank makes must end after the kernel's bounded
wait with fault bit 0x8, leaving the context usable; the communicator is
then unusable on both ranks: the rank that gave up refuses its next call,
and the peer's next call exchanges nothing, raises fault bit 0x8 and is then
refused too.  Skipped with fewer than two GPUs.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, id_q, res_q):
    import ctypes
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    from oracle import oracle as O
    from xnpu_b200 import _lib, hal, lib, synth
    from xnpu_b200._lib import check
    from test_gpu_kernels import rel_metrics

    torch.cuda.set_device(rank)
    L = lib()
    dev = hal.Device.open(rank)
    uid = (ctypes.c_char * 128)()
    if rank == 0:
        check(L.xq4_comm_unique_id(ctypes.addressof(uid)))
        for _ in range(world - 1):
            id_q.put(bytes(uid))
    else:
        uid = (ctypes.c_char * 128).from_buffer_copy(id_q.get(timeout=60))
    comm = ctypes.c_void_p()
    check(L.xq4_comm_init(dev.handle, rank, world, ctypes.addressof(uid), ctypes.byref(comm)))
    out = {}
    try:
        n, k = 4096, 4096
        q = synth.unpack_codes_signed(synth.synth_codes(n, k, 55))
        s = synth.synth_scales(n, k, 55)
        ns = n // world
        src = synth.planes_bytes(synth.pack_codes_signed(q), s)
        w = hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=rank * ns,
                                                          row_end=(rank + 1) * ns))
        rows = np.arange(0, n, 7)
        for m, f32 in ((1, 0), (1, 1), (3, 0), (20, 0), (40, 0)):
            x = synth.synth_x(m, k, 56 + m)
            xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
            yd = torch.empty((m, n), dtype=torch.float32 if f32 else torch.bfloat16, device="cuda")
            ws = torch.empty((m, n), dtype=yd.dtype, device="cuda")
            st = torch.cuda.current_stream().cuda_stream
            check(L.xq4_linear_sharded(comm, w.handle, xd.data_ptr(), yd.data_ptr(), ws.data_ptr(), m, f32, st))
            torch.cuda.synchronize()
            got = yd.float().cpu().numpy()[:, rows]
            if m < 25:  # the GEMV path (unrounded weights); the GEMM from m = 25
                ref = O.gemv_q(q[rows], s[rows], x)
            else:
                ref = O.gemv_bf16(O.dequant_planes(q[rows], s[rows]), x)
            if not f32:
                ref = synth.bf16_bits_to_f32(O.round_bf16(ref))
            max_rel, mae, _ = rel_metrics(got, ref)
            out[(m, f32)] = (max_rel, mae)
            # no workspace: the gather stages through the library's scratch array
            yn = torch.full((m, n), float("nan"), dtype=yd.dtype, device="cuda")
            check(L.xq4_linear_sharded_noalloc(comm, w.handle, xd.data_ptr(), yn.data_ptr(), m, f32, st))
            torch.cuda.synchronize()
            iv = torch.int32 if f32 else torch.int16
            out[("noalloc", m, f32)] = bool(torch.equal(yn.view(iv), yd.view(iv)))
            if m < 16:
                # the same call with the gather fused into the GEMV over peer
                # memory: identical bits on every rank, twice in a row (the
                # two inbox halves)
                for rep in range(2):
                    yf = torch.full((m, n), float("nan"), dtype=yd.dtype, device="cuda")
                    check(L.xq4_linear_sharded_fused(comm, w.handle, xd.data_ptr(), yf.data_ptr(), m, f32, st))
                    torch.cuda.synchronize()
                    iv = torch.int32 if f32 else torch.int16
                    out[("fused", m, f32, rep)] = bool(torch.equal(yf.view(iv), yd.view(iv)))
                bits = ctypes.c_uint32()
                check(L.xq4_device_fault(dev.handle, ctypes.byref(bits)))
                out[("fault", m, f32)] = bits.value
        out.update(_sharded_chain(dev, comm, rank, world, L))
        # a peer that never makes the call: this rank's kernel gives up after
        # its bounded wait (about 2 s), reports fault bit 0x8 and the context
        # stays usable
        if rank == 0:
            x = synth.synth_x(1, k, 57)
            xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
            yf = torch.empty((1, n), dtype=torch.bfloat16, device="cuda")
            check(L.xq4_linear_sharded_fused(comm, w.handle, xd.data_ptr(), yf.data_ptr(), 1, 0, st))
            torch.cuda.synchronize()
            bits = ctypes.c_uint32()
            check(L.xq4_device_fault(dev.handle, ctypes.byref(bits)))
            out[("lone_fault",)] = bits.value
            yl = torch.empty((1, ns), dtype=torch.bfloat16, device="cuda")
            check(L.xq4_linear_raw(w.handle, xd.data_ptr(), yl.data_ptr(), 1, 0, st))
            torch.cuda.synchronize()
            out[("lone_after",)] = bool(torch.equal(yl.view(torch.int16), yf[:, :ns].view(torch.int16)))
            id_q.put("lone done")
        else:
            assert id_q.get(timeout=120) == "lone done"
        # the communicator is unusable from now on, on both ranks
        x = synth.synth_x(1, k, 58)
        xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
        yf = torch.full((1, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = L.xq4_linear_sharded_fused(comm, w.handle, xd.data_ptr(), yf.data_ptr(), 1, 0, st)
        torch.cuda.synchronize()
        bits = ctypes.c_uint32()
        check(L.xq4_device_fault(dev.handle, ctypes.byref(bits)))
        rc2 = L.xq4_linear_sharded_fused(comm, w.handle, xd.data_ptr(), yf.data_ptr(), 1, 0, st)
        torch.cuda.synchronize()
        if rank == 0:  # it gave up itself: refused on the host
            out[("poisoned",)] = rc == _lib.XQ4_ETIMEDOUT and rc2 == _lib.XQ4_ETIMEDOUT
        else:  # its peer poisoned it: the kernel exchanges nothing and flags it, then refused
            out[("poisoned",)] = rc == 0 and bits.value == 0x8 and rc2 == _lib.XQ4_ETIMEDOUT
        out[("poisoned_detail",)] = (rc, bits.value, rc2)
        w.destroy()
        res_q.put((rank, "ok", out))
    except Exception as e:
        res_q.put((rank, "error", repr(e)))
        raise
    finally:
        L.xq4_comm_destroy(comm)
        dev.close()


def _sharded_chain(dev, comm, rank, world, L):
    """A chain with column-sharded ops against the same chain unsharded."""
    import ctypes
    from xnpu_b200 import hal, synth
    from xnpu_b200._lib import check

    def imp(n, k, seed, r0=0, r1=0):
        src = synth.planes_bytes(synth.synth_codes(n, k, seed), synth.synth_scales(n, k, seed))
        return hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=r0, row_end=r1))

    k, ng, nl, nr, nd = 4096, 8192, 8192, 1024, 1024  # gate/up (interleaved) rows, f32 op rows, replicated, down
    shard = lambda n: (rank * n // world, (rank + 1) * n // world)  # noqa: E731
    wg_s, wg_f = imp(ng, k, 71, *shard(ng)), imp(ng, k, 71)
    wl_s, wl_f = imp(nl, k, 72, *shard(nl)), imp(nl, k, 72)
    wr = imp(nr, k, 73)
    wd = imp(nd, ng // 2, 74)  # reads the gathered SwiGLU intermediate
    x = torch.from_numpy(synth.synth_x(1, k, 75).view(np.int16)).cuda().view(torch.bfloat16)

    def outputs():
        return (torch.full((1, ng // 2), float("nan"), dtype=torch.bfloat16, device="cuda"),
                torch.full((1, nl), float("nan"), dtype=torch.float32, device="cuda"),
                torch.full((1, nr), float("nan"), dtype=torch.bfloat16, device="cuda"),
                torch.full((1, nd), float("nan"), dtype=torch.bfloat16, device="cuda"))

    def ops(ys, sharded):
        c = comm if sharded else None
        return [(wg_s if sharded else wg_f, x.data_ptr(), ys[0].data_ptr(), 1, 0, 0, c, {"swiglu": True}),
                (wl_s if sharded else wl_f, x.data_ptr(), ys[1].data_ptr(), 1, 1, 0, c),
                (wr, x.data_ptr(), ys[2].data_ptr(), 1, 0, 0),
                (wd, ys[0].data_ptr(), ys[3].data_ptr(), 1, 0, 1)]

    ref = outputs()
    full = hal.Chain(dev, ops(ref, False))
    full.run()
    torch.cuda.synchronize()
    got = outputs()
    sh = hal.Chain(dev, ops(got, True))
    res = {}
    for rep in range(2):  # both inbox halves
        for t in got:
            t.fill_(float("nan"))
        sh.run()
        torch.cuda.synchronize()
        for i, (a, b) in enumerate(zip(got, ref)):
            iv = torch.int32 if a.dtype == torch.float32 else torch.int16
            res[("chain", i, rep)] = bool(torch.equal(a.view(iv), b.view(iv)))
    bits = ctypes.c_uint32()
    check(L.xq4_device_fault(dev.handle, ctypes.byref(bits)))
    res[("fault", "chain")] = bits.value
    sh.destroy()
    full.destroy()
    for w in (wg_s, wg_f, wl_s, wl_f, wr, wd):
        w.destroy()
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_linear_sharded_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    id_q, res_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, id_q, res_q)) for r in range(2)]
    for p in procs:
        p.start()
    # Read the results before joining: a child cannot exit while its queued
    # result is still in the pipe, and a child killed in the middle of a put
    # leaves a message the reader would wait on forever.  The results stay
    # small (flags and metrics, no output arrays).
    results, deadline = [], time.monotonic() + 300
    try:
        for _ in range(2):
            results.append(res_q.get(timeout=max(1.0, deadline - time.monotonic())))
    finally:
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    assert all(p.exitcode == 0 for p in procs), (results, [p.exitcode for p in procs])
    for rank, status, out in results:
        assert status == "ok", (rank, out)
        for key, val in out.items():
            if key[0] in ("fused", "lone_after", "noalloc", "chain", "poisoned"):
                assert val, (rank, key, "differs from the reference path", out.get(("poisoned_detail",)))
            elif key[0] == "poisoned_detail":
                continue
            elif key[0] == "fault":
                assert val == 0, (rank, key, val)
            elif key[0] == "lone_fault":
                assert val == 0x8, (rank, key, val)
            else:
                max_rel, mae = val
                assert max_rel <= 1e-2 and mae <= 1e-3, (rank, key, max_rel, mae)
