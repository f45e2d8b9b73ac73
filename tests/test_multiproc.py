"""Host-side logic of the column (N) sharded path, on CPU with gloo ranks.

Each of two ranks imports only its row shard of the matrix through the C ABI
repacker (xq4_repack_host with row_begin/row_end, no GPU), decodes the GPU
image with the independent numpy decoder, computes its output slice with the
oracle GEMV (main.rs:2287-2296) and all-gathers the slices; the gathered
output must equal the oracle over the full matrix bit for bit, and the
m > 1 gather order ([rank][token][row] -> [token][rank*ns + row], the
permutation xq4_linear_sharded applies after its all-gather) must reassemble
the full [m][n] output.
"""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, result_q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from xnpu_b200 import hal, synth
    import xq4g_ref

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k, m = 512, 1024, 3
        q = synth.unpack_codes_signed(synth.synth_codes(n, k, 77))
        s = synth.synth_scales(n, k, 77)
        x = synth.synth_x(m, k, 78)
        ns = n // world
        r0, r1 = rank * ns, (rank + 1) * ns
        src = synth.planes_bytes(synth.pack_codes_signed(q), s)
        desc = hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=r0, row_end=r1)
        img = hal.repack_host(src, desc)
        qs, ss, _, _ = xq4g_ref.decode(img, ns, k)
        local = O.gemv_q(qs, ss, x)  # [m][ns]
        # m == 1: rank slices concatenate along N
        parts = [torch.zeros(ns, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(local[0])))
        y1 = torch.cat(parts).numpy()
        # m > 1: gathered buffer is [rank][token][row]; permute to [token][rank*ns + row]
        partsm = [torch.zeros(m * ns, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(partsm, torch.from_numpy(np.ascontiguousarray(local).reshape(-1)))
        ws = torch.cat(partsm).numpy().reshape(world, m, ns)
        ym = ws.transpose(1, 0, 2).reshape(m, world * ns)
        if rank == 0:
            full = O.gemv_q(q, s, x)
            result_q.put(("ok", bool(np.array_equal(y1, full[0])), bool(np.array_equal(ym, full)),
                          bool(np.array_equal(qs, q[r0:r1])) and bool(np.array_equal(ss, s[r0:r1]))))
    except Exception as e:  # report instead of hanging the other rank
        result_q.put(("error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_sharded_gather_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = q.get(timeout=5)
    assert res[0] == "ok", res
    _, y1_ok, ym_ok, shard_ok = res
    assert shard_ok, "row-shard import does not hold the shard's codes/scales"
    assert y1_ok, "m == 1 all-gather differs from the full-matrix oracle"
    assert ym_ok, "m > 1 gather permutation differs from the full-matrix oracle"
