"""Benchmark of the B200 int4 (Q4NX / w4) decode path.

Workload (one step = one token): the Llama-3-8B-shaped decode linear set at
batch 1 -- 32 layers x {QKV 4096->6144, O 4096->4096, gate+up 4096->2x14336,
down 14336->4096} -- with independent seeded random int4 weights per layer (group 32, bf16 scales |N(0,0.02)|/7.5, zero point 8) and
bf16 N(0,1) activations; each projection reads a fixed activation, as the
reference's projection-stream benchmark does (crates/xnpu-cli/src/main.rs:
2487-2499, :3288).  3.93 GB of weights per step, far above the 126 MB L2, so
no flush is needed between steps.

Gate and up are one fused "gateup" projection, as in the reference's own
layer chain (crates/xnpu-cli/src/main.rs:2464, :2488: 4 GEMV shapes per
layer, qkv / o / gateup / down); the weight bytes are those of the two.

On one GPU the step is ONE launch of the GEMV chain kernel over the 128
projections (xq4_chain_run, after a small kernel that prepares the fp16
activation images; the ops are independent because each reads its fixed
activation).  The same chain with every op waiting for the previous
one (a real decode step's dependency order) and the 128 separate GEMV
launches (one CUDA graph) are timed beside it (``other_step_forms_ms``).

On N GPUs (torchrun, one process per GPU) the FFN gateup projection is
column-sharded N ways, with the all-gather inside the GEMV kernel over NVLink
peer memory (xq4_linear_sharded_fused); QKV, O and down are replicated; the
step is the 128 launches in one CUDA graph.  The step is the same token, so
scaling is "strong".  The line also reports the lm_head 4096->128256 (f32 logits)
sharded the same way.

Metric: tokens/s (higher is better); GB/s of algorithmic bytes (packed codes
+ scales + x + y) and its fraction of the measured HBM peak are in
``roofline``.  ``--impl reference`` times the reference's CPU path (the C
restatement in oracle/, all host threads) on a bounded row sample.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS = 32
SHAPES = [("qkv", 6144, 4096), ("o", 4096, 4096), ("gateup", 28672, 4096), ("down", 4096, 14336)]
SHARDED = ("gateup",)  # column-sharded over ranks; the rest are replicas
# DRAM bytes (read + write) per launch of each projection at one GPU, from
#   ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
#       --clock-control none -k regex:gemv --csv python bench.py --layers 4 --steps 1
#       --warmup 3 --skip-e2e --skip-lmhead --no-cpu-baseline
# (every launch of the capture; the figures repeat to within 0.01 %).
DRAM_PER_LAUNCH = {"qkv": 14231808, "o": 9512960, "gateup": 66216960, "down": 33126912}
# DRAM bytes (read + write) of one chain launch (the whole 32-layer step), from
#   ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
#       --clock-control none -k regex:gemv_chain --csv python bench.py --layers 4
#       --steps 1 --warmup 3 --skip-e2e --skip-lmhead --no-cpu-baseline
# (a 4-layer chain; its bytes scaled by 8 = the ratio of algorithmic bytes).
CHAIN_DRAM_PER_STEP = 3929139200
LMHEAD = (128256, 4096)


def algo_bytes(n, k, m=1, out_bytes=2):
    return n * k // 2 + n * (k // 32) * 2 + m * k * 2 + m * n * out_bytes


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event (throttle) reasons polled through NVML from a
    host thread every ~2 ms while the timed region runs (read-only queries)."""

    REASONS = {  # NVML clocks-event reason bits
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4,
    }

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.err = None
        self._stop = threading.Event()

    def _poll(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            while not self._stop.is_set():
                mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((mhz, bits))
                time.sleep(0.002)
        except Exception as e:  # NVML missing: report it, do not fail the bench
            self.err = f"{type(e).__name__}: {e}"

    def __enter__(self):
        self._t = threading.Thread(target=self._poll, daemon=True)
        self._t.start()
        time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"]}
        reasons = sorted({n for _, b in self.rows for n, bit in self.REASONS.items() if b & bit})
        return {"sm_mhz": float(np.median([r[0] for r in self.rows])), "sm_max_mhz": float(self.max_mhz),
                "reasons": reasons, "samples": len(self.rows), "source": "NVML, 2 ms polling"}


# ---------------------------------------------------------------- CPU baseline
def cpu_baseline(steps=1, budget_s=12.0):
    """The reference's CPU path (oracle restatement of main.rs:2287-2296 over
    the L1 layout, rows split over all host threads) on a row sample of one
    layer's four projections; scaled to tokens/s of the 32-layer set."""
    from oracle import oracle as O
    from xnpu_b200 import synth
    threads = os.cpu_count() or 1
    frac = 1.0 / 16  # rows sampled per projection
    samples = []
    for name, n, k in SHAPES:
        rows = max(128, int(n * frac) // 128 * 128)
        q = synth.unpack_codes_signed(synth.synth_codes(rows, k, 7))
        s = synth.synth_scales(rows, k, 7)
        tsi = 4 if name == "down" else 16
        pack = O.l1_pack(q, s, tsi=tsi)
        x = synth.synth_x(1, k, 7)
        samples.append((n, k, rows, tsi, pack, x))
    t_layer = []
    t_end = time.time() + budget_s
    for _ in range(max(1, steps)):
        t = 0.0
        for n, k, rows, tsi, pack, x in samples:
            t0 = time.perf_counter()
            O.gemv_l1(pack, rows, k, tsi, x, nthreads=threads)
            t += (time.perf_counter() - t0) * (n / rows)
        t_layer.append(t)
        if time.time() > t_end:
            break
    tok_s = 1.0 / (np.median(t_layer) * LAYERS)
    return {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"1/16 of the rows of each of the 4 projections of one layer (L1 layout, sequential "
                      f"f32 per row), {len(t_layer)} timed pass(es), scaled to 32 layers",
            "gbs": sum(algo_bytes(n, k) for _, n, k in SHAPES) * LAYERS * tok_s / 1e9}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as O  # noqa: F401  (builds the oracle if needed)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(steps=1, budget_s=30.0)
        if i >= args.warmup:
            vals.append(r["value"])
    v = float(np.median(vals))
    line = {"metric": "decode tok/s, 8B-shaped int4 linear set (32 layers, batch 1)", "value": v,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 / v, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights, bf16 x, f32 accumulate", "data": "synthetic (seeded)",
            "impl": "reference",
            "config": {"workload": "llama3-8b decode linear set, 32 layers x (qkv 4096x6144, o 4096x4096, "
                                   "gateup 4096x28672, down 14336x4096), M=1", "group": 32},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": r["cores"], "kind": r["kind"],
                             "sample": r["sample"]},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def make_weights(dev, rank, world, seed_base=1):
    """All 32 layers' weights; gateup rows sharded over ranks."""
    from concurrent.futures import ThreadPoolExecutor
    from xnpu_b200 import hal, synth

    def one(li, si):
        name, n, k = SHAPES[si]
        seed = seed_base + 1000 * li + si
        codes = synth.synth_codes(n, k, seed)
        scales = synth.synth_scales(n, k, seed)
        src = synth.planes_bytes(codes, scales)
        r0, r1 = 0, 0
        if world > 1 and name in SHARDED:
            r0, r1 = rank * n // world, (rank + 1) * n // world
        return hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=r0, row_end=r1), src

    weights = []
    with ThreadPoolExecutor(max_workers=4) as ex:
        for li in range(LAYERS):
            futs = [ex.submit(one, li, si) for si in range(len(SHAPES))]
            layer = {}
            for si, f in enumerate(futs):
                desc, src = f.result()
                layer[SHAPES[si][0]] = hal.Weight.import_(dev, src, desc)
                del src
            weights.append(layer)
    return weights


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="xq4", choices=["xq4", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=32,
                    help="layers of the weight set (32 = the benchmark; fewer only for profiler captures)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiler captures only")
    ap.add_argument("--skip-lmhead", action="store_true", help="profiler captures only")
    ap.add_argument("--kernel-case", choices=["gemv", "gemm", "w4a8"],
                    help="profiler captures: one projection launched warmup+steps times on GPU 0 "
                         "(gemv and w4a8: 65536x4096 at m=1, 151 MB of weights; gemm: 14336x4096 at m=2048)")
    ap.add_argument("--case-m", type=int, default=None, help="token count of --kernel-case")
    args = ap.parse_args()
    if args.kernel_case:
        kernel_case(args)
        return
    global LAYERS
    LAYERS = args.layers

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from xnpu_b200 import hal, synth, lib
    from xnpu_b200._lib import check

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = hal.Device.open(local)
    meta = dev.metadata()
    L = lib()

    weights = make_weights(dev, rank, world)
    comm = None
    if world > 1:
        import ctypes
        uid = (ctypes.c_char * 128)()
        if rank == 0:
            check(L.xq4_comm_unique_id(ctypes.addressof(uid)))
        t = torch.frombuffer(bytearray(bytes(uid)), dtype=torch.uint8).cuda()
        dist.broadcast(t, 0)
        uid = (ctypes.c_char * 128).from_buffer_copy(t.cpu().numpy().tobytes())
        h = ctypes.c_void_p()
        check(L.xq4_comm_init(dev.handle, rank, world, ctypes.addressof(uid), ctypes.byref(h)))
        comm = h

    # activations / outputs (fixed per shape, as the reference's stream benchmark)
    xs = {k: torch.from_numpy(synth.synth_x(1, k, 11 + k).view(np.int16)).cuda().view(torch.bfloat16)
          for k in (4096, 14336)}
    ys = {name: torch.empty((1, n), dtype=torch.bfloat16, device="cuda") for name, n, _ in SHAPES}
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def step(st):
        launches = 0
        for layer in weights:
            for name, n, k in SHAPES:
                w = layer[name]
                if comm is not None and name in SHARDED:
                    check(L.xq4_linear_sharded_fused(comm, w.handle, xs[k].data_ptr(), ys[name].data_ptr(), 1, 0, st))
                else:
                    check(L.xq4_linear_raw(w.handle, xs[k].data_ptr(), ys[name].data_ptr(), 1, 0, st))
                launches += 1
        return launches

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(run_one, steps):
        """Device time per step (ms, max over ranks) of `steps` calls of
        run_one on `stream`, bracketed by barrier + synchronize."""
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        ev0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(steps):
                run_one()
        ev1.record(stream)
        barrier()
        t_ms = ev0.elapsed_time(ev1) / steps
        if world > 1:
            tt = torch.tensor([t_ms], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t_ms = float(tt.item())
        return t_ms

    # Separate launches: warm-up (eager), then one step captured into a CUDA
    # graph (128 launches per token are too many to issue from the host at
    # HBM speed).
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step(sp)
    barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        per_step = step(stream.cuda_stream)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    barrier()

    # One GPU: the step as ONE chain launch (xq4_chain_run).  Every
    # projection reads its fixed activation (the reference's projection-stream
    # benchmark, main.rs:2487-2499), so the ops are independent (wait_prev =
    # 0); the same chain with every op waiting for the previous one (the
    # dependency order of a real decode step) is timed beside it.
    chains = {}
    if world == 1:
        for wp in (0, 1):
            chains[wp] = hal.Chain(dev, [(layer[name], xs[k].data_ptr(), ys[name].data_ptr(), 1, 0, wp)
                                         for layer in weights for name, n, k in SHAPES])
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    chains[wp].run(stream)
        barrier()

    # device-timed steps (inputs resident in HBM)
    with ClockSampler(local) as clk:
        if world == 1:
            ms = timed(lambda: chains[0].run(stream), args.steps)
            per_step = 2  # the activation prep kernel + the chain kernel
        else:
            ms = timed(graph.replay, args.steps)
    clocks = clk.summary()
    launches = per_step * args.steps
    alt = {"separate_launches_graph_ms": timed(graph.replay, args.steps)}
    if world == 1:
        alt["chain_dependent_ms"] = timed(lambda: chains[1].run(stream), args.steps)
    for c in chains.values():
        c.destroy()

    # roofline: algorithmic bytes of the step's GEMVs (per GPU) over the
    # timed region's duration
    gpu_step_bytes = 0
    for name, n, k in SHAPES:
        ns = n // world if (world > 1 and name in SHARDED) else n
        gpu_step_bytes += algo_bytes(ns, k) * LAYERS
    achieved = gpu_step_bytes / (ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()

    # isolated single-launch durations per shape (events around each launch;
    # includes launch latency) -- diagnostic detail only
    per = {name: [] for name, _, _ in SHAPES}
    evs = []
    with torch.cuda.stream(stream):
        for layer in weights[:8]:
            for name, n, k in SHAPES:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                check(L.xq4_linear_raw(layer[name].handle, xs[k].data_ptr(), ys[name].data_ptr(), 1, 0, sp))
                b.record(stream)
                evs.append((name, a, b))
    torch.cuda.synchronize()
    for name, a, b in evs:
        per[name].append(a.elapsed_time(b))
    del graph

    # end-to-end through the C ABI with host buffers (pinned), copies inside
    e2e = None if args.skip_e2e else e2e_run(dev, weights, comm, world, args)

    # lm_head (sharded the same way), f32 logits
    lm = None if args.skip_lmhead else lmhead_run(dev, rank, world, comm, L, stream)

    # W4A8 parity mode (the reference's NPU numerics) on the same step, 1 GPU
    w4a8 = None if (args.skip_e2e or world > 1) else w4a8_run(weights, xs, stream, args)

    step_bytes = sum(algo_bytes(n, k) for _, n, k in SHAPES) * LAYERS
    if rank == 0:
        cpu = None if args.no_cpu_baseline or world > 1 else cpu_baseline()
        line = {
            "metric": "decode tok/s, 8B-shaped int4 linear set (32 layers, batch 1)",
            "value": 1e3 / ms, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights (u4 codes, bf16 scales), bf16 x, f32 accumulate",
            "data": "synthetic (seeded PCG64; random-init 8B-shaped weights)",
            "config": {"workload": "llama3-8b decode linear set, 32 layers x (qkv 4096x6144, o 4096x4096, "
                                   "gateup 4096x28672, down 14336x4096), M=1",
                       "group": 32, "layers": LAYERS, "batch": 1,
                       "parallelism": "single GPU" if world == 1 else f"gateup column-sharded x{world}, rows gathered by the GEMV over NVLink peer memory; qkv/o/down replicated",
                       "l2": "inputs 3.93 GB per step >> 126 MB L2 (no flush needed)"},
            "gbs": step_bytes * (1e3 / ms) / 1e9,
            "roofline": ({"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                          "frac": achieved / peak, "peak_kind": peak_kind,
                          "kernel": "gemv_chain_kernel (the step's 128 GEMVs in one launch, m=1)",
                          "traffic": (CHAIN_DRAM_PER_STEP * LAYERS / 32 if CHAIN_DRAM_PER_STEP else None),
                          "traffic_unit": "bytes per launch (ncu, 4-layer chain scaled by bytes to 32 layers)",
                          "algorithmic_bytes_per_launch": gpu_step_bytes,
                          "region": "one chain launch per step"}
                         if world == 1 else
                         {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                          "frac": achieved / peak, "peak_kind": peak_kind,
                          "kernel": "gemv_kernel<1> (decode GEMV, m=1)", "traffic": None,
                          "algorithmic_bytes_per_launch": gpu_step_bytes / LAYERS / len(SHAPES),
                          "region": "all GEMV launches of the timed steps (CUDA graph replays)"}),
            "isolated_launch_us": {k: 1e3 * float(np.mean(v)) for k, v in per.items()},
            "other_step_forms_ms": alt,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
            "lm_head": lm,
            "w4a8": w4a8,
            "device": meta["name"],
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if comm is not None:
        check(L.xq4_comm_destroy(comm))
    for layer in weights:
        for w in layer.values():
            w.destroy()
    dev.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def e2e_run(dev, weights, comm, world, args):
    """Same step through the public C ABI with host buffers: one pinned H2D of
    the step's activations, 128 xq4_linear submits on the device queue, one
    D2H of every output, xq4_wait -- timed on the host clock."""
    import ctypes
    import torch
    from xnpu_b200 import hal, lib, synth
    from xnpu_b200._lib import check
    L = lib()
    # per step inputs: one x per distinct K (the reference's benchmark feeds a
    # fixed activation per shape); outputs: every projection of every layer
    k_off = {4096: 0, 14336: 4096 * 2}
    x_bytes = (4096 + 14336) * 2
    y_sizes = [(li, name, n) for li in range(LAYERS) for name, n, _ in SHAPES]
    y_off, off = {}, 0
    for li, name, n in y_sizes:
        y_off[(li, name)] = off
        off += ((n * 2 + 255) // 256) * 256
    y_bytes = off
    xb = hal.BufferObject.new(dev, x_bytes)
    yb = hal.BufferObject.new(dev, y_bytes)
    hx = torch.empty(x_bytes, dtype=torch.uint8).pin_memory()
    hy = torch.empty(y_bytes, dtype=torch.uint8).pin_memory()
    hx.numpy()[:] = synth.synth_x(1, x_bytes // 2, 5).reshape(-1).view(np.uint8)
    seq = ctypes.c_uint64()

    chain = None
    if comm is None:  # one GPU: the step is one chain submit (ops independent, as the timed step)
        chain = hal.Chain(dev, [(layer[name], xb.device_ptr() + k_off[k], yb.device_ptr() + y_off[(li, name)],
                                 1, 0, 0) for li, layer in enumerate(weights) for name, n, k in SHAPES])

    def one():
        check(L.xq4_buffer_upload(xb.handle, hx.data_ptr(), 0, x_bytes))
        if chain is not None:
            chain.submit()
            check(L.xq4_wait(dev.handle, L.xq4_last_seq(dev.handle), 60_000_000_000))
            check(L.xq4_buffer_download(yb.handle, hy.data_ptr(), 0, y_bytes))
            return
        for li, layer in enumerate(weights):
            for name, n, k in SHAPES:
                if comm is not None and name in SHARDED:
                    xp = xb.device_ptr() + k_off[k]
                    yp = yb.device_ptr() + y_off[(li, name)]
                    check(L.xq4_linear_sharded_fused(comm, layer[name].handle, xp, yp, 1, 0,
                                                     dev.stream_handle()))
                else:
                    check(L.xq4_linear(dev.handle, layer[name].handle, xb.handle, k_off[k], yb.handle,
                                       y_off[(li, name)], 1, 0, ctypes.byref(seq)))
        check(L.xq4_wait(dev.handle, L.xq4_last_seq(dev.handle), 60_000_000_000))
        check(L.xq4_buffer_download(yb.handle, hy.data_ptr(), 0, y_bytes))

    import torch.distributed as dist
    for _ in range(max(1, args.warmup)):
        one()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = (time.perf_counter() - t0) / args.steps
    if world > 1:
        t = torch.tensor([dt], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    if chain is not None:
        chain.destroy()
    xb.destroy()
    yb.destroy()
    path = ("xq4_buffer_upload -> xq4_chain_submit (the step's 128 GEMVs) -> xq4_wait -> xq4_buffer_download "
            "(pinned host buffers)" if chain is not None else
            "xq4_buffer_upload -> 128 x xq4_linear (gateup: xq4_linear_sharded_fused) -> xq4_wait -> "
            "xq4_buffer_download (pinned host buffers)")
    return {"value": 1.0 / dt, "unit": "tok/s", "h2d_bytes_per_step": x_bytes, "d2h_bytes_per_step": y_bytes,
            "ms_per_step": dt * 1e3, "path": path}


def w4a8_run(weights, xs, stream, args):
    """The decode step in the W4A8 parity mode: per projection, quantize its
    activation (xq4_quantize_x) and run the int8-activation GEMV
    (xq4_linear_w4a8); CUDA-graph replays timed with events."""
    import torch
    from xnpu_b200 import lib
    from xnpu_b200._lib import check
    L = lib()
    sp = stream.cuda_stream
    qd = {k: (torch.empty((1, k), dtype=torch.int8, device="cuda"),
              torch.empty((1, k // 32), dtype=torch.int16, device="cuda")) for k in xs}
    ys = {name: torch.empty((1, n), dtype=torch.bfloat16, device="cuda") for name, n, _ in SHAPES}

    def step():
        for layer in weights:
            for name, n, k in SHAPES:
                q, d = qd[k]
                check(L.xq4_quantize_x(xs[k].data_ptr(), 1, k, q.data_ptr(), d.data_ptr(), 0, sp))
                check(L.xq4_linear_w4a8(layer[name].handle, q.data_ptr(), d.data_ptr(), ys[name].data_ptr(), 1, 0,
                                        sp))

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    del g
    step_bytes = sum(algo_bytes(n, k) for _, n, k in SHAPES) * LAYERS
    return {"tok_s": 1e3 / ms, "ms_per_step": ms, "gbs": step_bytes / (ms * 1e-3) / 1e9,
            "gpu_launches_per_step": 2 * len(SHAPES) * LAYERS,
            "path": "per projection: xq4_quantize_x + xq4_linear_w4a8 (int8 activations, bf16 2048-K partials)"}


def lmhead_run(dev, rank, world, comm, L, stream, reps=20):
    """lm_head 4096 -> 128256, f32 logits, rows sharded over ranks and
    gathered inside the GEMV over peer memory; 8 rotating weight copies
    (>2x L2 at every N)."""
    import torch
    import torch.distributed as dist
    from xnpu_b200 import hal, synth
    from xnpu_b200._lib import check
    n, k = LMHEAD
    r0, r1 = rank * n // world, (rank + 1) * n // world
    copies = 8 if world == 1 else max(8, 2 * world)
    codes = synth.synth_codes(n, k, 424242)
    scales = synth.synth_scales(n, k, 424242)
    src = synth.planes_bytes(codes, scales)
    ws = [hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=r0, row_end=r1))
          for _ in range(copies)]
    del src
    x = torch.from_numpy(synth.synth_x(1, k, 9).view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty((1, n), dtype=torch.float32, device="cuda")
    sp = stream.cuda_stream

    def go(i):
        if comm is not None:
            check(L.xq4_linear_sharded_fused(comm, ws[i % copies].handle, x.data_ptr(), y.data_ptr(), 1, 1, sp))
        else:
            check(L.xq4_linear_raw(ws[i % copies].handle, x.data_ptr(), y.data_ptr(), 1, 1, sp))

    with torch.cuda.stream(stream):
        for i in range(5):
            go(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    with torch.cuda.stream(stream):
        for i in range(reps):
            go(i)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    for w in ws:
        w.destroy()
    shard_bytes = algo_bytes(r1 - r0, k, out_bytes=4)
    return {"us": ms * 1e3, "shard_rows": r1 - r0, "gbs_per_gpu": shard_bytes / (ms * 1e-3) / 1e9,
            "logits_gather_bytes_in": (n - (r1 - r0)) * 4}


def kernel_case(args):
    """One projection launched warmup+steps times through the C ABI (the
    small, single-kernel command that profiler captures run on)."""
    import torch
    from xnpu_b200 import hal, lib, synth
    from xnpu_b200._lib import check
    n, k, m = (14336, 4096, 2048) if args.kernel_case == "gemm" else (65536, 4096, 1)
    m = args.case_m or m
    dev = hal.Device.open(0)
    L = lib()
    w = hal.Weight.import_(dev, synth.planes_bytes(synth.synth_codes(n, k, 31), synth.synth_scales(n, k, 31)),
                           hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k))
    x = torch.from_numpy(synth.synth_x(m, k, 32).view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.Stream()
    q = torch.empty((m, k), dtype=torch.int8, device="cuda")
    d = torch.empty((m, k // 32), dtype=torch.int16, device="cuda")

    def one():
        if args.kernel_case == "w4a8":
            check(L.xq4_quantize_x(x.data_ptr(), m, k, q.data_ptr(), d.data_ptr(), 0, stream.cuda_stream))
            check(L.xq4_linear_w4a8(w.handle, q.data_ptr(), d.data_ptr(), y.data_ptr(), m, 0, stream.cuda_stream))
        else:
            check(L.xq4_linear_raw(w.handle, x.data_ptr(), y.data_ptr(), m, 0, stream.cuda_stream))
    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        one()
    b.record(stream)
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / max(1, args.steps)
    print(json.dumps({"kernel_case": args.kernel_case, "n": n, "k": k, "m": m, "us_per_launch": us,
                      "algo_gbs": algo_bytes(n, k, m) / us / 1e3, "tflops": 2.0 * m * n * k / us / 1e6}),
          flush=True)
    w.destroy()
    dev.close()


if __name__ == "__main__":
    main()
