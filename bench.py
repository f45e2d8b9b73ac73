"""Benchmark of the B200 int4 (Q4NX / w4) decode path.

Workload (one step = one token): the Llama-3-8B-shaped decode linear set at
batch 1 -- 32 layers x {QKV 4096->6144, O 4096->4096, gate+up 4096->2x14336,
down 14336->4096} -- with independent seeded random int4 weights per layer
(group 32, bf16 scales |N(0,0.02)|/7.5, zero point 8) and bf16 N(0,1)
activations; each projection reads a fixed activation, as the reference's
projection-stream benchmark does (crates/xnpu-cli/src/main.rs:2487-2499,
:3288).  3.93 GB of weights per step, far above the 126 MB L2, so no flush is
needed between steps.

Gate and up are one fused "gateup" projection, as in the reference's own
layer chain (crates/xnpu-cli/src/main.rs:2464, :2488: 4 GEMV shapes per
layer, qkv / o / gateup / down); the weight bytes are those of the two, and
its SwiGLU (the FFN's next step, main.rs:4732-4745) is fused into its
epilogue, so it writes the 14336-value intermediate.

The step is ONE launch of the GEMV chain kernel over the 128 projections
(xq4_chain_run, after a small kernel that prepares the fp16 activation
images).  On N GPUs (torchrun, one process per GPU) the gate/up projection is
column-sharded N ways and each rank's SwiGLU values reach the peers inside
the chain kernel over NVLink peer memory; QKV, O and down are replicated.
The token is the same at every N, so scaling is "strong".  The same chain
with every op waiting for the previous one (a real decode step's dependency
order) is timed beside it, and at N = 1 the 128 GEMVs as separate launches in
one CUDA graph.

Also reported: the lm_head 4096->128256 (f32 logits, sharded the same way),
config 0 (one 4096x4096 GEMV over rotating copies), config 2 (the gate
projection at m = 1..64), config 3 (prefill GEMM, m = 2048), the W4A8 parity
mode, and the reference's CPU path timed in full on this host
(``cpu_baseline``).  ``--impl reference`` times that CPU path as the
reference arm, one whole token per step.
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
SHARDED = ("gateup",)  # column-sharded over ranks, its SwiGLU intermediate gathered; the rest are replicas
# DRAM bytes (read + write) per layer of one chain launch, from
#   ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
#       --clock-control none -k regex:gemv_chain --csv python bench.py --layers 4
#       --steps 1 --warmup 3 --skip-e2e --skip-lmhead --skip-configs --no-cpu-baseline
# (a 4-layer chain's steady-state bytes, 492,145,408, / 4; every layer has the
# same shapes).
CHAIN_DRAM_PER_LAYER = 492145408 // 4
LMHEAD = (128256, 4096)
METRIC = "decode tok/s, 8B-shaped int4 linear set (32 layers, batch 1)"
DTYPE = "int4 weights (u4 codes, bf16 scales), bf16 x, f32 accumulate"
DATA = "synthetic (seeded PCG64; random-init 8B-shaped weights)"


def config_of(world):
    return {"workload": "llama3-8b decode linear set, 32 layers x (qkv 4096x6144, o 4096x4096, "
                        "gateup 4096x28672 with its SwiGLU epilogue, down 14336x4096), M=1",
            "group": 32, "layers": LAYERS, "batch": 1,
            "parallelism": ("single GPU" if world == 1 else
                            f"gate/up column-sharded x{world}, SwiGLU intermediate gathered inside the chain "
                            f"kernel over NVLink peer memory; qkv/o/down replicated"),
            "l2": "inputs 3.93 GB per step >> 126 MB L2 (no flush needed)"}


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
        self._ready = threading.Event()

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
                self._ready.set()
                time.sleep(0.002)
        except Exception as e:  # NVML missing: report it, do not fail the bench
            self.err = f"{type(e).__name__}: {e}"
        finally:
            self._ready.set()

    def __enter__(self):
        # NVML's initialisation (~0.1 s) finishes before the timed region:
        # inside it, it held up the launching thread between the events
        self._t = threading.Thread(target=self._poll, daemon=True)
        self._t.start()
        self._ready.wait(10.0)
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
def layer_seed(li, si):
    return 1 + 1000 * li + si


def l1_image(codes, scales, tsi):
    """The reference's L1 tile layout (tools/w4_import.py:4-14,
    crates/xnpu-cli/src/main.rs:2186-2252) of a weight given as packed code
    and scale planes: rows run through the 8 columns in order, so the image
    is, tile by tile (tsi consecutive rows), the tile's nibble rows then its
    bf16 scale rows."""
    n = codes.shape[0]
    c = codes.reshape(n // tsi, -1)
    sc = np.ascontiguousarray(scales.astype("<u2")).view(np.uint8).reshape(n // tsi, -1)
    return np.concatenate([c, sc], axis=1).reshape(-1)


def cpu_layers(layers, seed_base=1):
    """Every layer's four projections in the L1 layout (the reference's CPU
    path reads that layout), the same seeded weights as the GPU arm."""
    from concurrent.futures import ThreadPoolExecutor
    from xnpu_b200 import synth

    def one(li, si):
        name, n, k = SHAPES[si]
        seed = layer_seed(li, si) if seed_base == 1 else seed_base + 1000 * li + si
        tsi = 4 if name == "down" else 16  # crates/xnpu-cli/src/main.rs:2461-2466
        return (n, k, tsi, l1_image(synth.synth_codes(n, k, seed), synth.synth_scales(n, k, seed), tsi))

    with ThreadPoolExecutor(max_workers=4) as ex:
        futs = [[ex.submit(one, li, si) for si in range(len(SHAPES))] for li in range(layers)]
        return [[f.result() for f in row] for row in futs]


def cpu_token(O, layers, xs, threads):
    """One full token of the reference's CPU path: every row of every
    projection of every layer, the oracle restatement of the sequential-f32
    GEMV of crates/xnpu-cli/src/main.rs:2287-2296 over the L1 layout, rows
    split over `threads` host threads.  Returns seconds."""
    t0 = time.perf_counter()
    for layer in layers:
        for n, k, tsi, pack in layer:
            O.gemv_l1(pack, n, k, tsi, xs[k], nthreads=threads)
    return time.perf_counter() - t0


def cpu_baseline(layers=None, tokens=3):
    """The reference's CPU path timed in full on this host's cores: `tokens`
    whole tokens (all rows of all 32 layers each), median."""
    from oracle import oracle as O
    from xnpu_b200 import synth
    threads = os.cpu_count() or 1
    layers = layers or cpu_layers(LAYERS)
    xs = {k: synth.synth_x(1, k, 11 + k) for k in (4096, 14336)}
    cpu_token(O, layers[:1], xs, threads)  # warm-up: page the first layer in
    ts = [cpu_token(O, layers, xs, threads) for _ in range(tokens)]
    t = float(np.median(ts))
    return {"value": 1.0 / t, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{tokens} whole tokens (every row of the 4 projections of all {len(layers)} layers, L1 "
                      f"layout, sequential f32 per row, rows split over {threads} threads), median; no extrapolation",
            "gbs": sum(algo_bytes(n, k) for _, n, k in SHAPES) * len(layers) / t / 1e9,
            "seconds_per_token": t}


def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path (the oracle port:
    the reference's CPU code is Rust, which this image cannot build), on the
    same workload, one whole token per step, all host threads; rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as O
    from xnpu_b200 import synth
    threads = os.cpu_count() or 1
    layers = cpu_layers(LAYERS)
    xs = {k: synth.synth_x(1, k, 11 + k) for k in (4096, 14336)}
    for _ in range(args.warmup):
        cpu_token(O, layers, xs, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_token(O, layers, xs, threads)
    t = (time.perf_counter() - t0) / args.steps
    v = 1.0 / t
    sample = (f"whole tokens: every row of qkv/o/gateup/down of all {LAYERS} layers per step (L1 layout, "
              f"sequential f32 per row, rows split over {threads} threads); no extrapolation")
    line = {"metric": METRIC, "value": v,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * t, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": DTYPE, "data": DATA, "impl": "reference", "config": config_of(world),
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def make_weights(dev, rank, world, layers, seed_base=1):
    """All layers' weights; the gate/up projection's rows sharded over ranks."""
    from concurrent.futures import ThreadPoolExecutor
    from xnpu_b200 import hal, synth

    def one(li, si):
        name, n, k = SHAPES[si]
        seed = seed_base + 1000 * li + si
        src = synth.planes_bytes(synth.synth_codes(n, k, seed), synth.synth_scales(n, k, seed))
        r0, r1 = 0, 0
        if world > 1 and name in SHARDED:
            r0, r1 = rank * n // world, (rank + 1) * n // world
        return hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=r0, row_end=r1), src

    weights = []
    with ThreadPoolExecutor(max_workers=4) as ex:
        for li in range(layers):
            futs = [ex.submit(one, li, si) for si in range(len(SHAPES))]
            layer = {}
            for si, f in enumerate(futs):
                desc, src = f.result()
                layer[SHAPES[si][0]] = hal.Weight.import_(dev, src, desc)
                del src
            weights.append(layer)
    return weights


def step_ops(weights, xs, ys, comm, wait_prev):
    """The step's 128 ops: per layer qkv, o, gateup (+ SwiGLU; column-sharded
    over `comm` when given), down, each reading its fixed activation."""
    ops = []
    for li, layer in enumerate(weights):
        for name, n, k in SHAPES:
            op = [layer[name], xs[k].data_ptr(), ys[li][name].data_ptr(), 1, 0, wait_prev]
            if name in SHARDED:
                op += [comm, {"swiglu": True}]
            ops.append(tuple(op))
    return ops


def out_rows(name, n):
    return n // 2 if name in SHARDED else n  # gate/up writes one SwiGLU value per row pair


class Timer:
    """CUDA events on `stream` around `steps` calls, bracketed by a barrier
    and a synchronize; the max over ranks."""

    def __init__(self, stream, world):
        import torch
        self.torch, self.stream, self.world = torch, stream, world

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
        self.torch.cuda.synchronize()

    def __call__(self, run_one, steps):
        torch = self.torch
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.barrier()
        ev0.record(self.stream)
        with torch.cuda.stream(self.stream):
            for i in range(steps):
                run_one(i)
        ev1.record(self.stream)
        self.barrier()
        t_ms = ev0.elapsed_time(ev1) / steps
        if self.world > 1:
            import torch.distributed as dist
            tt = torch.tensor([t_ms], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t_ms = float(tt.item())
        return t_ms


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
    ap.add_argument("--skip-configs", action="store_true",
                    help="profiler captures only: no config 0/2/3 objects, no W4A8 or other step forms")
    ap.add_argument("--kernel-case", choices=["gemv", "gemm", "w4a8", "attn"],
                    help="profiler captures: one projection launched warmup+steps times on GPU 0 "
                         "(gemv and w4a8: 65536x4096 at m=1, 151 MB of weights; gemm: 14336x4096 at m=2048; "
                         "attn: decode attention, 32 q over 8 kv heads, 4096-position caches, position "
                         "--case-m or 1024)")
    ap.add_argument("--case-m", type=int, default=None, help="token count of --kernel-case")
    ap.add_argument("--case-n", type=int, default=None, help="rows of --kernel-case")
    ap.add_argument("--case-k", type=int, default=None, help="K of --kernel-case")
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

    weights = make_weights(dev, rank, world, LAYERS)
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

    # activations (fixed per K, as the reference's stream benchmark) and one
    # output per op
    xs = {k: torch.from_numpy(synth.synth_x(1, k, 11 + k).view(np.int16)).cuda().view(torch.bfloat16)
          for k in (4096, 14336)}
    ys = [{name: torch.empty((1, out_rows(name, n)), dtype=torch.bfloat16, device="cuda") for name, n, _ in SHAPES}
          for _ in range(LAYERS)]
    stream = torch.cuda.Stream()
    timed = Timer(stream, world)

    # The step: ONE chain launch (plus the activation prep kernel) over the
    # 128 projections, independent ops (each reads its fixed activation, the
    # reference's projection-stream benchmark, main.rs:2487-2499).  At N > 1
    # the gate/up op is column-sharded and its SwiGLU intermediate reaches the
    # peers inside the kernel over NVLink; the other projections are replicas.
    chains = {wp: hal.Chain(dev, step_ops(weights, xs, ys, comm, wp)) for wp in (0, 1)}
    for wp in (0, 1):
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                chains[wp].run(stream)
    timed.barrier()
    with ClockSampler(local) as clk:
        ms = timed(lambda i: chains[0].run(stream), args.steps)
    clocks = clk.summary()
    launches = 2 * args.steps  # the prep kernel + the chain kernel per step
    alt = {"chain_dependent_ms": timed(lambda i: chains[1].run(stream), args.steps)}

    # Dominant kernel's launch duration, measured live: the chain kernel's
    # share is nearly all of the step (the prep is one small CTA per distinct
    # activation); its roofline uses the step's algorithmic bytes.
    gpu_step_bytes = step_bytes_per_gpu(world)
    achieved = gpu_step_bytes / (ms * 1e-3) / 1e9
    peak, peak_kind = measured_peaks()

    sharded_parity = None
    if world > 1:
        sharded_parity = check_sharded_step(dev, weights, xs, ys, chains[0], stream, rank, world)

    if world == 1 and not args.skip_configs:
        alt["separate_launches_graph_ms"] = separate_launch_graph(weights, xs, stream, timed, args)

    e2e = None if args.skip_e2e else e2e_run(dev, weights, comm, world, args)
    for c in chains.values():
        c.destroy()

    lm = None if args.skip_lmhead else lmhead_run(dev, rank, world, comm, L, stream, timed)
    configs = None
    if world == 1 and not args.skip_configs:
        configs = {"config0_gemv_4096x4096": config0_run(dev, stream, timed, peak),
                   "config2_gate_batch_sweep": config2_run(dev, stream, timed, peak),
                   "config3_prefill_gemm": config3_run(dev, stream, timed)}
    w4a8 = None if (args.skip_configs or world > 1) else w4a8_run(weights, xs, stream, timed, args)
    dstep = None if args.skip_configs else decode_step_run(dev, weights, comm, world, stream, timed, args, peak)

    if rank == 0:
        cpu = None if args.no_cpu_baseline or world > 1 else cpu_baseline()
        line = {
            "metric": METRIC,
            "value": 1e3 / ms, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": DTYPE, "data": DATA, "config": config_of(world),
            "gbs": gpu_step_bytes * (1e3 / ms) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "kernel": "gemv_chain_kernel (the step's 128 GEMVs in one launch, m=1)",
                         "traffic": (CHAIN_DRAM_PER_LAYER * LAYERS if world == 1 else None),
                         "traffic_unit": "bytes per launch (ncu dram read+write of a 4-layer chain, "
                                         "per layer x layers)",
                         "algorithmic_bytes_per_launch": gpu_step_bytes,
                         "region": "one chain launch (+ the activation prep) per step, CUDA events"},
            "other_step_forms_ms": alt,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
            "lm_head": lm,
            "configs": configs,
            "w4a8": w4a8,
            "decode_step": dstep,
            "sharded_parity": sharded_parity,
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


def step_bytes_per_gpu(world):
    """Algorithmic bytes of one step on one GPU: codes + scales of its weights,
    x, and its outputs (the gate/up op writes one SwiGLU value per pair)."""
    total = 0
    for name, n, k in SHAPES:
        ns = n // world if name in SHARDED else n
        total += algo_bytes(ns, k, out_bytes=2) - ns * 2 + out_rows(name, ns) * 2
    return total * LAYERS


def check_sharded_step(dev, weights, xs, ys, chain, stream, rank, world):
    """Per-rank parity of the sharded op: layer 0's gate/up (+ SwiGLU)
    intermediate as gathered by the sharded chain, against the same op run
    unsharded on the full weight on this rank (the same kernel arithmetic per
    row, so the bits must agree)."""
    import torch
    from xnpu_b200 import hal, synth
    name, n, k = next(sh for sh in SHAPES if sh[0] in SHARDED)
    seed = layer_seed(0, [sh[0] for sh in SHAPES].index(name))
    src = synth.planes_bytes(synth.synth_codes(n, k, seed), synth.synth_scales(n, k, seed))
    full = hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k))
    ref = torch.full((1, n // 2), float("nan"), dtype=torch.bfloat16, device="cuda")
    one = hal.Chain(dev, [(full, xs[k].data_ptr(), ref.data_ptr(), 1, 0, 0, None, {"swiglu": True})])
    with torch.cuda.stream(stream):
        chain.run(stream)
        one.run(stream)
    torch.cuda.synchronize()
    got = ys[0][name]
    same = bool(torch.equal(got.view(torch.int16), ref.view(torch.int16)))
    a, b = got.float(), ref.float()
    err = (a - b).abs()
    floor = 1e-2 * b.pow(2).mean().sqrt()
    res = {"rank": rank, "op": f"layer 0 {name} {n}x{k} + SwiGLU, {n // world} rows per rank",
           "bit_identical_to_unsharded": same,
           "max_rel": float((err / torch.maximum(b.abs(), floor)).max().item()),
           "mae": float(err.mean().item()), "fault_bits": dev.fault()}
    one.destroy()
    full.destroy()
    import torch.distributed as dist
    gathered = [None] * world
    dist.all_gather_object(gathered, res)
    return gathered


def separate_launch_graph(weights, xs, stream, timed, args):
    """The same 128 GEMVs (gate/up without the SwiGLU epilogue) as separate
    launches captured in one CUDA graph: the form the chain replaces."""
    import torch
    from xnpu_b200 import lib
    from xnpu_b200._lib import check
    L = lib()
    ys = {name: torch.empty((1, n), dtype=torch.bfloat16, device="cuda") for name, n, _ in SHAPES}

    def step(sp):
        for layer in weights:
            for name, n, k in SHAPES:
                check(L.xq4_linear_raw(layer[name].handle, xs[k].data_ptr(), ys[name].data_ptr(), 1, 0, sp))

    with torch.cuda.stream(stream):
        step(stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(stream.cuda_stream)
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            graph.replay()
    ms = timed(lambda i: graph.replay(), args.steps)
    del graph
    return ms


def rotating_weights(dev, n, k, copies, seed):
    """`copies` imports of one seeded n x k weight (each its own HBM copy):
    launches cycle through them so that no launch finds its weights in L2."""
    from xnpu_b200 import hal, synth
    src = synth.planes_bytes(synth.synth_codes(n, k, seed), synth.synth_scales(n, k, seed))
    return [hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k)) for _ in range(copies)]


def config0_run(dev, stream, timed, peak, copies=36, reps=288):
    """Config 0: one decode GEMV, m = 1, 4096 -> 4096 (9.45 MB), timed over
    36 rotating weight copies (340 MB, > 2x the 126 MB L2).
      * burst: back-to-back xq4_linear_raw launches, one per copy, captured
        once in a CUDA graph and replayed (the reference's pipelined mode,
        submit everything then drain, crates/xnpu-cli/src/main.rs:2404-2431),
        CUDA events around the replays;
      * sequential: submit one launch from the host and wait for it, each
        (the reference's sequential mode), events around each;
      * chained: the 36 GEMVs as one chain launch (xq4_chain_run)."""
    import torch
    from xnpu_b200 import hal, lib, synth
    from xnpu_b200._lib import check
    L = lib()
    n, k = 4096, 4096
    ws = rotating_weights(dev, n, k, copies, 1001)
    x = torch.from_numpy(synth.synth_x(1, k, 1002).view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty((1, n), dtype=torch.bfloat16, device="cuda")
    sp = stream.cuda_stream

    def go(i):
        check(L.xq4_linear_raw(ws[i % copies].handle, x.data_ptr(), y.data_ptr(), 1, 0, sp))

    with torch.cuda.stream(stream):
        for i in range(2 * copies):
            go(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(copies):
            go(i)
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    burst_us = 1e3 * timed(lambda i: graph.replay(), reps // copies) / copies
    del graph
    seq = []
    for i in range(copies):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        with torch.cuda.stream(stream):
            go(i)
        b.record(stream)
        b.synchronize()
        seq.append(a.elapsed_time(b))
    ys = [torch.empty((1, n), dtype=torch.bfloat16, device="cuda") for _ in range(copies)]
    chain = hal.Chain(dev, [(w, x.data_ptr(), yy.data_ptr(), 1, 0, 0) for w, yy in zip(ws, ys)])
    with torch.cuda.stream(stream):
        for _ in range(3):
            chain.run(stream)
    chain_us = 1e3 * timed(lambda i: chain.run(stream), 8) / copies
    chain.destroy()
    for w in ws:
        w.destroy()
    b = algo_bytes(n, k)
    gbs = b / (burst_us * 1e-6) / 1e9
    return {"shape": "m=1, k=4096, n=4096", "algorithmic_bytes": b, "copies": copies,
            "l2": f"{copies} rotating weight copies = {copies * b / 1e6:.0f} MB > 2x 126 MB L2",
            "burst_us_per_gemv": burst_us, "sequential_us_per_gemv": 1e3 * float(np.median(seq)),
            "chained_us_per_gemv": chain_us,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "region": "burst: 36 launches per CUDA graph replay, events around the replays"},
            "chained_gbs": b / (chain_us * 1e-6) / 1e9,
            "roofline_chained": {"bound": "hbm", "achieved": b / (chain_us * 1e-6) / 1e9, "peak": peak,
                                 "unit": "GB/s", "frac": b / (chain_us * 1e-6) / 1e9 / peak,
                                 "region": "the 36 GEMVs (36 weight copies) as one chain launch, the reference's "
                                           "chained op submission; CUDA events, per GEMV"}}


def config2_run(dev, stream, timed, peak, copies=8, reps=48):
    """Config 2: the gate projection 4096 -> 14336 (33 MB) at m in {1, 2, 4,
    8, 16, 32, 64} through xq4_linear (decode GEMV below m = 25, tcgen05 GEMM
    from m = 25), back-to-back launches over 8 rotating copies (264 MB),
    captured once in a CUDA graph and replayed."""
    import json as _json
    import torch
    from xnpu_b200 import lib, synth
    from xnpu_b200._lib import check
    L = lib()
    tflops_peak = _json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("bf16_tflops", 1590.0) \
        if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
    n, k = 14336, 4096
    ws = rotating_weights(dev, n, k, copies, 2001)
    sp = stream.cuda_stream
    out = {}
    for m in (1, 2, 4, 8, 16, 32, 64):
        x = torch.from_numpy(synth.synth_x(m, k, 2002 + m).view(np.int16)).cuda().view(torch.bfloat16)
        y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")

        def go(i):
            check(L.xq4_linear_raw(ws[i % copies].handle, x.data_ptr(), y.data_ptr(), m, 0, sp))

        with torch.cuda.stream(stream):
            for i in range(copies):
                go(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                go(i)
        with torch.cuda.stream(stream):
            graph.replay()
        us = 1e3 * timed(lambda i: graph.replay(), reps // copies) / copies
        del graph
        b = algo_bytes(n, k, m)
        gbs = b / (us * 1e-6) / 1e9
        tfl = 2.0 * m * n * k / (us * 1e-6) / 1e12
        out[str(m)] = {"us": us, "path": "gemv" if m < 25 else "tcgen05 gemm", "gbs": gbs,
                       "hbm_frac": gbs / peak, "tflops": tfl, "tensor_frac": tfl / tflops_peak}
    for w in ws:
        w.destroy()
    return {"shape": "k=4096, n=14336", "copies": copies, "l2": f"{copies} rotating weight copies (264 MB)",
            "peaks": {"hbm_gbs": peak, "bf16_tflops": tflops_peak}, "by_m": out}


def config3_run(dev, stream, timed, copies=3, reps=12):
    """Config 3: prefill m = 2048, 4096 -> 14336, bf16 out, tcgen05 GEMM;
    3 rotating weight and activation copies (150 MB of inputs)."""
    import json as _json
    import torch
    from xnpu_b200 import lib, synth
    from xnpu_b200._lib import check
    L = lib()
    pk = _json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    burst, sustained = pk.get("bf16_tflops", 1590.0), pk.get("bf16_tflops_sustained", 1400.0)
    n, k, m = 14336, 4096, 2048
    ws = rotating_weights(dev, n, k, copies, 3001)
    xs = [torch.from_numpy(synth.synth_x(m, k, 3002 + i).view(np.int16)).cuda().view(torch.bfloat16)
          for i in range(copies)]
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    sp = stream.cuda_stream

    def go(i):
        check(L.xq4_linear_raw(ws[i % copies].handle, xs[i % copies].data_ptr(), y.data_ptr(), m, 0, sp))

    with torch.cuda.stream(stream):
        for i in range(2 * copies):
            go(i)
    us = 1e3 * timed(go, reps)
    for w in ws:
        w.destroy()
    fl = 2.0 * m * n * k
    tf = fl / (us * 1e-6) / 1e12
    return {"shape": "m=2048, k=4096, n=14336", "flops": fl, "us": us,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": burst, "unit": "TFLOP/s", "frac": tf / burst,
                         "peak_kind": "measured burst (cuBLAS bf16)", "frac_of_sustained": tf / sustained}}


def decode_step_run(dev, weights, comm, world, stream, timed, args, peak, pos=1024, cache_seq=4096):
    """Config 4's full decode step: the 32 layers of the benchmark's weights
    as a Llama-3-8B decoder (32 q heads over 8 kv heads, head dim 128, RoPE
    base 500000, random-init RMSNorm weights), one token at context position
    `pos` over 4096-position KV caches: per layer RMSNorm + qkv, RoPE +
    KV-cache append + GQA attention, o + residual, RMSNorm + gate/up + SwiGLU
    (column-sharded at N > 1) + down + residual (xnpu_b200.decode, 6 launches
    per layer), captured once in a CUDA graph and replayed."""
    import torch
    from xnpu_b200 import decode, synth
    rng = np.random.default_rng(4242)

    def norm_w(n):
        w = synth.f32_to_bf16_bits((1.0 + 0.02 * rng.standard_normal(n)).astype(np.float32))
        return torch.from_numpy(w.view(np.int16)).cuda().view(torch.bfloat16)

    layers = [decode.DecodeLayerWeights(lw["qkv"], lw["o"], lw["gateup"], lw["down"], norm_w(4096), norm_w(4096))
              for lw in weights]
    step = decode.DecodeStep(dev, layers, 4096, 32, 8, cache_seq, rope_base=500000.0, comm=comm, world=world)
    for kc, vc in zip(step.k_cache, step.v_cache):  # earlier tokens' keys and values
        kc.normal_()
        vc.normal_()
    step.x.normal_()
    step.pos.fill_(pos)
    with torch.cuda.stream(stream):
        for _ in range(2):
            step.run(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step.run(stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    ms = timed(lambda i: graph.replay(), args.steps)
    finite = bool(torch.isfinite(step.x.float()).all().item())
    del graph
    step.destroy()
    kv_bytes = LAYERS * 8 * (pos + 1) * 2 * 128 * 2
    b = step_bytes_per_gpu(world) + kv_bytes
    gbs = b / (ms * 1e-3) / 1e9
    return {"tok_s": 1e3 / ms, "ms_per_step": ms, "context_pos": pos, "cache_seq": cache_seq,
            "launches_per_step": step.launches_per_step, "output_finite": finite,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "bytes": b, "kv_cache_bytes": kv_bytes},
            "path": "per layer: chain(RMSNorm + qkv) -> xq4_attn_decode -> chain(o + residual) -> "
                    "chain(RMSNorm + gate/up + SwiGLU, down + residual); one CUDA graph per token"}


def e2e_run(dev, weights, comm, world, args):
    """The same step through the public C ABI with host buffers: one pinned
    H2D of the step's activations, one xq4_chain_submit of the 128 ops on
    the device queue, xq4_wait, one D2H of every output -- timed on the host
    clock, max over ranks."""
    import ctypes
    import torch
    from xnpu_b200 import hal, lib, synth
    from xnpu_b200._lib import check
    L = lib()
    k_off = {4096: 0, 14336: 4096 * 2}
    x_bytes = (4096 + 14336) * 2
    y_off, off = {}, 0
    for li in range(LAYERS):
        for name, n, _ in SHAPES:
            y_off[(li, name)] = off
            off += ((out_rows(name, n) * 2 + 255) // 256) * 256
    y_bytes = off
    xb = hal.BufferObject.new(dev, x_bytes)
    yb = hal.BufferObject.new(dev, y_bytes)
    hx = torch.empty(x_bytes, dtype=torch.uint8).pin_memory()
    hy = torch.empty(y_bytes, dtype=torch.uint8).pin_memory()
    hx.numpy()[:] = synth.synth_x(1, x_bytes // 2, 5).reshape(-1).view(np.uint8)
    ops = []
    for li, layer in enumerate(weights):
        for name, n, k in SHAPES:
            op = [layer[name], xb.device_ptr() + k_off[k], yb.device_ptr() + y_off[(li, name)], 1, 0, 0]
            if name in SHARDED:
                op += [comm, {"swiglu": True}]
            ops.append(tuple(op))
    chain = hal.Chain(dev, ops)

    def one():
        check(L.xq4_buffer_upload(xb.handle, hx.data_ptr(), 0, x_bytes))
        chain.submit()
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
    chain.destroy()
    xb.destroy()
    yb.destroy()
    return {"value": 1.0 / dt, "unit": "tok/s", "h2d_bytes_per_step": x_bytes, "d2h_bytes_per_step": y_bytes,
            "ms_per_step": dt * 1e3,
            "path": "xq4_buffer_upload -> xq4_chain_submit (the step's 128 ops) -> xq4_wait -> "
                    "xq4_buffer_download (pinned host buffers)"}


def w4a8_run(weights, xs, stream, timed, args):
    """The step in the W4A8 parity mode: per projection, quantize its
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
    ms = timed(lambda i: g.replay(), args.steps)
    del g
    # the same step as one chain of W4A8 ops: the prep kernel quantizes each
    # distinct activation once, the chain runs the 128 integer-MMA GEMVs
    from xnpu_b200 import hal
    ysc = {name: torch.empty((1, n), dtype=torch.bfloat16, device="cuda") for name, n, _ in SHAPES}
    chain = hal.Chain(weights[0]["qkv"].dev,
                      [(layer[name], xs[k].data_ptr(), ysc[name].data_ptr(), 1, 0, 0, None, {"w4a8": True})
                       for layer in weights for name, n, k in SHAPES])
    with torch.cuda.stream(stream):
        for _ in range(3):
            chain.run(stream)
    ms_chain = timed(lambda i: chain.run(stream), args.steps)
    chain.destroy()
    step_bytes = sum(algo_bytes(n, k) for _, n, k in SHAPES) * LAYERS
    return {"tok_s": 1e3 / ms_chain, "ms_per_step": ms_chain, "gbs": step_bytes / (ms_chain * 1e-3) / 1e9,
            "gpu_launches_per_step": 2,
            "path": "one chain of 128 W4A8 ops (prep kernel: int8 quantization of each activation, bit-exact "
                    "with xq4_quantize_x; chain: integer-MMA GEMVs, bf16 2048-K partials summed in f32)",
            "separate_launches": {"tok_s": 1e3 / ms, "ms_per_step": ms, "gpu_launches_per_step": 2 * len(SHAPES) * LAYERS,
                                  "path": "per projection: xq4_quantize_x + xq4_linear_w4a8 in one CUDA graph"}}


def lmhead_run(dev, rank, world, comm, L, stream, timed, reps=20):
    """lm_head 4096 -> 128256, f32 logits, rows sharded over ranks and
    gathered inside the GEMV over peer memory; 8 rotating weight copies
    (>2x L2 at every N).  At N > 1 each rank also runs the full matrix once
    and compares the gathered logits with it."""
    import torch
    from xnpu_b200 import hal, synth
    from xnpu_b200._lib import check
    n, k = LMHEAD
    r0, r1 = rank * n // world, (rank + 1) * n // world
    copies = 8 if world == 1 else max(8, 2 * world)
    src = synth.planes_bytes(synth.synth_codes(n, k, 424242), synth.synth_scales(n, k, 424242))
    ws = [hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k, row_begin=r0, row_end=r1))
          for _ in range(copies)]
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
    ms = timed(go, reps)
    parity = None
    if world > 1:
        full = hal.Weight.import_(dev, src, hal.layout_desc(hal.XQ4_LAYOUT_PLANES, n, k))
        yf = torch.empty((1, n), dtype=torch.float32, device="cuda")
        with torch.cuda.stream(stream):
            go(0)
            check(L.xq4_linear_raw(full.handle, x.data_ptr(), yf.data_ptr(), 1, 1, sp))
        torch.cuda.synchronize()
        err = (y - yf).abs()
        floor = 1e-2 * yf.pow(2).mean().sqrt()
        parity = {"rank": rank, "vs": "the unsharded lm_head GEMV on this rank",
                  "max_rel": float((err / torch.maximum(yf.abs(), floor)).max().item()),
                  "mae": float(err.mean().item()), "argmax_equal": int(y.argmax()) == int(yf.argmax())}
        full.destroy()
    del src
    for w in ws:
        w.destroy()
    shard_bytes = algo_bytes(r1 - r0, k, out_bytes=4)
    return {"us": ms * 1e3, "shard_rows": r1 - r0, "gbs_per_gpu": shard_bytes / (ms * 1e-3) / 1e9,
            "logits_gather_bytes_in": (n - (r1 - r0)) * 4, "parity_rank0": parity}


def attn_case(args):
    """Decode attention of the 8B shapes (32 q heads over 8 kv heads, head
    dim 128, RoPE base 500000, 4096-position caches) at one position,
    launched warmup+steps times (the profiler captures' command)."""
    import torch
    from xnpu_b200 import hal
    dev = hal.Device.open(0)
    heads, nkv, cs = 32, 8, 4096
    pos = args.case_m if args.case_m is not None else 1024
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn((heads + 2 * nkv) * 128, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn((nkv, cs, 128), device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn((nkv, cs, 128), device="cuda", generator=g).to(torch.bfloat16)
    pd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = torch.empty(heads * 128, dtype=torch.bfloat16, device="cuda")
    at = hal.Attention(dev, heads, nkv, cs, 500000.0)
    stream = torch.cuda.Stream()
    for _ in range(args.warmup):
        at.decode(qkv, kc, vc, pd, out=out, stream=stream)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        at.decode(qkv, kc, vc, pd, out=out, stream=stream)
    b.record(stream)
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / max(1, args.steps)
    kv_bytes = 2 * nkv * (pos + 1) * 128 * 2
    print(json.dumps({"kernel_case": "attn", "heads": heads, "nkv": nkv, "pos": pos, "us_per_launch": us,
                      "kv_gbs": kv_bytes / us / 1e3, "fault": dev.fault()}), flush=True)
    at.destroy()
    dev.close()


def kernel_case(args):
    """One projection launched warmup+steps times through the C ABI (the
    small, single-kernel command that profiler captures run on)."""
    import torch
    from xnpu_b200 import hal, lib, synth
    from xnpu_b200._lib import check
    if args.kernel_case == "attn":
        attn_case(args)
        return
    n, k, m = (14336, 4096, 2048) if args.kernel_case == "gemm" else (65536, 4096, 1)
    m = args.case_m or m
    n = args.case_n or n
    k = args.case_k or k
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
