"""bench.py's JSON line contract, on the CPU-only reference arm: one line
with the metric, value, step counts, scaling, the config, the CPU baseline
(kind, cores, sample) and the zero-copy e2e object of the reference arm."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["value"] > 0 and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_clock_sampler_ready_before_the_timed_region():
    """The NVML sampler has finished starting (or failed to: no NVML here)
    when its context opens, so its initialisation is never inside the timed
    region; without NVML it reports why instead of failing the bench."""
    import time
    sys.path.insert(0, str(ROOT))
    import bench
    t0 = time.time()
    with bench.ClockSampler(0) as clk:
        assert clk._ready.is_set()
    assert time.time() - t0 < 10.0
    s = clk.summary()
    assert set(s) >= {"sm_mhz", "sm_max_mhz", "reasons"}
