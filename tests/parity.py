"""Parity metrics shared by the GPU tests, and the record of every figure.

The bars (main.rs:2287-2296 defines the op, main.rs:2705-2714 the reference's
own golden tier, main.rs:2713 its relative-error denominator):

  * max relative error <= 1e-2, with the denominator max(|ref|, 1e-2 * rms(ref));
  * mean absolute error <= 1e-3;
  * |g - w| <= 0.01 + 0.01 |w| for every output (the golden tier).

Why the floor: any two f32 summation orders of a K-term dot product differ by
about 1e-7..1e-6 absolute, which is more than 1e-2 relative for the rare
outputs within ~1e-4 of zero.  The unfloored figure (denominator |ref| + 1e-6,
as the reference computes it at main.rs:2713) and the count of outputs whose
unfloored relative error exceeds 1e-2 are recorded for every comparison and
printed in the terminal summary of the run (tests/conftest.py), next to the
floored figure the assert uses.
"""
import os

import numpy as np

MAX_REL = 1e-2
MAE = 1e-3

# one entry per comparison: (test id, label, outputs, floored max rel, mae,
# unfloored max rel, outputs above 1e-2 unfloored)
RECORDS = []


def _test_id():
    cur = os.environ.get("PYTEST_CURRENT_TEST", "")
    return cur.rsplit(" ", 1)[0] if cur else "?"


def record(label, n, max_rel, mae, raw, above):
    RECORDS.append((_test_id(), label, int(n), float(max_rel), float(mae), float(raw), int(above)))


def rel_metrics(got, ref, label=""):
    """(max relative error with the floored denominator, mean absolute error,
    max relative error with the unfloored |ref| + 1e-6 denominator); the
    figures and the count of outputs above 1e-2 unfloored are recorded."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref)
    floor = 1e-2 * np.sqrt(np.mean(ref ** 2))
    raw_rel = err / (np.abs(ref) + 1e-6)
    max_rel = float((err / np.maximum(np.abs(ref), floor)).max()) if err.size else 0.0
    mae = float(err.mean()) if err.size else 0.0
    raw = float(raw_rel.max()) if err.size else 0.0
    record(label, err.size, max_rel, mae, raw, int((raw_rel > 1e-2).sum()))
    return max_rel, mae, raw


def assert_parity(got_f32, ref_f32, what):
    """Outputs (f32 values) within the bars against the oracle's outputs of
    the same type."""
    got = np.asarray(got_f32, dtype=np.float64)
    ref = np.asarray(ref_f32, dtype=np.float64)
    max_rel, mae, raw = rel_metrics(got, ref, what)
    tier_ok = bool(np.all(np.abs(got - ref) <= 0.01 + 0.01 * np.abs(ref)))
    assert max_rel <= MAX_REL and mae <= MAE and tier_ok, \
        f"{what}: max_rel={max_rel:.3e} mae={mae:.3e} (unfloored {raw:.3e}) tier={tier_ok}"


def summary_lines():
    """The recorded figures as text lines (empty when nothing was recorded)."""
    if not RECORDS:
        return []
    lines = ["parity figures (max_rel: floored denominator, the assert's; raw: |ref|+1e-6 denominator; "
             ">1e-2: outputs above 1e-2 unfloored)",
             f"{'test':<70} {'outputs':>10} {'max_rel':>9} {'mae':>9} {'raw':>9} {'>1e-2':>6}"]
    tot_n = tot_above = 0
    for tid, label, n, mr, mae, raw, above in RECORDS:
        name = tid.split("::", 1)[-1]
        if label:
            name = f"{name} [{label}]"
        lines.append(f"{name[:70]:<70} {n:>10} {mr:>9.2e} {mae:>9.2e} {raw:>9.2e} {above:>6}")
        tot_n += n
        tot_above += above
    lines.append(f"{len(RECORDS)} comparisons, {tot_n} outputs, {tot_above} above 1e-2 unfloored "
                 f"({tot_above / max(tot_n, 1):.2e} of outputs)")
    return lines
