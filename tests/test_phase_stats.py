"""bench.py's reduction of the small-layer phase stamps (`--phase-stamps`), on synthetic stamps
with known phase lengths, hand-offs and a straggling CTA (no GPU needed)."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _synthetic(steps=3, attn=(100, 200, 1200, 1100, 600, 1000, 500, 300, 450, 0),
               mlp=(700, 900, 1250, 800, 600, 850, 130, 130, 0), handoff=500, straggler=64):
    """Stamps (ns) of `steps` steps: every CTA of a launch runs the same phase lengths except
    CTA 5 of every launch, which ends `straggler` ns late; launch p + 1 leaves its wait
    `handoff` ns after launch p's last CTA ends."""
    st = np.zeros((steps, 24, 96, 12), dtype=np.int64)
    t = 1_000_000
    for s in range(steps):
        for p in range(24):
            ph = attn if p % 2 == 0 else mlp
            start = t if p == 0 else end + handoff - ph[0] - ph[1]
            stamps = np.concatenate([[0], np.cumsum(ph)]) + start
            st[s, p, :, : len(stamps)] = stamps
            st[s, p, 5, len(stamps) - 1] += straggler
            end = stamps[-1] + straggler
        t = end + 100_000
    return st


def test_phase_stats_recovers_phase_lengths_handoff_and_span():
    bench = _bench()
    st = _synthetic()
    out = bench.phase_stats(st, [150.0, 149.0, 151.0])
    assert out["steps"] == 3 and out["step_us_events"] == 150.0
    assert list(out["attn"]) == bench.SL_ATTN_PHASES and list(out["mlp"]) == bench.SL_MLP_PHASES
    assert out["attn"]["x in + LN1"] == 1.2 and out["attn"]["cluster barrier 2"] == 0.5
    assert out["mlp"]["fc_in + GELU"] == 0.8 and out["mlp"]["exit"] == 0.0
    # after the wait: the phases after stamp 2 plus the straggler
    assert out["attn_after_wait_us"] == round((1200 + 1100 + 600 + 1000 + 500 + 300 + 450 + 64) / 1000, 3)
    assert out["mlp_after_wait_us"] == round((1250 + 800 + 600 + 850 + 130 + 130 + 64) / 1000, 3)
    assert out["handoff_us"] == 0.5
    # layers: launch 0's start to launch 23's last CTA end = 12 (attn + mlp after wait) + 23 hand-offs
    # + launch 0's pre-wait part
    per_layer = out["attn_after_wait_us"] + out["mlp_after_wait_us"]
    assert abs(out["layers_us"] - (0.3 + 12 * per_layer + 23 * 0.5)) < 0.006  # rounded to 0.01 µs
