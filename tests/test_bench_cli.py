"""bench.py's command line parses (no GPU needed): the driver runs it with --gpus/--steps/
--warmup and --impl, and the ncu captures use --profile-frames."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_bench_help_lists_the_contract_options():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                         timeout=120)
    assert out.returncode == 0, out.stderr
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--profile-frames", "--no-cpu-baseline", "--workload"):
        assert opt in out.stdout


def test_reference_arm_prints_the_contract_line():
    """--impl reference times the reference's own generate() (or the C port when the
    reference was not compiled) as one single-thread process per physical core and prints one
    JSON line with the same metric and config keys as the GPU arm, a cpu_baseline describing
    the run and an e2e with no host copies.  Short KV lengths keep this CPU test light."""
    import json
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "3", "--lmin", "64", "--lmax", "256"], capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "frames/s" and line["higher_is_better"] is True
    assert line["metric"] == "LLM frames/sec (whole box)" and line["value"] > 0
    assert line["config"]["workload"].startswith("configs[4]") and line["scaling"] == "strong"
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert line["cpu_host"]["physical_cores"] >= 1 and line["cpu_host"]["cpu_model"]
    assert line["single_stream_all_threads"]["frames_per_s"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "frames/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
