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
    for opt in ("--gpus", "--steps", "--warmup", "--impl", "--profile-frames", "--no-cpu-baseline"):
        assert opt in out.stdout
