"""The C++ host side above the C ABI: moss::gpu::LlmModel (llm_gpu.h), compiled with g++
against libmossgpu.so and driven like the reference's moss_llm CLI."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from golden_inputs import prompt_rows
from oracle_py import Oracle, sample_params

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "dsh-moss-tts_b200"


@pytest.fixture(scope="module")
def demo(tmp_path_factory):
    import moss_b200
    moss_b200.build()
    exe = tmp_path_factory.mktemp("shim") / "shim_demo"
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-I", str(PKG / "csrc"),
                    str(ROOT / "tests" / "cpp" / "shim_demo.cpp"), "-L", str(PKG), "-lmossgpu",
                    f"-Wl,-rpath,{PKG}", "-o", str(exe)], check=True, capture_output=True, text=True)
    return exe


def test_shim_compiles_and_reports_load_errors(demo, tmp_path):
    rows = tmp_path / "rows.bin"
    prompt_rows(8, seed=1).tofile(rows)
    r = subprocess.run([str(demo), str(tmp_path / "missing.moss"), str(rows), "2"], capture_output=True, text=True)
    assert r.returncode == 2 and "load failed" in r.stderr


@pytest.mark.gpu
def test_shim_generate_and_prefix_cache_roundtrip(demo, tmp_path, weights_path):
    rows = prompt_rows(40, seed=3)
    (tmp_path / "rows.bin").write_bytes(rows.tobytes())
    plain = subprocess.run([str(demo), weights_path, str(tmp_path / "rows.bin"), "6"], capture_output=True, text=True)
    assert plain.returncode == 0, plain.stderr
    cached = subprocess.run([str(demo), weights_path, str(tmp_path / "rows.bin"), "6", str(tmp_path / "p.mosskv")],
                            capture_output=True, text=True)
    assert cached.returncode == 0, cached.stderr
    a, b = json.loads(plain.stdout), json.loads(cached.stdout)
    assert a["position"] == b["position"] == 40 + 5
    # the prefix file is the reference's .mosskv layout: 40-byte header + 12 x (K, V) fp32
    assert (tmp_path / "p.mosskv").stat().st_size == 40 + 12 * 2 * 40 * 768 * 4
    assert (tmp_path / "p.mosskv").read_bytes()[:8] == b"MOSSPFX1"
    ga, gb = np.array(a["codes"]), np.array(b["codes"])
    assert (ga == gb).all(-1).mean() >= 0.99
    orc = Oracle(weights_path, max_ctx=256, a16_prefill=True)
    orc.prefill_rows(rows)
    oc, _, _ = orc.generate(6, sample_params(greedy=True, rep=1.2, min_frames=1 << 20))
    assert (ga == oc).all(-1).mean() >= 0.99
