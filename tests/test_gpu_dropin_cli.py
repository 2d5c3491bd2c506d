"""The reference's own moss_llm CLI (main.cpp, compiled unchanged) on the GPU engine, against
the same CLI on the reference's CPU model, on identical inputs: a 40-row prompt, 20
teacher-forced greedy frames (--force-codes), the raw logits dump (--dump-logits), and the
debug state file the CPU run writes (--save-state) loaded by the GPU run (--load-state).

Both binaries are built in this checkout by oracle/Makefile (`ref`: the reference's CPU
build; `dropin`: the same sources on libmossgpu.so).  The CPU run uses MOSS_A16=all, the
W8A16 prefill that the GPU engine computes.  Tolerances (north_star): logits max-abs-err
<= 2e-2, per-frame KL <= 1e-4, codes identical on >= 99% of frames.
"""
from __future__ import annotations

import json
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

from golden_inputs import forced_codes, prompt_rows

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
CPU_CLI = ROOT / "oracle" / "_ref" / "moss_llm"
GPU_CLI = ROOT / "oracle" / "_ref" / "dropin" / "moss_llm_gpu"
FRAMES = 20


def kl_per_frame(ref, test):
    def sm(x):
        z = x.astype(np.float64)
        z -= z.max(-1, keepdims=True)
        e = np.exp(z)
        return e / e.sum(-1, keepdims=True)
    p, q = sm(ref), sm(test)
    return np.sum(p * (np.log(p + 1e-12) - np.log(q + 1e-12)), -1).mean(-1)


def run(cli, args, env=None):
    r = subprocess.run([str(cli), *map(str, args)], capture_output=True, text=True, timeout=600,
                       env={**os.environ, **(env or {})})
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout[r.stdout.index("{"):])


@pytest.mark.skipif(not (CPU_CLI.exists() and GPU_CLI.exists()),
                    reason="reference CLIs not built here (make -C oracle ref dropin)")
def test_reference_cli_on_gpu_matches_reference_cli_on_cpu(weights_path, tmp_path):
    prompt, forced = tmp_path / "prompt.txt", tmp_path / "forced.txt"
    prompt.write_text("\n".join(" ".join(map(str, r)) for r in prompt_rows(40, seed=3)) + "\n")
    forced.write_text("\n".join(" ".join(map(str, r)) for r in forced_codes(FRAMES, seed=4)) + "\n")
    # --min-frames: the synthetic model's end gate would otherwise stop generate at frame 0
    common = ["--weights", weights_path, "--prompt", prompt, "--frames", FRAMES, "--greedy", "--force-codes", forced,
              "--min-frames", 1000]
    cpu = run(CPU_CLI, [*common, "--threads", min(8, os.cpu_count() or 1), "--dump-logits", tmp_path / "cpu.bin",
                        "--save-state", tmp_path / "state.bin"], env={"MOSS_A16": "all"})
    gpu = run(GPU_CLI, [*common, "--dump-logits", tmp_path / "gpu.bin"])
    resumed = run(GPU_CLI, [*common, "--dump-logits", tmp_path / "gpu2.bin", "--load-state", tmp_path / "state.bin"])
    ref_logits = np.fromfile(tmp_path / "cpu.bin", np.float32).reshape(FRAMES, 16, 1024)
    for out, dump in ((gpu, "gpu.bin"), (resumed, "gpu2.bin")):
        assert out["frames"] == cpu["frames"] == FRAMES
        assert out["prompt_rows"] == 40 and "global_ms_per_frame" in out  # FrameTiming filled
        logits = np.fromfile(tmp_path / dump, np.float32).reshape(FRAMES, 16, 1024)
        assert np.abs(logits - ref_logits).max() <= 2e-2, dump
        assert kl_per_frame(ref_logits, logits).max() <= 1e-4, dump
        same = (np.array(out["codes"]) == np.array(cpu["codes"])).all(-1).mean()
        assert same >= 0.99, (dump, same)
        # the CLI's own teacher-forcing agreement count moves only with the frames that differ
        assert abs(out["teacher_match"] - cpu["teacher_match"]) <= 16 * round((1 - same) * FRAMES), dump


CPU_DEC = ROOT / "oracle" / "_ref" / "moss_decoder"
GPU_DEC = ROOT / "oracle" / "_ref" / "dropin" / "moss_decoder_gpu"


@pytest.mark.skipif(not (CPU_DEC.exists() and GPU_DEC.exists()),
                    reason="reference codec CLIs not built here (make -C oracle ref dropin)")
@pytest.mark.parametrize("stream", [0, 8, 3])
def test_reference_codec_cli_on_gpu_matches_reference_codec_cli_on_cpu(decoder_file, tmp_path, stream):
    """The reference's moss_decoder CLI (decoder_main.cpp, unchanged) on the GPU codec against the
    same CLI on the reference's CPU AudioDecoder: 40 frames of codes, whole-utterance decode
    (--stream 0) and streaming in chunks of 8 and 3 frames; samples within 5e-4."""
    from golden_inputs import codec_codes
    codes = codec_codes(40, seed=77)
    path = tmp_path / "codes.txt"
    path.write_text("\n".join(" ".join(map(str, codes[:, f])) for f in range(codes.shape[1])) + "\n")
    args = ["--weights", decoder_file, "--codes", path, "--stream", stream]
    cpu = run(CPU_DEC, [*args, "--threads", min(8, os.cpu_count() or 1), "--out", tmp_path / "cpu.f32"])
    gpu = run(GPU_DEC, [*args, "--out", tmp_path / "gpu.f32"])
    a = np.fromfile(tmp_path / "cpu.f32", np.float32)
    b = np.fromfile(tmp_path / "gpu.f32", np.float32)
    assert cpu["interleaved_samples"] == gpu["interleaved_samples"] == 40 * 7680 == a.size == b.size
    assert np.isfinite(b).all()
    assert np.abs(a - b).max() <= 5e-4, np.abs(a - b).max()
