"""The drop-in boundary, built: the reference's own C++ layers -- TtsEngine (engine.cpp), the
job Runtime (runtime.cpp), the moss_* C ABI (capi.cpp), the moss_llm CLI (main.cpp) and the
moss_decoder CLI (decoder_main.cpp) -- compiled from the reference checkout with no source
change against dsh-moss-tts_b200/csrc/dropin/moss/llm.h (moss::LlmModel = the GPU engine) and
dropin/moss/decoder.h (moss::AudioDecoder = the GPU codec), llm.cpp and decoder.cpp left out,
and linked to libmossgpu.so with every symbol resolved (oracle/Makefile `dropin`).

CPU only: the build, the exported C ABI, the engine symbols it binds, and -- on a machine
without a GPU -- the reference CLI reaching the GPU engine and reporting its error.  The GPU
run of the same CLI against the reference is tests/test_gpu_dropin_cli.py.
"""
from __future__ import annotations

import os
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF_ROOT = Path(os.environ.get("REF_ROOT", ROOT.parent / "reference"))
DROPIN = ROOT / "oracle" / "_ref" / "dropin"

pytestmark = pytest.mark.skipif(not (REF_ROOT / "csrc" / "src" / "engine.cpp").exists(),
                                reason="reference checkout not present")


@pytest.fixture(scope="module")
def built():
    import moss_b200
    moss_b200.build()
    r = subprocess.run(["make", "-C", str(ROOT / "oracle"), "-j8", "dropin", f"REF_ROOT={REF_ROOT}"],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return DROPIN


def test_reference_layers_link_against_the_gpu_engine(built):
    lib = built / "libmoss_tts_gpu.so"
    defined = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True).stdout
    for sym in ("moss_create", "moss_destroy", "moss_set_voice", "moss_speak", "moss_set_sampling", "moss_clone",
                "moss_text_tokens", "moss_last_error", "moss_version"):  # tts.h:25-41
        assert re.search(rf"\bT {sym}\b", defined), sym
    # no CPU model inside: llm.cpp is not linked, the model is the engine behind mossgpu.h
    demangled = subprocess.run(["nm", "-C", str(lib)], capture_output=True, text=True).stdout
    assert "moss::LlmModel::" not in demangled
    # no CPU codec decoder either: decoder.cpp is not linked, AudioDecoder is the GPU codec
    assert "moss::AudioDecoder::" not in demangled
    undefined = subprocess.run(["nm", "-D", "--undefined-only", str(lib)], capture_output=True, text=True).stdout
    bound = set(re.findall(r"\bU (mossgpu_\w+)", undefined))
    declared = set(re.findall(r"\b(mossgpu_\w+)\s*\(", (ROOT / "include" / "mossgpu.h").read_text()))
    assert {"mossgpu_create", "mossgpu_prefill", "mossgpu_step", "mossgpu_stream_fork"} <= bound
    assert {"mossgpu_codec_create", "mossgpu_codec_reset", "mossgpu_codec_decode_chunk"} <= bound
    assert bound <= declared


def test_reference_cli_runs_on_the_gpu_engine_or_reports_no_device(built, weights_path, tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: tests/test_gpu_dropin_cli.py runs the CLI against the reference")
    prompt = tmp_path / "p.txt"
    prompt.write_text("9 " + " ".join(str(100 + i) for i in range(16)) + "\n")
    r = subprocess.run([str(built / "moss_llm_gpu"), "--weights", weights_path, "--prompt", str(prompt),
                        "--frames", "2", "--greedy"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 1
    assert "cuda" in r.stderr.lower()  # the engine's own error, through LlmModel::load's err


def test_reference_job_request_drives_the_text_runtime(built, tmp_path):
    """TextJobRuntime::submit takes the reference's own moss::JobRequest and moss::PcmSink
    (runtime.h:45-62,83), compiled from the reference's runtime.h, over the engine double."""
    exe = tmp_path / "job_request_compat"
    src = ROOT / "tests" / "cpp" / "job_request_compat.cpp"
    r = subprocess.run(["g++", "-std=c++20", "-O2", "-pthread", "-include", "cstring", "-w",
                        "-I", str(ROOT / "dsh-moss-tts_b200" / "csrc" / "dropin"), "-I", str(REF_ROOT / "csrc" / "include"),
                        "-I", str(ROOT / "dsh-moss-tts_b200" / "csrc"), "-I", str(ROOT / "tests" / "cpp"), str(src),
                        "-o", str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-4000:]
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr


def test_reference_codec_cli_on_the_gpu_codec_or_reports_no_device(built, decoder_file, tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: tests/test_gpu_dropin_cli.py runs the codec CLI against the reference")
    codes = tmp_path / "codes.txt"
    codes.write_text("\n".join(" ".join(str((17 * f + 31 * i) % 1024) for i in range(16)) for f in range(3)) + "\n")
    r = subprocess.run([str(built / "moss_decoder_gpu"), "--weights", decoder_file, "--codes", str(codes),
                        "--out", str(tmp_path / "a.f32")], capture_output=True, text=True, timeout=120)
    assert r.returncode == 1
    assert "cuda" in r.stderr.lower()  # the codec's own error, through AudioDecoder::load's err
