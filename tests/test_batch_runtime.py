"""The batching job runtime (batch_runtime.h): the reference Runtime's submit / wait / job /
cancel / queue_depth (runtime.h:92-113) with one worker advancing every admitted job in
shared mossgpu_prefill_batch / mossgpu_step_frames calls, each job producing what
TtsEngine::synthesize's token loop produces for it (engine.cpp:415-545).

CPU: the runtime over a host-only engine double, against a sequential restatement of the
reference loop, and ShardedRuntime over two doubles (one per GPU) with jobs balanced by
outstanding work (tests/cpp/batch_runtime_test.cpp).  GPU: the runtime over the real engine
through the C ABI (tests/cpp/batch_runtime_demo.cpp), against the same engine calls made
directly through the Python API in the order the runtime makes them."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

from golden_inputs import prompt_rows

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "dsh-moss-tts_b200"
CXX = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-pthread", "-I", str(PKG / "csrc")]


def test_batch_runtime_on_engine_double(tmp_path):
    exe = tmp_path / "batch_runtime_test"
    subprocess.run([*CXX, str(ROOT / "tests" / "cpp" / "batch_runtime_test.cpp"), "-o", str(exe)], check=True,
                   capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = dict(line.split(" ", 1) for line in r.stdout.strip().splitlines())
    assert set(lines) == {"A", "B", "C", "D", "E", "F"}
    stats = dict(kv.split("=") for kv in lines["A"].split())
    # jobs really shared calls: several segments per prefill call, several streams per step call
    assert int(stats["prefill_max"]) > 1 and int(stats["step_max"]) > 1
    # two engines behind ShardedRuntime: both took work
    shards = dict(kv.split("=") for kv in lines["E"].split())
    assert int(shards["shard0_cost"]) > 0 and int(shards["shard1_cost"]) > 0


def test_text_job_runtime_on_engine_double(tmp_path):
    """TextJobRuntime (job_runtime.h): the reference Runtime's text-level submit(JobRequest,
    PcmSink) over the batching runtime, with a test front end and codec: every job's PCM equals
    the sequential synthesis of the same text, decoded and converted as the reference does;
    unknown voices, a full queue, failing sinks and codecs, and cancel end jobs as the reference's
    Runtime does."""
    exe = tmp_path / "job_runtime_test"
    subprocess.run([*CXX, "-I", str(ROOT / "tests" / "cpp"), str(ROOT / "tests" / "cpp" / "job_runtime_test.cpp"),
                    "-o", str(exe)], check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.split() == ["A", "jobs=10", "B", "ok"]


# ---- GPU: the runtime over the engine, replayed through the Python API

PREFIX_M = 24
MAX_CTX = 512
MAX_STREAMS = 16
FRAMES_PER_CALL = 16
# (seed, greedy, rep_x1000, min_frames, max_frames, chunk_frames, use_prefix, prompt rows)
JOBS = [
    (11, 1, 1200, 2, 10, 4, 1, 20),
    (12, 0, 1200, 2, 12, 8, 1, 33),
    (13, 1, 1200, 2, 10, 3, 0, 41),
    (14, 0, 1200, 2, 12, 5, 0, 18),
    (15, 1, 1200, 2, 10, 8, 1, 27),
    (16, 0, 1200, 2, 12, 1, 1, 30),
]


def params_for(pkg, job):
    seed, greedy, rep, min_frames = job[:4]
    return pkg.SampleParams.make(greedy=bool(greedy), temperature=0.8, top_k=25, top_p=0.95,
                                 repetition_penalty=rep / 1000.0, end_greedy=True, min_frames=min_frames)


def write_jobs(path: Path, prefix, rows):
    ints = [len(JOBS), PREFIX_M, *prefix.reshape(-1).tolist()]
    for job, r in zip(JOBS, rows):
        ints += [*job[:7], r.shape[0], *r.reshape(-1).tolist()]
    np.asarray(ints, np.int32).tofile(path)


def parse_output(text: str):
    jobs = {}
    cur = None
    for line in text.splitlines():
        f = line.split()
        if f[0] == "job":
            cur = int(f[1])
            jobs[cur] = {"state": f[2], "frames": int(f[3]), "blocks": []}
        else:
            n = int(f[2])
            codes = np.array([int(v) for v in f[3:]], np.int32).reshape(16, n)
            jobs[cur]["blocks"].append((int(f[1]), codes))
    return jobs


@pytest.mark.gpu
def test_batch_runtime_on_engine_matches_direct_calls(tmp_path, weights_path):
    import moss_b200 as pkg
    pkg.build()
    exe = tmp_path / "batch_runtime_demo"
    subprocess.run([*CXX, str(ROOT / "tests" / "cpp" / "batch_runtime_demo.cpp"), "-L", str(PKG), "-lmossgpu",
                    f"-Wl,-rpath,{PKG}", "-o", str(exe)], check=True, capture_output=True, text=True)
    prefix = prompt_rows(PREFIX_M, seed=70)
    rows = [prompt_rows(job[7], seed=80 + i) for i, job in enumerate(JOBS)]
    write_jobs(tmp_path / "jobs.bin", prefix, rows)
    r = subprocess.run([str(exe), weights_path, str(tmp_path / "jobs.bin"), str(tmp_path / "out.txt"), "8",
                        str(FRAMES_PER_CALL)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    got = parse_output((tmp_path / "out.txt").read_text())
    assert sorted(got) == list(range(len(JOBS)))

    # the same engine calls, made directly: one batched prefill of every job (all are admitted
    # at once), then one step_frames call per parameter group in order of first appearance
    e = pkg.Engine(weights_path, device=0, max_streams=MAX_STREAMS, max_ctx=MAX_CTX)
    try:
        p0 = e.open()
        e.prefill(p0, prefix)
        sids = [e.fork(p0, PREFIX_M) if job[6] else e.open() for job in JOBS]
        e.prefill_batch(sids, rows, starts=[PREFIX_M if job[6] else 0 for job in JOBS])
        for s, job in zip(sids, JOBS):
            e.generate_begin(s, job[0])
        groups = []
        for i, job in enumerate(JOBS):
            key = job[1:5]
            for g in groups:
                if g[0] == key:
                    g[1].append(i)
                    break
            else:
                groups.append((key, [i]))
        want = {}
        for key, members in groups:
            frames = min(FRAMES_PER_CALL, *(JOBS[i][4] for i in members))
            codes, done = e.step_frames([sids[i] for i in members], params_for(pkg, JOBS[members[0]]), frames)
            for k, i in enumerate(members):
                want[i] = codes[: int(done[k]), k, :]
    finally:
        e.close()

    total = 0
    for i, job in enumerate(JOBS):
        j = got[i]
        assert j["state"] == "completed", (i, j["state"])
        n_frames = want[i].shape[0]
        assert j["frames"] == n_frames
        # block sizes: min(4, chunk) first, then chunk, then the remainder
        chunk = job[5]
        sizes, left, first = [], n_frames, min(4, chunk)
        while left > 0:
            take = min(first if not sizes else chunk, left)
            sizes.append(take)
            left -= take
        assert [c.shape[1] for _, c in j["blocks"]] == sizes
        assert all(seg == 0 for seg, _ in j["blocks"])
        if n_frames:
            frames = np.concatenate([c.T for _, c in j["blocks"]], axis=0)
            assert (frames == want[i]).all(), i
        total += n_frames
    assert total > 0


# Two GPUs, one process: ShardedRuntime over an engine per device.  Every job has the same cost
# (no prefix, 24 prompt rows, 10 frames), so the least-loaded rule alternates: even jobs on
# GPU 0, odd jobs on GPU 1.  Each GPU's jobs are then replayed directly on that device.
JOBS2 = [(31 + i, int(i % 4 < 2), 1200, 2, 10, 4 + i % 3, 0, 24) for i in range(8)]


@pytest.mark.gpu
def test_sharded_runtime_on_two_gpus_matches_direct_calls(tmp_path, weights_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import moss_b200 as pkg
    pkg.build()
    exe = tmp_path / "batch_runtime_demo"
    subprocess.run([*CXX, str(ROOT / "tests" / "cpp" / "batch_runtime_demo.cpp"), "-L", str(PKG), "-lmossgpu",
                    f"-Wl,-rpath,{PKG}", "-o", str(exe)], check=True, capture_output=True, text=True)
    prefix = prompt_rows(PREFIX_M, seed=71)
    rows = [prompt_rows(job[7], seed=90 + i) for i, job in enumerate(JOBS2)]
    ints = [len(JOBS2), PREFIX_M, *prefix.reshape(-1).tolist()]
    for job, r in zip(JOBS2, rows):
        ints += [*job[:7], r.shape[0], *r.reshape(-1).tolist()]
    np.asarray(ints, np.int32).tofile(tmp_path / "jobs.bin")
    r = subprocess.run([str(exe), weights_path, str(tmp_path / "jobs.bin"), str(tmp_path / "out.txt"), "8",
                        str(FRAMES_PER_CALL), "2"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    text = (tmp_path / "out.txt").read_text()
    shard_of = {int(l.split()[1]): int(l.split()[4]) for l in text.splitlines() if l.startswith("job ")}
    assert shard_of == {i: i % 2 for i in range(len(JOBS2))}
    got = parse_output(text)

    want = {}
    for dev in (0, 1):
        mine = [i for i in range(len(JOBS2)) if i % 2 == dev]
        e = pkg.Engine(weights_path, device=dev, max_streams=MAX_STREAMS, max_ctx=MAX_CTX)
        try:
            p0 = e.open()
            e.prefill(p0, prefix)
            sids = [e.open() for _ in mine]
            e.prefill_batch(sids, [rows[i] for i in mine], starts=[0] * len(mine))
            for s, i in zip(sids, mine):
                e.generate_begin(s, JOBS2[i][0])
            groups = []
            for k, i in enumerate(mine):
                key = JOBS2[i][1:5]
                for g in groups:
                    if g[0] == key:
                        g[1].append(k)
                        break
                else:
                    groups.append((key, [k]))
            for key, members in groups:
                frames = min(FRAMES_PER_CALL, *(JOBS2[mine[k]][4] for k in members))
                codes, done = e.step_frames([sids[k] for k in members], params_for(pkg, JOBS2[mine[members[0]]]),
                                            frames)
                for c, k in enumerate(members):
                    want[mine[k]] = codes[: int(done[c]), c, :]
        finally:
            e.close()
    for i in range(len(JOBS2)):
        assert got[i]["state"] == "completed", (i, got[i]["state"])
        n = want[i].shape[0]
        assert got[i]["frames"] == n
        if n:
            frames = np.concatenate([c.T for _, c in got[i]["blocks"]], axis=0)
            assert (frames == want[i]).all(), i


@pytest.mark.gpu
def test_batch_runtime_with_gpu_codec_streams(tmp_path, weights_path, decoder_file):
    """The runtime's frames through the GPU codec (CodecStreams: one codec stream per job, fed
    each block in order on the worker thread) give the samples that decoding each job's blocks
    directly with mossgpu_codec_decode_chunk gives -- bit for bit, the same kernels."""
    import moss_b200 as pkg
    pkg.build()
    exe = tmp_path / "batch_runtime_demo"
    subprocess.run([*CXX, str(ROOT / "tests" / "cpp" / "batch_runtime_demo.cpp"), "-L", str(PKG), "-lmossgpu",
                    f"-Wl,-rpath,{PKG}", "-o", str(exe)], check=True, capture_output=True, text=True)
    prefix = prompt_rows(PREFIX_M, seed=70)
    rows = [prompt_rows(job[7], seed=80 + i) for i, job in enumerate(JOBS)]
    write_jobs(tmp_path / "jobs.bin", prefix, rows)
    out = tmp_path / "out.txt"
    r = subprocess.run([str(exe), weights_path, str(tmp_path / "jobs.bin"), str(out), "8", str(FRAMES_PER_CALL)],
                       capture_output=True, text=True, timeout=600, env={**os.environ, "MOSS_DEMO_DECODER": decoder_file})
    assert r.returncode == 0, r.stderr
    got = parse_output(out.read_text())
    codec = pkg.Codec(decoder_file, device=0, max_streams=1, max_batch_frames=16)
    try:
        sid = codec.open()
        checked = 0
        for i in sorted(got):
            pcm = np.fromfile(f"{out}.pcm{i}", np.float32)
            codec.reset(sid)
            want = [codec.decode_chunk(sid, c) for _, c in got[i]["blocks"]]
            want = np.concatenate(want) if want else np.zeros(0, np.float32)
            assert pcm.size == sum(c.shape[1] for _, c in got[i]["blocks"]) * 7680
            assert np.array_equal(pcm, want), i
            checked += pcm.size > 0
        assert checked > 0
    finally:
        codec.close()
