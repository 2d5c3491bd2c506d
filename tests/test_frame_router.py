"""The hand-off from the batched step to the codec (frame_router.h; the reference's FrameQueue
and decode_pending, engine.cpp:91-124,480-502): per-stream bounded queues fed from
mossgpu_step / mossgpu_step_frames results, nq-major blocks of 4 frames first and then
chunk_frames, streams ending on the end gate, inside a multi-frame call, or closed by the
caller.  Host C++ only (g++ -pthread), no GPU."""
from __future__ import annotations

import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_frame_router_routes_and_chunks(tmp_path):
    exe = tmp_path / "frame_router_test"
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-pthread", "-I",
                    str(ROOT / "dsh-moss-tts_b200" / "csrc"), str(ROOT / "tests" / "cpp" / "frame_router_test.cpp"),
                    "-o", str(exe)], check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr  # 1 = a block's nq-major codes were wrong
    got = {int(line.split()[0]): [int(v) for v in line.split()[1:]] for line in r.stdout.strip().splitlines()}
    # stream id: frames, then the block sizes (first block 4 frames, then 8, then the rest)
    assert got[5] == [25, 4, 8, 8, 5]
    assert got[9] == [10, 4, 6]       # ended inside its second 6-frame call
    assert got[11] == [20, 4, 8, 8]   # end gate at frame 20
    assert got[2] == [22, 4, 8, 8, 2]  # closed by the caller after 22 frames
