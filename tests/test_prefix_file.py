""".mosskv prefix-file and state-file interchange with the reference (save_prefix / load_prefix /
save_state / load_state, llm.cpp:441-632).

tests/golden/prefix_file.npz holds the header and payload digest of a file written by the
reference's own save_prefix after a 3-row prompt (tests/golden/make_golden.py).  Here:
- the shim (llm_gpu.h) lays its header out the same way and computes the same row and
  weight fingerprints, so each side's loader accepts the other's files;
- the payload is the prompt's K and V, layer by layer, in fp32: the oracle's prefill of the
  same rows reproduces it byte for byte.  The engine's cache is fp16, so a file the shim
  writes carries the same layout with fp16-rounded values.
No GPU: the header test calls no engine function."""
from __future__ import annotations

import hashlib
import struct
import subprocess
from pathlib import Path

import numpy as np

from golden_inputs import PREFIX_FILE_ROWS, prompt_rows
from oracle_py import Oracle

ROOT = Path(__file__).resolve().parents[1]
G = ROOT / "tests" / "golden"


def fnv1a(h: int, data: bytes) -> int:
    for b in data:
        h = ((h ^ b) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def test_reference_header_fields():
    g = np.load(G / "prefix_file.npz")
    magic, version, layers, n_pos, hidden, rows_fp, weights_fp = struct.unpack("<8s4I2Q", g["header"].tobytes())
    assert (magic, version, layers, n_pos, hidden) == (b"MOSSPFX1", 1, 12, PREFIX_FILE_ROWS, 768)
    rows = prompt_rows(PREFIX_FILE_ROWS, seed=61)
    assert rows_fp == fnv1a(1469598103934665603, rows.astype("<i4").tobytes())
    assert int(g["size"]) == 40 + 12 * 2 * PREFIX_FILE_ROWS * 768 * 4


def test_shim_header_and_fingerprints_match_the_reference(tmp_path, weights_path):
    exe = tmp_path / "prefix_header_test"
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-I", str(ROOT / "dsh-moss-tts_b200" / "csrc"),
                    str(ROOT / "tests" / "cpp" / "prefix_header_test.cpp"), "-o", str(exe)], check=True,
                   capture_output=True, text=True)
    rows = prompt_rows(PREFIX_FILE_ROWS, seed=61)
    (tmp_path / "rows.bin").write_bytes(rows.astype("<i4").tobytes())
    out = subprocess.run([str(exe), weights_path, str(tmp_path / "rows.bin")], capture_output=True, text=True,
                         timeout=60, check=True).stdout.split("\n")
    size = out[0].split()
    assert size[:2] == ["size", "40"] and [int(v) for v in size[3:]] == [0, 8, 12, 16, 20, 24, 32]
    fp = out[1].split()
    g = np.load(G / "prefix_file.npz")
    _, _, _, _, _, rows_fp, weights_fp = struct.unpack("<8s4I2Q", g["header"].tobytes())
    assert int(fp[1]) == rows_fp and int(fp[2]) == weights_fp
    magic = [int(v) for v in out[2].split()[1:]]
    assert bytes(magic[:8]) == g["header"].tobytes()[:8] and bytes(magic[8:]) == g["state_header"].tobytes()[:8]


def test_payload_is_the_prompts_kv_layer_by_layer(weights_path, weights_digest_ok):
    g = np.load(G / "prefix_file.npz")
    rows = prompt_rows(PREFIX_FILE_ROWS, seed=61)
    o = Oracle(weights_path, max_ctx=64)  # W8A8 prefill, the mode the fixture was made in
    o.prefill_rows(rows)
    h = hashlib.sha256()
    for layer in range(12):
        k, v = o.kv(layer, 0, PREFIX_FILE_ROWS)
        h.update(k.astype("<f4").tobytes())
        h.update(v.astype("<f4").tobytes())
    assert h.hexdigest() == str(g["payload_sha"])


def test_state_file_is_the_prefix_file_plus_hidden(weights_path, weights_digest_ok):
    """save_state (llm.cpp:561-587): the prefix header with magic "MOSSST1", the same K/V payload,
    then the last hidden state."""
    g = np.load(G / "prefix_file.npz")
    magic, version, layers, n_pos, hidden, rows_fp, weights_fp = struct.unpack("<8s4I2Q",
                                                                               g["state_header"].tobytes())
    assert magic == b"MOSSST1\0" and (version, layers, n_pos, hidden) == (1, 12, PREFIX_FILE_ROWS, 768)
    assert g["state_header"].tobytes()[8:] == g["header"].tobytes()[8:]
    assert int(g["state_size"]) == int(g["size"]) + 768 * 4
    rows = prompt_rows(PREFIX_FILE_ROWS, seed=61)
    o = Oracle(weights_path, max_ctx=64)
    o.prefill_rows(rows)
    h = hashlib.sha256()
    for layer in range(12):
        k, v = o.kv(layer, 0, PREFIX_FILE_ROWS)
        h.update(k.astype("<f4").tobytes())
        h.update(v.astype("<f4").tobytes())
    h.update(o.hidden().astype("<f4").tobytes())
    assert h.hexdigest() == str(g["state_payload_sha"])
