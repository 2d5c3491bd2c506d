"""The audio codec decoder's `.moss` weights (MOSS-Audio-Tokenizer-Nano decoder), in numpy.

The reference decoder (csrc/src/decoder.cpp:26-75) reads, by name:

* ``q{i}.cb`` [1024, 8] f32, ``q{i}.out.w`` [512, 8] f32, ``q{i}.out.b`` [512] f32 for the 16
  codebooks; ``q.out.w`` [C0, 512] and ``q.out.b`` [C0] (the quantizer's output projection);
* four stages ``d1 d3 d5 d7`` with time patches 4, 2, 2, 2 and 4, 2, 2, 4 layers: ``in.w``
  [256, C/p] and ``out.w`` [C', 256], and per layer ``attn.w`` [768, 256], ``proj.w`` [256, 256],
  ``f1.w`` [F, 256], ``f2.w`` [256, F], ``n1.w n1.b n2.w n2.b ls1 ls2`` [256] f32;
* the last stage's ``out.w`` has 240 rows, which a final patch of 240 turns into the output
  samples (interleaved stereo at 48 kHz: 7,680 values per 80 ms frame).

d_model 256, 4 heads x 64 and the patches are constants of the reference decoder; the other
widths come from the file.  The production decoder file is not available here, so
`synth_decoder` writes a seeded synthetic one with C0 = 1024, C' = 512 and F = 1024: matrices
whose column count is a multiple of 32 are fp16 (dtype 0, as the reference's
tools/export_decoder.py writes them with --dtype f16), everything else f32 (dtype 3).
"""
from __future__ import annotations

import hashlib
import os
from pathlib import Path

import numpy as np

from .mossfile import DT_F32, write_moss

DT_F16 = 0
D_MODEL, C0, C_MID, FFN, N_CB, CB_SIZE, CB_DIM, Z_DIM = 256, 1024, 512, 1024, 16, 1024, 8, 512
STAGES = ((1, 4, 4, C_MID), (3, 2, 2, C_MID), (5, 2, 2, C_MID), (7, 2, 4, 240))  # id, patch, layers, out rows
SAMPLES_PER_FRAME = 4 * 2 * 2 * 2 * 240


def decoder_specs() -> list[tuple[str, str, int, int]]:
    """(name, kind, rows, cols) of every tensor the reference decoder loads."""
    s = [("q.out.w", "matrix", C0, Z_DIM), ("q.out.b", "bias", 1, C0)]
    for i in range(N_CB):
        s += [(f"q{i}.cb", "codebook", CB_SIZE, CB_DIM), (f"q{i}.out.w", "small", Z_DIM, CB_DIM),
              (f"q{i}.out.b", "bias", 1, Z_DIM)]
    cin = C0
    for sid, patch, layers, cout in STAGES:
        p = f"d{sid}."
        s += [(p + "in.w", "matrix", D_MODEL, cin // patch), (p + "out.w", "matrix", cout, D_MODEL)]
        for n in range(layers):
            lp = f"{p}l{n}."
            s += [(lp + "attn.w", "matrix", 3 * D_MODEL, D_MODEL), (lp + "proj.w", "matrix", D_MODEL, D_MODEL),
                  (lp + "f1.w", "matrix", FFN, D_MODEL), (lp + "f2.w", "matrix", D_MODEL, FFN),
                  (lp + "n1.w", "lnw", 1, D_MODEL), (lp + "n1.b", "bias", 1, D_MODEL),
                  (lp + "n2.w", "lnw", 1, D_MODEL), (lp + "n2.b", "bias", 1, D_MODEL),
                  (lp + "ls1", "scale", 1, D_MODEL), (lp + "ls2", "scale", 1, D_MODEL)]
        cin = cout
    return s


def synth_decoder(path: str | os.PathLike, seed: int = 1, add: dict[str, float] | None = None) -> str:
    """Write the seeded synthetic decoder; returns the file's sha256.  Matrices N(0, 1/cols)
    (so activations keep their scale through the stages), codebooks N(0, 1), LayerNorm weights
    1 + N(0, 0.05), biases N(0, 0.02), layer scales 0.1 + N(0, 0.02).  `add` adds a constant to
    the named f32 tensors (for tests of out-of-range activations)."""
    rng = np.random.default_rng(seed)
    add = add or {}
    entries = []
    for name, kind, rows, cols in decoder_specs():
        if kind == "matrix":
            w = rng.standard_normal((rows, cols), dtype=np.float32) / np.float32(np.sqrt(cols))
            entries.append((name, DT_F16 if cols % 32 == 0 else DT_F32, (rows, cols),
                            (w.astype(np.float16) if cols % 32 == 0 else w).tobytes()))
        elif kind == "codebook":
            entries.append((name, DT_F32, (rows, cols), rng.standard_normal((rows, cols), dtype=np.float32).tobytes()))
        elif kind == "small":
            w = rng.standard_normal((rows, cols), dtype=np.float32) / np.float32(np.sqrt(cols))
            entries.append((name, DT_F32, (rows, cols), w.tobytes()))
        else:
            base, sd = {"lnw": (1.0, 0.05), "bias": (0.0, 0.02), "scale": (0.1, 0.02)}[kind]
            v = (base + sd * rng.standard_normal(cols, dtype=np.float32) + add.get(name, 0.0)).astype(np.float32)
            entries.append((name, DT_F32, (1, cols), v.tobytes()))
    write_moss(path, entries)
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def ensure_synth_decoder(path: str | os.PathLike, seed: int = 1) -> str:
    """Create the synthetic decoder at `path` unless a file of the right size is there."""
    p = Path(path)
    expect = synth_size()
    if not (p.exists() and p.stat().st_size == expect):
        tmp = p.with_suffix(p.suffix + f".tmp{os.getpid()}")
        synth_decoder(tmp, seed)
        os.replace(tmp, p)
    return str(p)


def synth_size() -> int:
    """Byte size of the synthetic decoder file (header, table and 32-byte aligned payloads)."""
    specs = decoder_specs()
    off = 16 + 80 * len(specs)
    for _, kind, rows, cols in specs:
        off += (-off) % 32
        off += rows * cols * (2 if kind == "matrix" and cols % 32 == 0 else 4)
    return off
