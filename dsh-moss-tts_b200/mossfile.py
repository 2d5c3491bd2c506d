"""The `.moss` weight container and the Q8_0_4X4 matrix layout, in numpy.

Format (reference: tools/export_weights.py:244-268 writes it, csrc/src/weights.cpp:27-126
reads it):

* 16-byte header: ``b"MOSW"``, u32 version (1), u32 tensor count, u32 0.
* one 80-byte entry per tensor: ``name[48]`` (NUL padded), u8 dtype, u8 ndim (2), u16 0,
  u32 dims[3] = (rows, cols, 1) at byte 52, u64 payload offset at 64, u64 byte count at 72.
* payloads, each starting on a 32-byte boundary.

dtype 3 = f32 (all vectors: LayerNorm weights/biases and linear biases), dtype 4 = Q8_0_4X4.

Q8_0_4X4 (tools/export_weights.py:160-179, csrc/src/quant.cpp:56-65): rows are taken in
groups of four; every 32-column block of a group is 136 bytes: the four rows' fp16 scales
``d_k`` (8 bytes), then the four rows' 32 int8 quants ``q_k`` (4 x 32 bytes).  The value is
``f32(d_k) * q``.  Quantiser: ``d = fp16(amax / 127)``, ``q = clip(rint(w / f32(d)), -127, 127)``.

`synth_weights` writes the seeded synthetic model every test and benchmark here uses: the
reference architecture (12 global GPT-2 blocks + 1 local block, d 768, FF 3072, 16 x 1024
audio embeddings tied to the heads, 16384-row text embedding) with N(0, 0.02) matrices.
"""
from __future__ import annotations

import hashlib
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"MOSW"
HEADER = 16
ENTRY = 80
NAME = 48
ALIGN = 32
DT_F32 = 3
DT_Q8X4 = 4

HIDDEN, FF, VOCAB, NVQ, CODEBOOK, LAYERS = 768, 3072, 16384, 16, 1024, 12


def pack_q8x4(w: np.ndarray) -> np.ndarray:
    """Quantise an fp32 [rows, cols] matrix to Q8_0_4X4 bytes, shape [rows/4, cols/32*136]."""
    rows, cols = w.shape
    if rows % 4 or cols % 32:
        raise ValueError(f"Q8_0_4X4 needs rows % 4 == 0 and cols % 32 == 0, got {w.shape}")
    nb = cols // 32
    blk = w.astype(np.float32, copy=False).reshape(rows, nb, 32)
    d16 = (np.abs(blk).max(axis=2, keepdims=True) / 127.0).astype(np.float16)
    d32 = d16.astype(np.float32)
    inv = np.where(d32 == 0, 0.0, 1.0 / np.where(d32 == 0, 1.0, d32))
    q = np.clip(np.rint(blk * inv), -127, 127).astype(np.int8)
    g = rows // 4
    out = np.empty((g, nb, 136), dtype=np.uint8)
    out[:, :, :8] = (np.ascontiguousarray(d16.reshape(g, 4, nb).transpose(0, 2, 1))
                     .view(np.uint8).reshape(g, nb, 8))
    out[:, :, 8:] = (np.ascontiguousarray(q.reshape(g, 4, nb, 32).transpose(0, 2, 1, 3))
                     .view(np.uint8).reshape(g, nb, 128))
    return out.reshape(g, nb * 136)


def unpack_q8x4(blob: np.ndarray, rows: int, cols: int) -> tuple[np.ndarray, np.ndarray]:
    """Split Q8_0_4X4 bytes into (q int8 [rows, cols], d fp16 [rows, cols/32])."""
    nb = cols // 32
    b = np.asarray(blob, dtype=np.uint8).reshape(rows // 4, nb, 136)
    d = np.ascontiguousarray(b[:, :, :8]).view(np.float16).reshape(rows // 4, nb, 4)
    q = np.ascontiguousarray(b[:, :, 8:]).view(np.int8).reshape(rows // 4, nb, 4, 32)
    return (q.transpose(0, 2, 1, 3).reshape(rows, cols),
            np.ascontiguousarray(d.transpose(0, 2, 1)).reshape(rows, nb))


def dequant_q8x4(blob: np.ndarray, rows: int, cols: int) -> np.ndarray:
    q, d = unpack_q8x4(blob, rows, cols)
    return (q.reshape(rows, cols // 32, 32).astype(np.float32)
            * d.astype(np.float32)[:, :, None]).reshape(rows, cols)


def write_moss(path: str | os.PathLike, entries: list[tuple[str, int, tuple[int, int], bytes]]) -> None:
    """entries: (name, dtype, (rows, cols), payload bytes), written in order."""
    table = bytearray()
    payload = bytearray()
    start = HEADER + ENTRY * len(entries)
    for name, dtype, (rows, cols), blob in entries:
        payload += b"\0" * ((-(start + len(payload))) % ALIGN)
        off = start + len(payload)
        nm = name.encode("ascii")
        if len(nm) >= NAME:
            raise ValueError(f"tensor name too long: {name}")
        table += nm.ljust(NAME, b"\0")
        table += struct.pack("<BBH", dtype, 2, 0)
        table += struct.pack("<III", rows, cols, 1)
        table += struct.pack("<QQ", off, len(blob))
        payload += blob
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as fh:
        fh.write(MAGIC + struct.pack("<III", 1, len(entries), 0))
        fh.write(table)
        fh.write(payload)


@dataclass
class Tensor:
    name: str
    dtype: int
    rows: int
    cols: int
    offset: int
    nbytes: int


def read_moss(path: str | os.PathLike) -> tuple[bytes, dict[str, Tensor]]:
    data = Path(path).read_bytes()
    if data[:4] != MAGIC:
        raise ValueError("not a .moss file (bad magic)")
    version, n, _ = struct.unpack_from("<III", data, 4)
    if version != 1:
        raise ValueError(f"unsupported .moss version {version}")
    out = {}
    for i in range(n):
        base = HEADER + i * ENTRY
        name = data[base:base + NAME].split(b"\0", 1)[0].decode("ascii")
        dtype = data[base + NAME]
        rows, cols, _ = struct.unpack_from("<III", data, base + 52)
        off, nbytes = struct.unpack_from("<QQ", data, base + 64)
        if off + nbytes > len(data):
            raise ValueError(f"tensor out of bounds: {name}")
        out[name] = Tensor(name, dtype, rows, cols, off, nbytes)
    return data, out


def tensor_specs() -> list[tuple[str, str, int, int]]:
    """(name, kind, rows, cols) in the reference's export order (export_weights.py:51-92)."""
    s = [("wte", "embed", VOCAB, HIDDEN), ("lnf.w", "lnw", 1, HIDDEN), ("lnf.b", "bias", 1, HIDDEN)]
    blk = [("ln1.w", "lnw", 1, HIDDEN), ("ln1.b", "bias", 1, HIDDEN),
           ("attn.w", "matrix", 3 * HIDDEN, HIDDEN), ("attn.b", "bias", 1, 3 * HIDDEN),
           ("proj.w", "matrix", HIDDEN, HIDDEN), ("proj.b", "bias", 1, HIDDEN),
           ("ln2.w", "lnw", 1, HIDDEN), ("ln2.b", "bias", 1, HIDDEN),
           ("fc_in.w", "matrix", FF, HIDDEN), ("fc_in.b", "bias", 1, FF),
           ("fc_out.w", "matrix", HIDDEN, FF), ("fc_out.b", "bias", 1, HIDDEN)]
    for i in range(LAYERS):
        s += [(f"g{i}.{n}", k, r, c) for n, k, r, c in blk]
    s += [(f"aemb.{ch}", "embed", CODEBOOK, HIDDEN) for ch in range(NVQ)]
    s += [(f"local.{n}", k, r, c) for n, k, r, c in blk]
    s += [("local.lnf.w", "lnw", 1, HIDDEN), ("local.lnf.b", "bias", 1, HIDDEN)]
    return s


def synth_weights(path: str | os.PathLike, seed: int = 0, std: float = 0.02) -> str:
    """Write the seeded synthetic model; returns the file's sha256.

    Matrices and embeddings ~ N(0, std) quantised to Q8_0_4X4; LayerNorm weights
    1 + N(0, 0.1); LayerNorm and linear biases N(0, 0.02); all vectors f32.  Deterministic
    for a given seed (numpy default_rng)."""
    rng = np.random.default_rng(seed)
    entries = []
    for name, kind, rows, cols in tensor_specs():
        if kind in ("matrix", "embed"):
            w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)
            entries.append((name, DT_Q8X4, (rows, cols), pack_q8x4(w).tobytes()))
        elif kind == "lnw":
            v = 1.0 + 0.1 * rng.standard_normal(cols, dtype=np.float32)
            entries.append((name, DT_F32, (1, cols), v.astype(np.float32).tobytes()))
        else:
            v = 0.02 * rng.standard_normal(cols, dtype=np.float32)
            entries.append((name, DT_F32, (1, cols), v.astype(np.float32).tobytes()))
    write_moss(path, entries)
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def ensure_synth_weights(path: str | os.PathLike, seed: int = 0) -> str:
    """Create the synthetic weights at `path` unless a file of the right size is there."""
    p = Path(path)
    expect = 125_047_648
    if not (p.exists() and p.stat().st_size == expect):
        tmp = p.with_suffix(p.suffix + f".tmp{os.getpid()}")
        synth_weights(tmp, seed)
        os.replace(tmp, p)
    return str(p)
