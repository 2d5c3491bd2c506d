"""Build libmossgpu.so (the C-ABI engine) in-tree with nvcc for sm_100a."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libmossgpu.so"
SOURCES = ["engine.cu", "ops.cu", "codec.cu", "capi.cpp"]
HEADERS = ["types.h", "kernels.cuh", "gemm_tc.cuh", "attn_tc.cuh", "local_fused.cuh", "layer_small.cuh", "engine.h", "../../include/mossgpu.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall", "-diag-suppress", "550", "-shared"]


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if force or stale():
        tmp = LIB.with_name(f".libmossgpu.{os.getpid()}.so")
        cmd = [NVCC, *FLAGS, "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
        r = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
        if r.returncode != 0:
            tmp.unlink(missing_ok=True)
            raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)  # atomic: concurrent builders never expose a half-written library
        if verbose:
            print(r.stdout + r.stderr)
    return LIB
