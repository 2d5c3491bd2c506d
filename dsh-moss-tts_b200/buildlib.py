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


# variants: "" = the product library; "stamps" = the same sources with phase stamps in the
# small-batch layer kernels (-DMOSSGPU_PHASE_STAMPS), a profiling build beside it
VARIANTS = {"": ([], LIB), "stamps": (["-DMOSSGPU_PHASE_STAMPS"], PKG / "libmossgpu_stamps.so")}


def stale(lib: Path = LIB) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False, variant: str = "") -> Path:
    defs, lib = VARIANTS[variant]
    if force or stale(lib):
        tmp = lib.with_name(f".{lib.stem}.{os.getpid()}.so")
        cmd = [NVCC, *FLAGS, *defs, "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
        r = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
        if r.returncode != 0:
            tmp.unlink(missing_ok=True)
            raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)  # atomic: concurrent builders never expose a half-written library
        if verbose:
            print(r.stdout + r.stderr)
    return lib
