"""Builds the C-ABI library build/libasmllm.so from asmllm_b200/csrc with nvcc.

The library is compiled for sm_100a only (B200) and links the CUDA runtime
statically, so it loads next to torch's own runtime without version clashes
and, on a machine without a GPU driver, still loads (its entry points then
report cudaErrorNoDevice / InsufficientDriver through the error channel).

Usage: python -m asmllm_b200.build [--verbose]   (prints ptxas register use)
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CSRC = Path(__file__).resolve().parent / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = ROOT / "build"
LIB_PATH = LIB_DIR / "libasmllm.so"

SOURCES = ["matvec.cu", "tma_matvec.cu", "capi.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the asmllm CUDA library cannot be built")
    return cand


def _inputs():
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + [INCLUDE / "asmllm.h", Path(__file__)]
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > t for f in _inputs() if f.exists())


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_DIR / f".libasmllm.{os.getpid()}.so"
    cmd = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static",
           f"-I{INCLUDE}", "-o", str(tmp)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(CSRC / s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(verbose="--verbose" in sys.argv, force=True)
    print(p)
