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

SOURCES = ["matvec.cu", "tma_matvec.cu", "decode.cu", "decode_persistent.cu", "q5_matvec.cu", "prefill_gemm.cu",
           "batch_decode.cu", "glue.cu", "capi.cu"]
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
    common = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC,-fvisibility=hidden", f"-I{INCLUDE}"]
    if verbose:
        common += ["-Xptxas", "-v"]
    # One nvcc per translation unit, in parallel, then one link.
    objs = [LIB_DIR / f".{Path(s).stem}.{os.getpid()}.o" for s in SOURCES]
    procs = [subprocess.Popen(common + ["-c", str(CSRC / s), "-o", str(o)],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
             for s, o in zip(SOURCES, objs)]
    errs = []
    for s, pr in zip(SOURCES, procs):
        out, err = pr.communicate()
        if pr.returncode != 0:
            errs.append(f"nvcc {s} failed ({pr.returncode}):\n{out}\n{err}")
        elif verbose:
            sys.stderr.write(err)
    try:
        if errs:
            raise RuntimeError("\n".join(errs))
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp)] + [str(o) for o in objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    finally:
        for o in objs:
            if o.exists():
                o.unlink()
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(verbose="--verbose" in sys.argv, force=True)
    print(p)
