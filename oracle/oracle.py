"""ctypes front end for the CPU oracle (oracle/asmllm_oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by __graft_entry__.smoke() and
by bench.py's cpu_baseline leg / ``--impl reference`` arm, always as the
checker or the timed CPU baseline -- never by the shipped package
``asmllm_b200``.

Every function mirrors one C entry; the C file cites the reference
(THRISHAL12345/asmllm) instruction ranges each restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libasmllm_oracle.so"

K_Q4Q8, K_Q8Q8, K_Q4F32, K_Q8F32, K_Q4F32_512 = 0, 1, 2, 3, 4

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    src = HERE / "asmllm_oracle.c"
    if LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= src.stat().st_mtime:
        return LIB_PATH
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        for name in ("ref_matmul_q4q8", "ref_matmul_q8q8", "ref_matmul_q4f32_avx2",
                     "ref_matmul_q4f32_avx512", "ref_matmul_q8f32_avx2", "ref_matmul_q8f32_neon"):
            f = getattr(L, name)
            f.argtypes = [vp, vp, vp, vp, i64, i64]
            f.restype = None
        L.ref_quantize_q8_0.argtypes = [vp, i64, vp, vp]
        L.ref_quantize_q8_0.restype = None
        L.ref_q8_0_block_qsum.argtypes = [vp, i64, vp]
        L.ref_q8_0_block_qsum.restype = None
        L.ref_q4q8_block_sums.argtypes = [vp, vp, vp, i64, i64]
        L.ref_q4q8_block_sums.restype = None
        L.ref_q8q8_block_sums.argtypes = [vp, vp, vp, i64, i64]
        L.ref_q8q8_block_sums.restype = None
        L.ref_mt_tile_rows.argtypes = [i64, ctypes.c_int]
        L.ref_mt_tile_rows.restype = i64
        L.ref_matmul_q5f32_avx2.argtypes = [vp, vp, vp, vp, vp, i64, i64]
        L.ref_matmul_q5f32_avx2.restype = None
        L.ref_matmul_mt.argtypes = [ctypes.c_int, vp, vp, vp, vp, i64, i64, ctypes.c_int]
        L.ref_matmul_mt.restype = ctypes.c_int
        _lib = L
    return _lib


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a, a.ctypes.data


def quantize_q8_0(x: np.ndarray):
    """fp32[K] -> (int8[K'] , fp32[K/32]) with K' = 32*(K//32)."""
    x, px = _c(x, np.float32)
    K = x.shape[-1]
    nb = K // 32
    xq = np.zeros(nb * 32, dtype=np.int8)
    xd = np.zeros(nb, dtype=np.float32)
    lib().ref_quantize_q8_0(px, K, xq.ctypes.data, xd.ctypes.data)
    return xq, xd


def block_qsum(xq: np.ndarray) -> np.ndarray:
    xq, p = _c(xq, np.int8)
    out = np.zeros(xq.size // 32, dtype=np.int32)
    lib().ref_q8_0_block_qsum(p, xq.size, out.ctypes.data)
    return out


def q4q8_block_sums(qs: np.ndarray, xq: np.ndarray, M: int, K: int) -> np.ndarray:
    qs, pq = _c(qs, np.uint8)
    xq, px = _c(xq, np.int8)
    out = np.zeros((M, K // 32), dtype=np.int32)
    lib().ref_q4q8_block_sums(pq, px, out.ctypes.data, M, K)
    return out


def q8q8_block_sums(qw: np.ndarray, xq: np.ndarray, M: int, K: int) -> np.ndarray:
    qw, pq = _c(qw, np.int8)
    xq, px = _c(xq, np.int8)
    out = np.zeros((M, K // 32), dtype=np.int32)
    lib().ref_q8q8_block_sums(pq, px, out.ctypes.data, M, K)
    return out


def _matvec(name, wdtype, w, scales, x, M, K):
    w, pw = _c(w, wdtype)
    s, ps = _c(scales, np.float32)
    x, px = _c(x, np.float32)
    y = np.zeros(M, dtype=np.float32)
    getattr(lib(), name)(pw, ps, px, y.ctypes.data, M, K)
    return y


def matmul_q4q8(qs, scales, x, M=None, K=None):
    """asm_matmul_q4 with NEON semantics (Q4_0 x Q8_0)."""
    M = M if M is not None else np.asarray(qs).shape[0]
    K = K if K is not None else np.asarray(x).shape[-1]
    return _matvec("ref_matmul_q4q8", np.uint8, qs, scales, x, M, K)


def matmul_q8q8(qw, scales, x, M=None, K=None):
    M = M if M is not None else np.asarray(qw).shape[0]
    K = K if K is not None else np.asarray(x).shape[-1]
    return _matvec("ref_matmul_q8q8", np.int8, qw, scales, x, M, K)


def matmul_q4f32_avx2(qs, scales, x, M=None, K=None):
    M = M if M is not None else np.asarray(qs).shape[0]
    K = K if K is not None else np.asarray(x).shape[-1]
    return _matvec("ref_matmul_q4f32_avx2", np.uint8, qs, scales, x, M, K)


def matmul_q4f32_avx512(qs, scales, x, M=None, K=None):
    M = M if M is not None else np.asarray(qs).shape[0]
    K = K if K is not None else np.asarray(x).shape[-1]
    return _matvec("ref_matmul_q4f32_avx512", np.uint8, qs, scales, x, M, K)


def matmul_q8f32_avx2(qw, scales, x, M=None, K=None):
    M = M if M is not None else np.asarray(qw).shape[0]
    K = K if K is not None else np.asarray(x).shape[-1]
    return _matvec("ref_matmul_q8f32_avx2", np.int8, qw, scales, x, M, K)


def matmul_q5f32_avx2(ql, qh, scales, x, M=None, K=None):
    """asm_matmul_q5 (Q5_0 x fp32, AVX2 lane structure): ql [M, K/32, 16], qh [M, K/32, 4]."""
    M = M if M is not None else np.asarray(ql).shape[0]
    K = K if K is not None else np.asarray(x).shape[-1]
    ql, pl = _c(ql, np.uint8)
    qh, ph = _c(qh, np.uint8)
    s, ps = _c(scales, np.float32)
    x, px = _c(x, np.float32)
    y = np.zeros(M, dtype=np.float32)
    lib().ref_matmul_q5f32_avx2(pl, ph, ps, px, y.ctypes.data, M, K)
    return y


def matmul_q8f32_neon(qw, scales, x, M=None, K=None):
    M = M if M is not None else np.asarray(qw).shape[0]
    K = K if K is not None else np.asarray(x).shape[-1]
    return _matvec("ref_matmul_q8f32_neon", np.int8, qw, scales, x, M, K)


def mt_tile_rows(M: int, nthreads: int) -> int:
    return int(lib().ref_mt_tile_rows(M, nthreads))


def matmul_mt(kind: int, w, scales, x, M: int, K: int, nthreads: int) -> np.ndarray:
    """Row-split multi-thread run of one of the kernels (threadpool tiling)."""
    wdt = np.uint8 if kind in (K_Q4Q8, K_Q4F32, K_Q4F32_512) else np.int8
    w, pw = _c(w, wdt)
    s, ps = _c(scales, np.float32)
    x, px = _c(x, np.float32)
    y = np.zeros(M, dtype=np.float32)
    rc = lib().ref_matmul_mt(kind, pw, ps, px, y.ctypes.data, M, K, int(nthreads))
    if rc != 0:
        raise RuntimeError("oracle: could not start worker threads")
    return y


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
