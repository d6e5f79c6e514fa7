"""The reference correctness harness's matvec checks, restated for this library.

THRISHAL12345/asmllm tests/correctness/test_runner.py:71-296 calls each
`asm_<kernel>` symbol with ctypes on the seed-42 fixture of
tools/reference_gen.py and compares max |y - expected| to a per-kernel
tolerance (:31-36).  This module does the same, with the same names,
argument types, tolerances and statuses ('PASS', 'FAIL', 'NOT IMPLEMENTED'),
on the fixture saved under tests/golden/, so the drop-in contract is checked
exactly as the reference checks its own kernels.
"""
from __future__ import annotations

import ctypes

import numpy as np

TOLERANCE_Q4 = 0.5   # test_runner.py:33
TOLERANCE_Q8 = 1e-2  # test_runner.py:34
TOLERANCE_Q5 = 1e-2  # test_runner.py:35

KERNELS = [
    ("matmul_q4", TOLERANCE_Q4),
    ("matmul_q4_mt", TOLERANCE_Q4),
    ("matmul_q8", TOLERANCE_Q8),
    ("matmul_q8_mt", TOLERANCE_Q8),
    ("matmul_q5", TOLERANCE_Q5),         # test_runner.py:43, :298-334
    ("matmul_q5_mt", TOLERANCE_Q5),      # test_runner.py:44, :336-372
    ("matmul_q4_avx512", TOLERANCE_Q4),  # appended by --avx512 (test_runner.py:484-485)
]

_SIX = [ctypes.c_void_p] * 4 + [ctypes.c_int64, ctypes.c_int64]


def run_kernel_test(kernel_name: str, tolerance: float, ref_data: dict, native_lib):
    if native_lib is None or not hasattr(native_lib, f"asm_{kernel_name}"):
        return "NOT IMPLEMENTED", None
    func = getattr(native_lib, f"asm_{kernel_name}")
    if kernel_name.startswith("matmul_q5"):  # ql, qh, scales, x, y, M, K (+ threads)
        ql = np.ascontiguousarray(ref_data["q5_matmul_ql"], dtype=np.uint8)
        qh = np.ascontiguousarray(ref_data["q5_matmul_qh"], dtype=np.uint8)
        scales = np.ascontiguousarray(ref_data["q5_matmul_scales"], dtype=np.float32)
        x_vec = np.ascontiguousarray(ref_data["q5_matmul_x"], dtype=np.float32)
        expected = ref_data["q5_matmul_expected"]
        M, K = ql.shape[0], x_vec.shape[0]
        y = np.zeros(M, dtype=np.float32)
        mt = kernel_name.endswith("_mt")
        func.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 2 + ([ctypes.c_int] if mt else [])
        func.restype = None
        args = [ql.ctypes.data, qh.ctypes.data, scales.ctypes.data, x_vec.ctypes.data, y.ctypes.data, int(M), int(K)]
        if mt:
            args.append(ctypes.c_int(4))
        func(*args)
        max_err = float(np.max(np.abs(y - expected)))
        return ("PASS" if max_err <= tolerance else "FAIL"), max_err
    prefix = "q8_matmul" if kernel_name.startswith("matmul_q8") else "q4_matmul"
    wdt = np.int8 if prefix == "q8_matmul" else np.uint8
    qweights = np.ascontiguousarray(ref_data[f"{prefix}_qweights"], dtype=wdt)
    scales = np.ascontiguousarray(ref_data[f"{prefix}_scales"], dtype=np.float32)
    x_vec = np.ascontiguousarray(ref_data[f"{prefix}_x"], dtype=np.float32)
    expected = ref_data[f"{prefix}_expected"]
    M, K = qweights.shape[0], x_vec.shape[0]
    y = np.zeros(M, dtype=np.float32)
    mt = kernel_name.endswith("_mt")
    func.argtypes = _SIX + ([ctypes.c_int] if mt else [])
    func.restype = None
    args = [qweights.ctypes.data, scales.ctypes.data, x_vec.ctypes.data, y.ctypes.data, int(M), int(K)]
    if mt:
        args.append(ctypes.c_int(4))
    func(*args)
    max_err = float(np.max(np.abs(y - expected)))
    return ("PASS" if max_err <= tolerance else "FAIL"), max_err
