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
TOLERANCE_FP32 = 1e-5  # test_runner.py:36

KERNELS = [
    ("matmul_q4", TOLERANCE_Q4),
    ("matmul_q4_mt", TOLERANCE_Q4),
    ("matmul_q8", TOLERANCE_Q8),
    ("matmul_q8_mt", TOLERANCE_Q8),
    ("matmul_q5", TOLERANCE_Q5),         # test_runner.py:43, :298-334
    ("matmul_q5_mt", TOLERANCE_Q5),      # test_runner.py:44, :336-372
    ("matmul_q4_avx512", TOLERANCE_Q4),  # appended by --avx512 (test_runner.py:484-485)
    ("rmsnorm", TOLERANCE_FP32),         # test_runner.py:45-48, :376-398
    ("rope", TOLERANCE_FP32),            # :400-422
    ("softmax", TOLERANCE_FP32),         # :424-438
    ("attention", TOLERANCE_FP32),       # :440-467
]

_SIX = [ctypes.c_void_p] * 4 + [ctypes.c_int64, ctypes.c_int64]


def run_kernel_test(kernel_name: str, tolerance: float, ref_data: dict, native_lib):
    if native_lib is None or not hasattr(native_lib, f"asm_{kernel_name}"):
        return "NOT IMPLEMENTED", None
    func = getattr(native_lib, f"asm_{kernel_name}")
    if kernel_name in ("rmsnorm", "rope", "softmax", "attention"):
        return _run_glue(kernel_name, tolerance, ref_data, func)
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


def _run_glue(kernel_name, tolerance, ref_data, func):
    """The glue kernels' calls as test_runner.py:376-467 makes them."""
    vp, i64, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
    func.restype = None
    if kernel_name == "rmsnorm":
        x = np.ascontiguousarray(ref_data["rmsnorm_x"], dtype=np.float32)
        w = np.ascontiguousarray(ref_data["rmsnorm_weight"], dtype=np.float32)
        y = np.zeros(x.shape[0], dtype=np.float32)
        func.argtypes = [vp, vp, vp, i64, f32]
        func(x.ctypes.data, w.ctypes.data, y.ctypes.data, int(x.shape[0]), f32(float(ref_data["rmsnorm_eps"])))
        max_err = float(np.max(np.abs(y - ref_data["rmsnorm_expected"])))
    elif kernel_name == "rope":
        q = np.ascontiguousarray(ref_data["rope_q"], dtype=np.float32).copy()
        k = np.ascontiguousarray(ref_data["rope_k"], dtype=np.float32).copy()
        func.argtypes = [vp, vp, i64, i64, f32]
        func(q.ctypes.data, k.ctypes.data, int(q.shape[-1]), int(ref_data["rope_pos"]), f32(10000.0))
        max_err = float(max(np.max(np.abs(q - ref_data["rope_q_expected"])),
                            np.max(np.abs(k - ref_data["rope_k_expected"]))))
    elif kernel_name == "softmax":
        x = np.ascontiguousarray(ref_data["softmax_x"], dtype=np.float32)
        y = np.zeros(x.shape[0], dtype=np.float32)
        func.argtypes = [vp, vp, i64]
        func(x.ctypes.data, y.ctypes.data, int(x.shape[0]))
        max_err = float(np.max(np.abs(y - ref_data["softmax_expected"])))
    else:
        q, k, v = (np.ascontiguousarray(ref_data[f"attention_{n}"], dtype=np.float32) for n in "qkv")
        seq_len, head_dim = q.shape
        y = np.zeros_like(q)
        func.argtypes = [vp, vp, vp, vp, i64, i64, f32]
        func(q.ctypes.data, k.ctypes.data, v.ctypes.data, y.ctypes.data, int(seq_len), int(head_dim),
             f32(1.0 / np.sqrt(head_dim)))
        max_err = float(np.max(np.abs(y - ref_data["attention_expected"])))
    return ("PASS" if max_err <= tolerance else "FAIL"), max_err
