"""CPU checks of the C-ABI library: it builds, loads, exports every symbol that
include/asmllm.h declares, and rejects bad arguments through its error channel
before touching the GPU.  No compute call is made here."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT


def header_symbols():
    text = (ROOT / "include" / "asmllm.h").read_text()
    return re.findall(r"ASMLLM_API\s+[\w\s\*]+?\b(asm_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def L():
    from asmllm_b200 import native

    return native.try_load_native_library()


def test_header_declares_reference_symbols():
    syms = set(header_symbols())
    # Exports of the reference library that this path replaces (build_kernel.py:85-104).
    for name in ("asm_matmul_q4", "asm_matmul_q8", "asm_threadpool_init", "asm_threadpool_shutdown",
                 "asm_matmul_q4_mt", "asm_matmul_q8_mt", "asm_threadpool_dispatch_q8",
                 "asm_threadpool_get_num_threads", "asm_matmul_q4_avx512"):
        assert name in syms


def test_library_exports_every_declared_symbol(L):
    import subprocess

    from asmllm_b200 import native

    out = subprocess.run(["nm", "-D", "--defined-only", str(native.library_path())],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(asm_\w+)", out))
    declared = set(header_symbols())
    assert declared, "no declarations parsed"
    assert declared <= exported, declared - exported
    # every declared symbol has a ctypes signature in the Python loader
    assert declared <= set(native.SIGNATURES), declared - set(native.SIGNATURES)
    for name in declared:
        assert getattr(L, name) is not None


def test_library_is_built_for_sm100a():
    from asmllm_b200 import build

    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version(L):
    assert b"sm_100a" in L.asm_version()


def _err(L):
    from asmllm_b200 import native

    return native.last_error()


def test_rejects_k_not_multiple_of_32(L):
    q = np.zeros(16 * 4, dtype=np.uint8)
    s = np.zeros(4, dtype=np.float32)
    x = np.zeros(48, dtype=np.float32)
    y = np.zeros(4, dtype=np.float32)
    L.asm_matmul_q4(q.ctypes.data, s.ctypes.data, x.ctypes.data, y.ctypes.data, 4, 48)
    code, msg = _err(L)
    assert code == 1 and "multiple of 32" in msg
    assert _err(L)[0] == 0  # reading clears it


def test_rejects_negative_sizes(L):
    for name in ("asm_matmul_q4", "asm_matmul_q8", "asm_matmul_q8q8", "asm_matmul_q4_avx512"):
        getattr(L, name)(None, None, None, None, -1, 32)
        code, msg = _err(L)
        assert code == 1 and "negative" in msg, name
    rc = L.asm_matmul_q4_async(None, None, None, None, 4, -32, None)
    assert rc == 1
    _err(L)


def test_rejects_null_pointers(L):
    L.asm_matmul_q4(None, None, None, None, 4, 32)
    code, msg = _err(L)
    assert code == 1 and "NULL" in msg


def test_zero_rows_is_a_noop(L):
    # M = 0: nothing to write, no device work (the reference loops zero times).
    L.asm_matmul_q4(None, None, None, None, 0, 0)
    assert _err(L)[0] == 0


def test_register_rejects_bad_format(L):
    q = np.zeros(16, dtype=np.uint8)
    s = np.zeros(1, dtype=np.float32)
    assert L.asm_weights_register(q.ctypes.data, s.ctypes.data, 1, 32, 5) == 1
    assert "fmt" in _err(L)[1]


def test_gguf_split_rejects_bad_args(L):
    assert L.asm_gguf_split_async(3, None, None, None, 0, 1, None) == 1
    _err(L)
    assert L.asm_gguf_split_async(2, None, None, None, 0, -1, None) == 1
    _err(L)


def test_threadpool_thread_count_roundtrip(L):
    # init records the count even when no device is present (it then reports
    # the missing device through the error channel instead of crashing).
    L.asm_threadpool_init(6)
    _err(L)
    assert L.asm_threadpool_get_num_threads() == 6
    L.asm_threadpool_shutdown()
    _err(L)
    assert L.asm_threadpool_get_num_threads() == 0


def test_package_has_no_cpu_fallback():
    # The shipped package must not import the oracle or any CPU compute path.
    pkg = ROOT / "asmllm_b200"
    for f in pkg.rglob("*.py"):
        text = f.read_text()
        assert "oracle" not in re.sub(r"#.*", "", text).replace('"""', ""), f


def test_every_runtime_option_is_documented_and_unknown_names_are_refused(L):
    # asm_set_option's names (capi.cu) all appear in the header's description,
    # and an unknown name returns -1 with an error (no GPU needed)
    src = (ROOT / "asmllm_b200" / "csrc" / "capi.cu").read_text()
    body = src[src.index("ASMLLM_API int asm_set_option("):]
    body = body[: body.index("\n}\n")]
    names = re.findall(r'strcmp\(name, "([a-z_0-9]+)"\)', body)
    assert names, "no option names found"
    header = (ROOT / "include" / "asmllm.h").read_text()
    for n in names:
        assert f'"{n}"' in header, f"option {n} is not described in include/asmllm.h"
    L.asm_set_option.argtypes = [ctypes.c_char_p, ctypes.c_int]
    L.asm_set_option.restype = ctypes.c_int
    assert L.asm_set_option(b"no_such_option", 1) == -1
    buf = ctypes.create_string_buffer(256)
    assert L.asm_get_last_error(buf, 256) != 0 and b"no_such_option" in buf.value
