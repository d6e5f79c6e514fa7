"""Loads build/libasmllm.so (the sm_100a C-ABI library) with ctypes.

Mirrors the reference's loader `try_load_native_library`
(THRISHAL12345/asmllm tests/correctness/test_runner.py:52-68), which looks for
build/libasmllm.so under the project root, with two differences: the library
is built from asmllm_b200/csrc when it is missing or stale, and a failure to
build or load raises instead of returning None.  There is no CPU fallback:
every op in this package runs through this library.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

from . import build as _build

_lock = threading.Lock()
_lib = None

ASM_OK, ASM_E_INVALID, ASM_E_UNSUPPORTED, ASM_E_CUDA, ASM_E_NOT_DEVICE = 0, 1, 2, 3, 4
FMT_Q4_0, FMT_Q8_0 = 2, 8

vp, i64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
i32, f32 = ctypes.c_int32, ctypes.c_float

# Epilogues of asm_fused_matvec_async (ASM_EPI_*) and device error bits.
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_ARGMAX, EPI_GATHER = 0, 1, 2, 3, 4
DEVERR_RING_TIMEOUT, DEVERR_DECODE_RANGE, DEVERR_XCHG_TIMEOUT = 1, 2, 4


class FusedMatvec(ctypes.Structure):
    """asm_fused_matvec_t (include/asmllm.h), field for field."""
    _fields_ = [
        ("fmt", i32), ("epilogue", i32),
        ("qweights", vp), ("scales", vp), ("x", vp), ("image", vp), ("norm_w", vp),
        ("embed", vp), ("x_copy", vp), ("y", vp), ("h", vp), ("image_out", vp),
        ("counters", vp), ("best", vp), ("done", vp), ("tokens", vp), ("pos", vp),
        ("eps", f32), ("vocab", i32), ("max_tokens", i32), ("n_prompt", i32),
        ("M", i64), ("K", i64),
        ("tp", i32), ("tp_rank", i32), ("xchg_rows", i32), ("vocab_offset", i32),
        ("xchg", vp * 8), ("ar_seq", vp), ("ar_done", vp),
    ]


class RowsplitWait(ctypes.Structure):
    """asm_rowsplit_wait_t (include/asmllm.h)."""
    _fields_ = [("n", i32), ("tp", i32), ("rank", i32), ("own", vp * 8), ("y_full", vp * 8), ("M", i64 * 8),
                ("seq", vp), ("done", vp)]


class DecodeLayer(ctypes.Structure):
    """asm_decode_layer_t (include/asmllm.h)."""
    _fields_ = [(n, vp) for n in ("wqkv", "sqkv", "wo", "so", "wgu", "sgu", "wdown", "sdown",
                                  "attn_norm", "ffn_norm", "k_cache", "v_cache")]


class DecodeModel(ctypes.Structure):
    """asm_decode_model_t (include/asmllm.h)."""
    _fields_ = ([(n, i32) for n in ("fmt", "n_layers", "dim", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab",
                                     "ctx", "max_tokens")]
                + [("eps", f32), ("sqrt_head_dim", f32), ("layers", ctypes.POINTER(DecodeLayer))]
                + [(n, vp) for n in ("lm_head", "lm_scales", "final_norm", "embed", "rope_cs", "x", "qkv", "img_attn",
                                     "h", "img_h", "counters", "logits", "best", "tokens", "pos")])


class Rows(ctypes.Structure):
    """asm_rows_t (include/asmllm.h): one batched RMSNorm / embed / residual step."""
    _fields_ = [("rows", i32), ("dim", i32), ("x", vp), ("delta", vp), ("embed", vp), ("tokens", vp), ("pos", vp),
                ("max_tokens", i32), ("vocab", i32), ("norm_w", vp), ("eps", f32), ("reserved", i32), ("tiles", vp)]


# name -> (argtypes, restype); every symbol include/asmllm.h declares.
SIGNATURES = {
    # reference ABI
    "asm_matmul_q4": ([vp, vp, vp, vp, i64, i64], None),
    "asm_matmul_q4_avx512": ([vp, vp, vp, vp, i64, i64], None),
    "asm_matmul_q8": ([vp, vp, vp, vp, i64, i64], None),
    "asm_matmul_q4_mt": ([vp, vp, vp, vp, i64, i64, c_int], None),
    "asm_matmul_q8_mt": ([vp, vp, vp, vp, i64, i64, c_int], None),
    "asm_matmul_q4_avx512_mt": ([vp, vp, vp, vp, i64, i64, c_int], None),
    "asm_threadpool_init": ([c_int], None),
    "asm_threadpool_shutdown": ([], None),
    "asm_threadpool_get_num_threads": ([], c_int),
    "asm_threadpool_dispatch_q8": ([vp, vp, vp, vp, i64, i64], None),
    "asm_threadpool_dispatch_q5": ([vp, vp, vp, vp, vp, i64, i64], None),
    "asm_rmsnorm": ([vp, vp, vp, i64, f32], None),
    "asm_rope": ([vp, vp, i64, i64, f32], None),
    "asm_softmax": ([vp, vp, i64], None),
    "asm_attention": ([vp, vp, vp, vp, i64, i64, f32], None),
    "asm_silu_hadamard": ([vp, vp, i64], None),
    "asm_matmul_q5": ([vp, vp, vp, vp, vp, i64, i64], None),
    "asm_matmul_q5_mt": ([vp, vp, vp, vp, vp, i64, i64, c_int], None),
    "asm_matmul_q5_async": ([vp, vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_gemm_image_async": ([c_int, vp, vp, vp, i64, vp, i64, i64, i64, vp], c_int),
    "asm_gemm_narrow_async": ([c_int, vp, vp, vp, i64, vp, i64, i64, i64, vp], c_int),
    "asm_act_tiles_bytes": ([i64, i64], i64),
    "asm_act_tiles_from_image_async": ([vp, i64, i64, i64, vp, vp], c_int),
    "asm_gemm_tiles_async": ([c_int, vp, vp, vp, vp, i64, i64, i64, vp], c_int),
    "asm_rows_norm_tiles_async": ([ctypes.POINTER(Rows), vp], c_int),
    "asm_rows_swiglu_tiles_async": ([vp, i32, i32, vp, vp], c_int),
    "asm_attention_batch_async": ([vp, i64, vp, vp, i64, vp, vp, vp, i32, i32, i32, i32, i32, f32, vp], c_int),
    "asm_rows_argmax_async": ([vp, i32, i32, i64, i32, vp, vp], c_int),
    "asm_rows_advance_async": ([vp, i32, vp, i32, vp, i32, vp], c_int),
    # additions
    "asm_matmul_q8q8": ([vp, vp, vp, vp, i64, i64], None),
    "asm_quantize_q8_0": ([vp, vp, vp, i64], None),
    "asm_matmul_q4_f32": ([vp, vp, vp, vp, i64, i64], None),
    "asm_weights_register": ([vp, vp, i64, i64, c_int], c_int),
    "asm_weights_unregister": ([vp], c_int),
    "asm_weights_resident_bytes": ([ctypes.POINTER(c_int)], i64),
    "asm_get_last_error": ([ctypes.c_char_p, ctypes.c_size_t], c_int),
    "asm_pointer_kind": ([vp, ctypes.POINTER(c_int)], c_int),
    "asm_matmul_q4_async": ([vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_matmul_q4_f16s_async": ([vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_matmul_q8q8_async": ([vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_matvec_ex_async": ([c_int, vp, vp, c_int, vp, vp, i64, i64, ctypes.c_uint, vp], c_int),
    "asm_packed_row_bytes": ([c_int, i64], i64),
    "asm_launch_floor_async": ([i32, i32, i32, vp], c_int),
    "asm_pack_rows_async": ([c_int, vp, vp, vp, i64, i64, vp], c_int),
    "asm_matvec_packed_async": ([c_int, vp, vp, vp, i64, i64, ctypes.c_uint, vp], c_int),
    "asm_matvec_rowsplit_async": ([c_int, vp, vp, vp, vp, i64, i64, i32, i32, ctypes.POINTER(vp), vp,
                                   ctypes.c_uint, vp], c_int),
    "asm_rowsplit_wait_async": ([ctypes.POINTER(RowsplitWait), vp], c_int),
    "asm_matmul_q8q8_f16s_async": ([vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_matmul_q4_f32_async": ([vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_matmul_q8_async": ([vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_quantize_q8_0_async": ([vp, vp, vp, i64, i64, vp], c_int),
    "asm_block_sums_async": ([c_int, vp, vp, vp, vp, vp, i64, i64, vp], c_int),
    "asm_gguf_split_async": ([c_int, vp, vp, vp, c_int, i64, vp], c_int),
    "asm_act_image_bytes": ([i64], i64),
    "asm_act_image_q8_0_async": ([vp, vp, i64, i64, vp], c_int),
    "asm_matmul_image_async": ([c_int, vp, vp, c_int, vp, vp, i64, i64, vp], c_int),
    "asm_act_image_q8_0_prefetch_async": ([vp, vp, i64, i64, vp, i64, vp, i64, vp], c_int),
    "asm_weights_mark_static": ([vp, i64], c_int),
    "asm_weights_unmark_static": ([vp], c_int),
    "asm_device_error": ([ctypes.POINTER(ctypes.c_uint)], c_int),
    "asm_set_option": ([ctypes.c_char_p, c_int], c_int),
    "asm_matmul_q4_noalloc_async": ([vp, vp, c_int, vp, vp, i64, i64, vp], c_int),
    "asm_fused_matvec_async": ([ctypes.POINTER(FusedMatvec), vp], c_int),
    "asm_ipc_alloc": ([i64, ctypes.POINTER(vp), ctypes.c_char_p], c_int),
    "asm_ipc_open": ([ctypes.c_char_p, ctypes.POINTER(vp)], c_int),
    "asm_ipc_close": ([vp], c_int),
    "asm_ipc_free": ([vp], c_int),
    "asm_attention_decode_async": ([vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, vp], c_int),
    "asm_decode_create": ([ctypes.POINTER(DecodeModel), ctypes.POINTER(vp)], c_int),
    "asm_decode_run_async": ([vp, i32, i32, vp], c_int),
    "asm_decode_destroy": ([vp], c_int),
    "asm_max_k": ([c_int, c_int], i64),
    "asm_version": ([], ctypes.c_char_p),
}


class AsmError(RuntimeError):
    """A libasmllm entry point reported an error through asm_get_last_error."""

    def __init__(self, code: int, message: str):
        super().__init__(f"asmllm error {code}: {message}")
        self.code = code


def library_path():
    alt = os.environ.get("ASMLLM_LIBRARY")
    return Path(alt) if alt else _build.LIB_PATH


def try_load_native_library() -> ctypes.CDLL:
    """Returns the loaded library, building it first if needed; raises on failure.

    ASMLLM_LIBRARY=<path> loads another build of the same library instead
    (for side-by-side measurements); it must exist, nothing is built then."""
    global _lib
    with _lock:
        if _lib is None:
            alt = os.environ.get("ASMLLM_LIBRARY")
            if alt:
                path = Path(alt)
                if not path.exists():
                    raise RuntimeError(f"ASMLLM_LIBRARY={alt} does not exist")
            else:
                path = _build.build()
            L = ctypes.CDLL(str(path))
            for name, (argt, rest) in SIGNATURES.items():
                f = getattr(L, name)
                f.argtypes = argt
                f.restype = rest
            _lib = L
    return _lib


lib = try_load_native_library


def last_error():
    """(code, message) of the calling thread's last library error; clears it."""
    buf = ctypes.create_string_buffer(1024)
    code = lib().asm_get_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(rc=None):
    """Raises AsmError if the last call failed (rc != 0 or an error is pending)."""
    code, msg = last_error()
    if rc not in (None, 0) and code == 0:
        code, msg = rc, "call failed"
    if code != 0:
        raise AsmError(code, msg)
