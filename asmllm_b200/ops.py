"""Python operator API over libasmllm.so.

Two layers, both going through the C ABI (no Python or torch compute path):

* Host layer -- numpy in, numpy out, through the reference's synchronous
  entry points (`asm_matmul_q4`, `asm_matmul_q8`, ...), exactly as the
  reference's ctypes callers use them (THRISHAL12345/asmllm
  tests/correctness/test_runner.py:84-111, src/runtime/generate.py:255-259).
* Device layer -- torch CUDA tensors, stream-ordered on torch's current
  stream through the `*_async` entries; this is what the decode driver and
  the benchmark use with weights resident in HBM.

Argument meanings follow the reference: qweights Q4_0 uint8 [M, K/32, 16]
(or flat), Q8_0 int8 [M, K/32, 32], scales [M, K/32], x fp32 [K], y fp32 [M].
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import native
from .native import FMT_Q4_0, FMT_Q8_0, AsmError

MV_INDEPENDENT = 1  # ASM_MV_INDEPENDENT (include/asmllm.h)
MV_PACKED = 2  # ASM_MV_PACKED

# --------------------------------------------------------------------------
# Host (numpy) layer: the reference-facing synchronous ABI
# --------------------------------------------------------------------------


def _np(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _mk(qw, scales, x, wdtype, bytes_per_block):
    qw = _np(qw, wdtype)
    scales = _np(scales, np.float32)
    x = _np(x, np.float32)
    K = x.shape[-1]
    M = scales.shape[0] if scales.ndim >= 2 else (qw.size // max(1, (K // 32) * bytes_per_block) if K else 0)
    return qw, scales, x, int(M), int(K)


def _sync_call(name, qw, scales, x, wdtype, bpb, *extra):
    qw, scales, x, M, K = _mk(qw, scales, x, wdtype, bpb)
    y = np.zeros(M, dtype=np.float32)
    getattr(native.lib(), name)(qw.ctypes.data, scales.ctypes.data, x.ctypes.data,
                                y.ctypes.data, M, K, *extra)
    native.check()
    return y


def matmul_q4(qweights, scales, x):
    """asm_matmul_q4: Q4_0 x Q8_0 (x quantized inside, NEON semantics)."""
    return _sync_call("asm_matmul_q4", qweights, scales, x, np.uint8, 16)


def matmul_q4_mt(qweights, scales, x, num_threads=4):
    return _sync_call("asm_matmul_q4_mt", qweights, scales, x, np.uint8, 16, int(num_threads))


def matmul_q4_avx512(qweights, scales, x):
    """asm_matmul_q4_avx512: Q4_0 x fp32 (x86 semantics)."""
    return _sync_call("asm_matmul_q4_avx512", qweights, scales, x, np.uint8, 16)


def matmul_q4_f32(qweights, scales, x):
    return _sync_call("asm_matmul_q4_f32", qweights, scales, x, np.uint8, 16)


def matmul_q8(qweights, scales, x):
    """asm_matmul_q8: Q8_0 x fp32 (x86 / NEON-scalar semantics)."""
    return _sync_call("asm_matmul_q8", qweights, scales, x, np.int8, 32)


def matmul_q8_mt(qweights, scales, x, num_threads=4):
    return _sync_call("asm_matmul_q8_mt", qweights, scales, x, np.int8, 32, int(num_threads))


def matmul_q8q8(qweights, scales, x):
    """asm_matmul_q8q8: Q8_0 x Q8_0."""
    return _sync_call("asm_matmul_q8q8", qweights, scales, x, np.int8, 32)


def quantize_q8_0(x):
    """asm_quantize_q8_0: fp32[K] -> (int8[K], fp32[K/32])."""
    x = _np(x, np.float32)
    K = x.shape[-1]
    xq = np.zeros(K, dtype=np.int8)
    xd = np.zeros(K // 32, dtype=np.float32)
    native.lib().asm_quantize_q8_0(x.ctypes.data, xq.ctypes.data, xd.ctypes.data, K)
    native.check()
    return xq, xd


def register_weights(qweights: np.ndarray, scales: np.ndarray, fmt: int) -> None:
    """asm_weights_register on host arrays (kept alive by the caller)."""
    scales = np.asarray(scales)
    if not (qweights.flags.c_contiguous and scales.flags.c_contiguous and scales.dtype == np.float32):
        raise ValueError("register_weights needs C-contiguous arrays and fp32 scales")
    M = scales.shape[0]
    K = scales.size // M * 32
    rc = native.lib().asm_weights_register(qweights.ctypes.data, scales.ctypes.data, M, K, fmt)
    native.check(rc)


def unregister_weights(qweights: np.ndarray) -> None:
    native.check(native.lib().asm_weights_unregister(qweights.ctypes.data))


def threadpool_init(num_threads: int) -> None:
    native.lib().asm_threadpool_init(int(num_threads))
    native.check()


def threadpool_shutdown() -> None:
    native.lib().asm_threadpool_shutdown()


def threadpool_get_num_threads() -> int:
    return int(native.lib().asm_threadpool_get_num_threads())


def max_k(fmt: int, fp32_activations: bool) -> int:
    return int(native.lib().asm_max_k(fmt, 1 if fp32_activations else 0))


# --------------------------------------------------------------------------
# Device (torch) layer
# --------------------------------------------------------------------------


def _torch():
    import torch  # imported lazily: the host layer needs no torch

    return torch


def _stream_handle(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _check_dev(t, dtypes, name):
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name}: expected a CUDA tensor")
    if t.dtype not in dtypes:
        raise TypeError(f"{name}: dtype {t.dtype} not in {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: tensor must be contiguous")


def matvec(fmt: int, qweights, scales, x, out=None, *, fp32_activations=False, stream=None, independent=False):
    """y = W x on device tensors.

    fmt: FMT_Q4_0 (qweights uint8 [M, K/32, 16]) or FMT_Q8_0 (int8 [M, K/32, 32]).
    scales: fp32 or fp16 [M, K/32].  fp32_activations selects the x86 (fp32-x)
    semantics instead of Q8_0-quantized activations (fp32 scales only).
    independent: the kernel enqueued just before this call neither writes x
    nor touches `out` (asm_matvec_ex_async with ASM_MV_INDEPENDENT), so the
    matvec may overlap it.
    """
    torch = _torch()
    wdt = torch.uint8 if fmt == FMT_Q4_0 else torch.int8
    _check_dev(qweights, (wdt,), "qweights")
    _check_dev(scales, (torch.float32, torch.float16), "scales")
    _check_dev(x, (torch.float32,), "x")
    M = scales.shape[0]
    K = x.shape[-1]
    if scales.numel() != M * (K // 32) or qweights.numel() != M * (K // 32) * (16 if fmt == FMT_Q4_0 else 32):
        raise ValueError(f"shape mismatch: qweights {tuple(qweights.shape)}, scales {tuple(scales.shape)}, K={K}")
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=x.device)
    else:
        _check_dev(out, (torch.float32,), "out")
    L = native.lib()
    f16 = scales.dtype == torch.float16
    st = _stream_handle(stream)
    args = (_ptr(qweights), _ptr(scales), _ptr(x), _ptr(out), M, K, st)
    if fp32_activations:
        if f16:
            raise ValueError("fp32-activation kernels take fp32 scales")
        rc = (L.asm_matmul_q4_f32_async if fmt == FMT_Q4_0 else L.asm_matmul_q8_async)(*args)
    elif independent:
        rc = L.asm_matvec_ex_async(fmt, _ptr(qweights), _ptr(scales), 1 if f16 else 0, _ptr(x), _ptr(out), M, K,
                                   MV_INDEPENDENT, st)
    elif fmt == FMT_Q4_0:
        rc = (L.asm_matmul_q4_f16s_async if f16 else L.asm_matmul_q4_async)(*args)
    else:
        rc = (L.asm_matmul_q8q8_f16s_async if f16 else L.asm_matmul_q8q8_async)(*args)
    native.check(rc)
    return out


def packed_row_bytes(fmt: int, K: int) -> int:
    """Bytes of one packed row (asm_packed_row_bytes); K a multiple of 256."""
    n = int(native.lib().asm_packed_row_bytes(fmt, int(K)))
    if n < 0:
        raise ValueError(f"no packed layout for fmt={fmt}, K={K} (K must be a multiple of 256)")
    return n


def pack_rows(fmt: int, qweights, scales_f16, out=None, stream=None):
    """Device qweights + fp16 scales -> packed rows uint8 [M, packed_row_bytes] (asm_pack_rows_async)."""
    torch = _torch()
    _check_dev(scales_f16, (torch.float16,), "scales")
    M, K = scales_f16.shape[0], scales_f16.shape[1] * 32
    if out is None:
        out = torch.empty((M, packed_row_bytes(fmt, K)), dtype=torch.uint8, device=qweights.device)
    native.check(native.lib().asm_pack_rows_async(fmt, _ptr(qweights), _ptr(scales_f16), _ptr(out), M, K,
                                                  _stream_handle(stream)))
    return out


def matvec_packed(fmt: int, packed, x, out=None, *, stream=None, independent=False):
    """y = W x on packed rows (asm_matvec_packed_async): Q4_0 / Q8_0 x Q8_0."""
    torch = _torch()
    _check_dev(packed, (torch.uint8,), "packed")
    _check_dev(x, (torch.float32,), "x")
    M, K = packed.shape[0], x.shape[-1]
    if packed.numel() != M * packed_row_bytes(fmt, K):
        raise ValueError(f"packed {tuple(packed.shape)} does not hold {M} rows of K={K}")
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=x.device)
    else:
        _check_dev(out, (torch.float32,), "out")
    native.check(native.lib().asm_matvec_packed_async(fmt, _ptr(packed), _ptr(x), _ptr(out), M, K,
                                                      MV_INDEPENDENT if independent else 0, _stream_handle(stream)))
    return out


def mark_static(*tensors) -> None:
    """Declares device tensors (model weights) static: see asm_weights_mark_static."""
    L = native.lib()
    for t in tensors:
        native.check(L.asm_weights_mark_static(_ptr(t), t.numel() * t.element_size()))


def unmark_static(*tensors) -> None:
    L = native.lib()
    for t in tensors:
        native.check(L.asm_weights_unmark_static(_ptr(t)))


def set_option(name: str, value: int) -> int:
    """asm_set_option: "tma" / "pdl" kernel-path switches, "image_min_k" (matvecs with
    K >= it quantize x in a pre-pass; 0 = never), "gemm_splits" (0 = automatic K split
    of the batched product, S = exactly S), "sync_map" (synchronous entries: bit 0 reads
    pinned host x in place, bit 1 writes pinned host y in place; default 3); returns the
    previous value."""
    prev = int(native.lib().asm_set_option(name.encode(), int(value)))
    if prev < 0:
        native.check()
    return prev


def device_error() -> int:
    """Reads and clears the device error word (0 = no kernel gave up a bounded wait)."""
    v = ctypes.c_uint(0)
    native.check(native.lib().asm_device_error(ctypes.byref(v)))
    return int(v.value)


def act_image_bytes(K: int) -> int:
    """Bytes of one row of the Q8_0 activation image (asm_act_image_bytes)."""
    n = int(native.lib().asm_act_image_bytes(int(K)))
    if n < 0:
        raise ValueError(f"K={K} is not a multiple of 32")
    return n


def act_image_dev(x, out=None, stream=None, prefetch=None):
    """Quantizes x fp32 [K] or [N, K] once into the activation image (uint8 [N, bytes]).

    prefetch: optional (qweights, scales) of the matvec that will read the
    image; their first bytes are streamed into L2 while the quantize waits for
    the previous kernel (a performance hint; results are unchanged)."""
    torch = _torch()
    _check_dev(x, (torch.float32,), "x")
    K = x.shape[-1]
    N = x.numel() // K if K else 0
    nbytes = act_image_bytes(K)
    if out is None:
        out = torch.empty((max(N, 1), nbytes), dtype=torch.uint8, device=x.device)
    L = native.lib()
    if prefetch is None:
        rc = L.asm_act_image_q8_0_async(_ptr(x), _ptr(out), N, K, _stream_handle(stream))
    else:
        w, s = prefetch
        rc = L.asm_act_image_q8_0_prefetch_async(_ptr(x), _ptr(out), N, K, _ptr(w), w.numel() * w.element_size(),
                                                 _ptr(s), s.numel() * s.element_size(), _stream_handle(stream))
    native.check(rc)
    return out


def matvec_image(fmt: int, qweights, scales, image, K: int, out=None, stream=None):
    """y = W x with x given as a prepared activation image (see act_image_dev)."""
    torch = _torch()
    wdt = torch.uint8 if fmt == FMT_Q4_0 else torch.int8
    _check_dev(qweights, (wdt,), "qweights")
    _check_dev(scales, (torch.float32, torch.float16), "scales")
    _check_dev(image, (torch.uint8,), "image")
    M = scales.shape[0]
    if image.numel() < act_image_bytes(K):
        raise ValueError("image too small for K")
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=image.device)
    rc = native.lib().asm_matmul_image_async(fmt, _ptr(qweights), _ptr(scales), 1 if scales.dtype == torch.float16 else 0,
                                             _ptr(image), _ptr(out), M, K, _stream_handle(stream))
    native.check(rc)
    return out


def quantize_q8_0_dev(x, xq=None, xd=None, stream=None):
    """Device quantize of x fp32 [N, K] or [K] -> (int8 same shape, fp32 [..., K/32])."""
    torch = _torch()
    _check_dev(x, (torch.float32,), "x")
    K = x.shape[-1]
    N = x.numel() // K if K else 0
    if xq is None:
        xq = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    if xd is None:
        xd = torch.empty((*x.shape[:-1], K // 32), dtype=torch.float32, device=x.device)
    rc = native.lib().asm_quantize_q8_0_async(_ptr(x), _ptr(xq), _ptr(xd), N, K, _stream_handle(stream))
    native.check(rc)
    return xq, xd


def block_sums_dev(fmt: int, qweights, scales, x, stream=None):
    """(y, isums int32 [M, K/32]) from the matvec kernel's own debug instantiation."""
    torch = _torch()
    M = scales.shape[0]
    K = x.shape[-1]
    y = torch.empty(M, dtype=torch.float32, device=x.device)
    isums = torch.empty((M, K // 32), dtype=torch.int32, device=x.device)
    rc = native.lib().asm_block_sums_async(fmt, _ptr(qweights), _ptr(scales), _ptr(x), _ptr(y),
                                           _ptr(isums), M, K, _stream_handle(stream))
    native.check(rc)
    return y, isums


def gguf_split_dev(fmt: int, raw, nblocks: int, scales_f16: bool = True, stream=None):
    """Split raw GGUF Q4_0 (18 B) / Q8_0 (34 B) blocks on the device.

    Returns (qs uint8/int8 [nblocks, 16|32], scales fp16|fp32 [nblocks]).
    Mirrors the reference's host split in src/runtime/generate.py:91-119.
    """
    torch = _torch()
    _check_dev(raw, (torch.uint8,), "raw")
    qb = 16 if fmt == FMT_Q4_0 else 32
    if raw.numel() < nblocks * (qb + 2):
        raise ValueError("raw buffer shorter than nblocks blocks")
    qs = torch.empty((nblocks, qb), dtype=torch.uint8 if fmt == FMT_Q4_0 else torch.int8, device=raw.device)
    scales = torch.empty(nblocks, dtype=torch.float16 if scales_f16 else torch.float32, device=raw.device)
    rc = native.lib().asm_gguf_split_async(fmt, _ptr(raw), _ptr(qs), _ptr(scales), 1 if scales_f16 else 0,
                                           nblocks, _stream_handle(stream))
    native.check(rc)
    return qs, scales


__all__ = [
    "AsmError", "FMT_Q4_0", "FMT_Q8_0",
    "matmul_q4", "matmul_q4_mt", "matmul_q4_avx512", "matmul_q4_f32", "matmul_q8", "matmul_q8_mt",
    "matmul_q8q8", "quantize_q8_0", "register_weights", "unregister_weights", "threadpool_init",
    "threadpool_shutdown", "threadpool_get_num_threads", "max_k", "matvec", "quantize_q8_0_dev",
    "block_sums_dev", "gguf_split_dev", "act_image_bytes", "act_image_dev", "matvec_image",
    "mark_static", "unmark_static", "device_error", "set_option",
]


def fused_matvec(fmt: int, qweights, scales, epilogue: int, *, y, x=None, image=None, norm_w=None,
                 eps: float = 1e-5, embed=None, x_copy=None, h=None, image_out=None, counters=None,
                 best=None, done=None, tokens=None, pos=None, vocab: int = 0, max_tokens: int = 0,
                 n_prompt: int = 0, stream=None):
    """One decode-step matvec with its prologue / epilogue fusion (asm_fused_matvec_async).

    epilogue: native.EPI_STORE, EPI_RESIDUAL (y += W x), EPI_SWIGLU (rows
    interleaved gate/up -> h and its Q8_0 image) or EPI_ARGMAX (y = logits,
    tokens[*pos + 1] = argmax, *pos += 1).  Scales must be fp16."""
    torch = _torch()
    _check_dev(scales, (torch.float16,), "scales")
    M, K = scales.shape[0], scales.shape[1] * 32
    d = native.FusedMatvec()
    d.fmt, d.epilogue, d.M, d.K, d.eps = fmt, epilogue, M, K, eps
    d.vocab, d.max_tokens, d.n_prompt = vocab, max_tokens, n_prompt
    for name, t in (("qweights", qweights), ("scales", scales), ("x", x), ("image", image), ("norm_w", norm_w),
                    ("embed", embed), ("x_copy", x_copy), ("y", y), ("h", h), ("image_out", image_out),
                    ("counters", counters), ("best", best), ("done", done), ("tokens", tokens), ("pos", pos)):
        if t is not None:
            setattr(d, name, t.data_ptr())
    native.check(native.lib().asm_fused_matvec_async(ctypes.byref(d), _stream_handle(stream)))
    return y


def attention_decode(qkv, k_cache, v_cache, rope_cs, pos, image_out, n_heads: int, n_kv_heads: int,
                     ctx: int, sqrt_head_dim: float, stream=None):
    """RoPE + fp16 KV append + attention at position *pos (asm_attention_decode_async)."""
    L = native.lib()
    rc = L.asm_attention_decode_async(_ptr(qkv), _ptr(k_cache), _ptr(v_cache), _ptr(rope_cs), _ptr(pos),
                                      _ptr(image_out), n_heads, n_kv_heads, 128, ctx, sqrt_head_dim,
                                      _stream_handle(stream))
    native.check(rc)
    return image_out


def gemm_image(fmt: int, qweights, scales, images, K: int, out=None, stream=None):
    """Y [N, M] = the matvec of every activation-image row (uint8 [N, bytes]), on the
    tensor cores (asm_gemm_image_async).  Scales fp16 [M, K/32]."""
    torch = _torch()
    wdt = torch.uint8 if fmt == FMT_Q4_0 else torch.int8
    _check_dev(qweights, (wdt,), "qweights")
    _check_dev(scales, (torch.float16,), "scales")
    _check_dev(images, (torch.uint8,), "images")
    M = scales.shape[0]
    N = images.shape[0]
    if out is None:
        out = torch.empty((N, M), dtype=torch.float32, device=images.device)
    rc = native.lib().asm_gemm_image_async(fmt, _ptr(qweights), _ptr(scales), _ptr(images), images.stride(0),
                                           _ptr(out), M, N, K, _stream_handle(stream))
    native.check(rc)
    return out


def gemm_narrow(fmt: int, qweights, scales, images, K: int, out=None, stream=None):
    """Y [N, M] for N <= 8 activation-image rows (uint8 [N, bytes]) on the CUDA cores,
    every weight byte read once for all N rows (asm_gemm_narrow_async); row n equals
    the warp-ring matvec of row n bit for bit.  Scales fp16 [M, K/32]."""
    torch = _torch()
    wdt = torch.uint8 if fmt == FMT_Q4_0 else torch.int8
    _check_dev(qweights, (wdt,), "qweights")
    _check_dev(scales, (torch.float16,), "scales")
    _check_dev(images, (torch.uint8,), "images")
    M = scales.shape[0]
    N = images.shape[0]
    if out is None:
        out = torch.empty((N, M), dtype=torch.float32, device=images.device)
    rc = native.lib().asm_gemm_narrow_async(fmt, _ptr(qweights), _ptr(scales), _ptr(images), images.stride(0),
                                            _ptr(out), M, N, K, _stream_handle(stream))
    native.check(rc)
    return out


def gemm(fmt: int, qweights, scales, X, out=None, stream=None, tiles=None):
    """Y [N, M] = W x_n for the N rows of X fp32 [N, K]: quantize every row to Q8_0
    into activation tiles (asm_rows_norm_tiles_async without a norm), then the
    tensor-core product (asm_gemm_tiles_async)."""
    torch = _torch()
    N, K = X.shape
    if tiles is None:
        tiles = torch.empty(act_tiles_bytes(N, K), dtype=torch.uint8, device=X.device)
    rows_norm_tiles(X, tiles, stream=stream)
    return gemm_tiles(fmt, qweights, scales, tiles, N, out=out, stream=stream)


def act_tiles_bytes(N: int, K: int) -> int:
    """Bytes of the activation tiles of N rows of K values (asm_act_tiles_bytes)."""
    n = int(native.lib().asm_act_tiles_bytes(N, K))
    if n <= 0:
        raise ValueError(f"no activation tiles for N={N}, K={K}")
    return n


def act_tiles_from_image(images, K: int, out=None, stream=None):
    """Activation tiles (uint8) of the N activation-image rows (asm_act_tiles_from_image_async)."""
    torch = _torch()
    _check_dev(images, (torch.uint8,), "images")
    N = images.shape[0]
    if out is None:
        out = torch.empty(act_tiles_bytes(N, K), dtype=torch.uint8, device=images.device)
    native.check(native.lib().asm_act_tiles_from_image_async(_ptr(images), images.stride(0), N, K, _ptr(out),
                                                             _stream_handle(stream)))
    return out


def gemm_tiles(fmt: int, qweights, scales, tiles, N: int, out=None, stream=None):
    """Y [N, M] from N rows of activation tiles on the tensor cores (asm_gemm_tiles_async)."""
    torch = _torch()
    wdt = torch.uint8 if fmt == FMT_Q4_0 else torch.int8
    _check_dev(qweights, (wdt,), "qweights")
    _check_dev(scales, (torch.float16,), "scales")
    _check_dev(tiles, (torch.uint8,), "tiles")
    M, K = scales.shape[0], scales.shape[1] * 32
    if tiles.numel() < act_tiles_bytes(N, K):
        raise ValueError("tiles buffer too small")
    if out is None:
        out = torch.empty((N, M), dtype=torch.float32, device=tiles.device)
    native.check(native.lib().asm_gemm_tiles_async(fmt, _ptr(qweights), _ptr(scales), _ptr(tiles), _ptr(out), M, N,
                                                   K, _stream_handle(stream)))
    return out


def rows_norm_tiles(x, tiles, norm_w=None, eps: float = 1e-5, delta=None, embed=None, tokens=None, pos=None,
                    stream=None):
    """asm_rows_norm_tiles_async on x fp32 [B, dim] (updated in place when embed or delta is given)."""
    d = native.Rows()
    d.rows, d.dim = x.shape[0], x.shape[1]
    d.eps = eps
    for name, t in (("x", x), ("delta", delta), ("embed", embed), ("tokens", tokens), ("pos", pos),
                    ("norm_w", norm_w), ("tiles", tiles)):
        if t is not None:
            setattr(d, name, t.data_ptr())
    if embed is not None:
        d.vocab, d.max_tokens = embed.shape[0], tokens.shape[1]
    native.check(native.lib().asm_rows_norm_tiles_async(ctypes.byref(d), _stream_handle(stream)))
    return tiles


def rows_swiglu_tiles(gu, tiles, stream=None):
    """asm_rows_swiglu_tiles_async: gu fp32 [B, 2*ffn] (gate/up pairs) -> tiles of h [B, ffn]."""
    native.check(native.lib().asm_rows_swiglu_tiles_async(_ptr(gu), gu.shape[0], gu.shape[1] // 2, _ptr(tiles),
                                                          _stream_handle(stream)))
    return tiles


def attention_batch(qkv, k_cache, v_cache, rope_cs, pos, tiles, n_heads: int, n_kv_heads: int, ctx: int,
                    sqrt_head_dim: float, stream=None):
    """asm_attention_batch_async: qkv fp32 [B, (nh + 2 nkv) * 128], caches fp16 [B, ctx, nkv, 128]."""
    rows = qkv.shape[0]
    native.check(native.lib().asm_attention_batch_async(
        _ptr(qkv), qkv.stride(0), _ptr(k_cache), _ptr(v_cache), k_cache.stride(0), _ptr(rope_cs), _ptr(pos),
        _ptr(tiles), rows, n_heads, n_kv_heads, 128, ctx, sqrt_head_dim, _stream_handle(stream)))
    return tiles


def rows_argmax(logits, keys, offset: int = 0, stream=None):
    """asm_rows_argmax_async: keys int64 [B] = signed-orderable (value, offset + index) maxima."""
    native.check(native.lib().asm_rows_argmax_async(_ptr(logits), logits.shape[0], logits.shape[1],
                                                    logits.stride(0), offset, _ptr(keys), _stream_handle(stream)))
    return keys


def rows_advance(keys, tokens, pos, n_prompt: int, stream=None):
    """asm_rows_advance_async: tokens[r][pos + 1] = argmax index of keys[r] after the prompt; pos += 1."""
    native.check(native.lib().asm_rows_advance_async(_ptr(keys), keys.shape[0], _ptr(tokens), tokens.shape[1],
                                                     _ptr(pos), n_prompt, _stream_handle(stream)))


def key_index(keys):
    """Index part of signed-orderable argmax keys (host or device int64 tensor)."""
    return ((keys ^ (-(1 << 63))) & 0xFFFFFFFF).neg().add(0xFFFFFFFF)
