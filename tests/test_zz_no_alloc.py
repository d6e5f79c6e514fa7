"""The allocation-free Q4_0 x Q8_0 entry point, asm_matmul_q4_noalloc_async.

It exists for callers that cannot allocate device memory during a call: a
server that reserves all device memory at start-up, a serving loop with a
fixed memory budget, or a plugin whose host application owns every
allocation.  Its quantize scratch is a fixed device array inside the library
(K up to 32768).  These tests call it through the C ABI and check it against
the existing entry point (asm_matmul_q4_f16s_async via ops.matvec), on two
calls in a row, with the parity tolerance of the other tests.

The file is named to be collected last, so a run that stops at the first
failure has run every other test; it also passes on its own in a fresh
process (the first call there does the per-device set-up).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from asmllm_b200 import native, ops, synth
from asmllm_b200.native import FMT_Q4_0
from conftest import YTOL, rel_err

pytestmark = pytest.mark.gpu

MAX_K = 32768


def call_noalloc(torch, w, s, x, y, M, K):
    L = native.lib()
    return L.asm_matmul_q4_noalloc_async(
        ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(s.data_ptr()), 1 if s.dtype == torch.float16 else 0,
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), M, K,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("M,K,f16", [(4096, 11008, True), (11008, 4096, False), (257, 1024, True)])
def test_noalloc_matches_existing_entry_twice(cuda, M, K, f16):
    torch = cuda
    w, s = synth.q4_0_weights(M, K, seed=31)
    dw = torch.from_numpy(w).cuda()
    ds = torch.from_numpy(s).cuda()
    if f16:
        ds = ds.half()
    for seed in (32, 33):  # two calls in a row, each checked against the existing entry
        x = torch.from_numpy(synth.activation(K, seed=seed)).cuda()
        ref = ops.matvec(FMT_Q4_0, dw, ds, x)
        y = torch.full((M,), float("nan"), device="cuda")
        rc = call_noalloc(torch, dw, ds, x, y, M, K)
        assert rc == 0, native.last_error()
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= YTOL
        # the same quantized activation reaches the same matvec plan either way: bit for bit
        assert torch.equal(y, ref)
    assert ops.device_error() == 0


def test_noalloc_allocates_nothing_after_setup(cuda):
    torch = cuda
    M, K = 4096, 4096
    w, s = synth.q4_0_weights(M, K, seed=34)
    dw, ds = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half()
    x = torch.from_numpy(synth.activation(K, seed=35)).cuda()
    y = torch.empty(M, device="cuda")
    assert call_noalloc(torch, dw, ds, x, y, M, K) == 0  # first call: per-device set-up
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert call_noalloc(torch, dw, ds, x, y, M, K) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_rejects_k_beyond_its_scratch(cuda):
    torch = cuda
    M, K = 8, MAX_K + 32
    dw = torch.zeros((M, K // 32, 16), dtype=torch.uint8, device="cuda")
    ds = torch.zeros((M, K // 32), dtype=torch.float16, device="cuda")
    x = torch.zeros(K, device="cuda")
    y = torch.zeros(M, device="cuda")
    rc = call_noalloc(torch, dw, ds, x, y, M, K)
    code, msg = native.last_error()
    assert rc == native.ASM_E_UNSUPPORTED and code == native.ASM_E_UNSUPPORTED
    assert "32768" in msg
    assert not np.isnan(y.cpu().numpy()).any() and not y.cpu().numpy().any()  # y untouched
