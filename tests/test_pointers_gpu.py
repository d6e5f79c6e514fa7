"""How the synchronous entries classify caller buffers (asm_pointer_kind):
the kind is asked of the driver on every call, so a buffer whose pinned
registration ended, or a device allocation that was freed, is seen as it is
now and never through a stale mapping.  Host-side queries only: nothing here
launches a kernel on a buffer whose state changed."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PAGEABLE, PINNED, DEVICE = 0, 1, 2


def kind(L, ptr):
    dev = ctypes.c_int(-2)
    return L.asm_pointer_kind(ptr, ctypes.byref(dev)), dev.value


def test_unregistered_host_buffer_is_classified_pageable_again(cuda):
    torch = cuda
    from asmllm_b200 import native

    L = native.lib()
    cudart = torch.cuda.cudart()
    buf = np.zeros(1 << 20, dtype=np.uint8)
    ptr = buf.ctypes.data
    assert kind(L, ptr) == (PAGEABLE, -1)
    assert int(cudart.cudaHostRegister(ptr, buf.nbytes, 0)) == 0
    try:
        k, dev = kind(L, ptr)
        assert k == PINNED and dev >= 0
        assert kind(L, ptr + 4096)[0] == PINNED  # an interior address of the registration
    finally:
        assert int(cudart.cudaHostUnregister(ptr)) == 0
    assert kind(L, ptr) == (PAGEABLE, -1)
    # and registered again: pinned again (no answer is remembered either way)
    assert int(cudart.cudaHostRegister(ptr, buf.nbytes, 0)) == 0
    try:
        assert kind(L, ptr)[0] == PINNED
    finally:
        cudart.cudaHostUnregister(ptr)
    assert kind(L, ptr)[0] == PAGEABLE


def test_device_and_pinned_tensors(cuda):
    torch = cuda
    from asmllm_b200 import native

    L = native.lib()
    d = torch.empty(1024, device="cuda")
    assert kind(L, d.data_ptr()) == (DEVICE, torch.cuda.current_device())
    h = torch.empty(1024).pin_memory()
    assert kind(L, h.data_ptr())[0] == PINNED
    p = np.zeros(1024, dtype=np.float32)
    assert kind(L, p.ctypes.data)[0] == PAGEABLE
    native.check()
