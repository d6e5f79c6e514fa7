"""Packed rows (each row's quant blocks followed by its fp16 scales, one
contiguous range per stage): the matvec on them equals the matvec on the two
planes bit for bit -- every plan adds a row's block products in the same
order -- and both stay within the north star's bound of the oracle."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import YTOL, rel_err

pytestmark = pytest.mark.gpu

SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (1000, 256), (300, 8192), (64, 28672), (24, 14336)]


@pytest.mark.parametrize("fmt", [2, 8], ids=["q4_0", "q8_0"])
@pytest.mark.parametrize("M,K", SHAPES)
def test_packed_matvec_equals_plane_matvec(cuda, oracle, fmt, M, K):
    torch = cuda
    from asmllm_b200 import ops, synth

    if fmt == 2:
        w, s = synth.q4_0_weights(M, K, seed=M + K)
    else:
        w, s = synth.q8_0_weights(M, K, seed=M + K)
    x = synth.activation(K, seed=K)
    dw, ds, dx = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half(), torch.from_numpy(x).cuda()
    packed = ops.pack_rows(fmt, dw, ds)
    assert packed.shape == (M, ops.packed_row_bytes(fmt, K))
    # layout: row r = its quants, then its fp16 scales
    ub = 16 if fmt == 2 else 32
    r = M // 2
    row = packed[r].cpu().numpy()
    assert np.array_equal(row[: K // 32 * ub], w[r].reshape(-1).view(np.uint8))
    assert np.array_equal(row[K // 32 * ub:].view(np.float16), s[r].astype(np.float16))
    # the warp-ring kernel on both layouts (independent launches always take it)
    y_planes = ops.matvec(fmt, dw, ds, dx, independent=True).cpu().numpy()
    y_packed = ops.matvec_packed(fmt, packed, dx).cpu().numpy()
    y_indep = ops.matvec_packed(fmt, packed, dx, independent=True).cpu().numpy()
    # a dependent launch on planes: the row-stage kernel for rows of more than
    # 128 blocks (another fixed summation order), the warp-ring kernel otherwise
    y_dep = ops.matvec(fmt, dw, ds, dx).cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(y_packed, y_planes)
    assert np.array_equal(y_indep, y_planes)
    if K // 32 <= 128:
        assert np.array_equal(y_dep, y_planes)
    ref = oracle.matmul_q4q8(w, s, x) if fmt == 2 else oracle.matmul_q8q8(w, s, x)
    assert rel_err(y_packed, ref) <= YTOL
    assert rel_err(y_dep, ref) <= YTOL
    assert ops.device_error() == 0


def test_registered_weights_are_packed_and_agree(cuda, oracle):
    from asmllm_b200 import native, ops, synth

    M, K = 2048, 4096
    w, s = synth.q4_0_weights(M, K, seed=3)  # fp16-exact scales: registered as packed rows
    x = synth.activation(K, seed=4)
    y0 = ops.matmul_q4(w, s, x)
    ops.register_weights(w, s, native.FMT_Q4_0)
    try:
        y1 = ops.matmul_q4(w, s, x)
    finally:
        ops.unregister_weights(w)
    assert np.array_equal(y0, y1)
    assert rel_err(y1, oracle.matmul_q4q8(w, s, x)) <= YTOL


def test_packed_entry_rejects_unsupported_k(cuda):
    torch = cuda
    from asmllm_b200 import native

    L = native.lib()
    assert L.asm_packed_row_bytes(2, 4096) == 128 * 18
    assert L.asm_packed_row_bytes(2, 96) == -1
    p = torch.zeros(4 * 128, dtype=torch.uint8, device="cuda")
    x = torch.zeros(96, device="cuda")
    y = torch.zeros(4, device="cuda")
    assert L.asm_matvec_packed_async(2, p.data_ptr(), x.data_ptr(), y.data_ptr(), 4, 96, 0, None) == 1
    code, msg = native.last_error()
    assert code == 1 and "256" in msg
