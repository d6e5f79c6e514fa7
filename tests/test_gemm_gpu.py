"""Batched (prefill) Q4_0 / Q8_0 x Q8_0 product on the tensor cores
(asm_gemm_image_async, tcgen05 kind::i8): every output row is the matvec of
one activation row with the reference's NEON combine (blocks in order,
acc = fma(float(isum), wd * xd, acc)), so it equals the oracle bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

from asmllm_b200 import native, ops, synth
from asmllm_b200.native import FMT_Q4_0, FMT_Q8_0

pytestmark = pytest.mark.gpu


def weights(fmt, M, K, seed):
    return (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=seed)


def oracle_rows(oracle, fmt, w, s, X):
    f = oracle.matmul_q4q8 if fmt == FMT_Q4_0 else oracle.matmul_q8q8
    return np.stack([f(w, s, x) for x in X])


@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
@pytest.mark.parametrize("M,N,K", [(128, 64, 256), (300, 70, 288), (64, 8, 4096), (1000, 130, 1024), (4096, 64, 4096)])
def test_gemm_bit_exact_vs_oracle(cuda, oracle, fmt, M, N, K):
    torch = cuda
    w, s = weights(fmt, M, K, seed=80 + M)
    X = synth.activation(K, seed=81, n=N) * 2
    y = ops.gemm(fmt, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half(), torch.from_numpy(X).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), oracle_rows(oracle, fmt, w, s, X))
    assert ops.device_error() == 0


@pytest.mark.parametrize("N", [8, 64, 512])
@pytest.mark.parametrize("M,K", [(4096, 4096), (11008, 4096), (4096, 11008)])
def test_gemm_7b_shapes_match_the_matvec(cuda, oracle, N, M, K):
    # the 7B prefill shapes of the benchmark config: every row against the GPU matvec
    # (1e-4 bound) and a few rows against the oracle (bit-exact)
    torch = cuda
    w, s = weights(FMT_Q4_0, M, K, seed=90)
    X = synth.activation(K, seed=91, n=N)
    dw, ds, dX = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half(), torch.from_numpy(X).cuda()
    img = ops.act_image_dev(dX)
    y = ops.gemm_image(FMT_Q4_0, dw, ds, img, K).cpu().numpy()
    for n in range(0, N, max(1, N // 8)):
        ref = ops.matvec_image(FMT_Q4_0, dw, ds, img[n], K).cpu().numpy()
        assert np.abs(y[n] - ref).max() <= 1e-4 * np.abs(ref).max()
    for n in (0, N - 1):
        np.testing.assert_array_equal(y[n], oracle.matmul_q4q8(w, s, X[n]))
    assert ops.device_error() == 0


def test_gemm_rejects_bad_arguments(cuda):
    torch = cuda
    w = torch.zeros((128, 8, 16), dtype=torch.uint8, device="cuda")
    s = torch.zeros((128, 8), dtype=torch.float16, device="cuda")
    img = torch.zeros((4, ops.act_image_bytes(256)), dtype=torch.uint8, device="cuda")
    L = native.lib()
    y = torch.zeros((4, 128), device="cuda")
    rc = L.asm_gemm_image_async(FMT_Q4_0, w.data_ptr(), s.data_ptr(), img.data_ptr(), 16, y.data_ptr(), 128, 4, 256,
                                None)
    assert rc == native.ASM_E_INVALID and "image_stride" in native.last_error()[1]
    rc = L.asm_gemm_image_async(3, w.data_ptr(), s.data_ptr(), img.data_ptr(), img.stride(0), y.data_ptr(), 128, 4,
                                256, None)
    assert rc == native.ASM_E_INVALID and "fmt 3" in native.last_error()[1]
