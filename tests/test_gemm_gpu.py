"""Batched (prefill) Q4_0 / Q8_0 x Q8_0 product on the tensor cores
(asm_gemm_image_async: tcgen05.mma kind::f16 on the exact small integers,
per-32-block scales applied in fp32 from tensor memory).  Unsplit, every
output row is the matvec of one activation row with the reference's NEON
combine (blocks in order, acc = fma(float(isum), wd * xd, acc)), so it equals
the oracle bit for bit; split over S ranges of K, it equals the oracle's
chains over those ranges added in range order, also bit for bit."""
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


def oracle_split(oracle, fmt, w, s, X, S):
    """The split-K result: the blocks are cut into 128-byte weight stages (8 Q4_0
    or 4 Q8_0 blocks), stage range z = [z * nst // S, (z + 1) * nst // S); each
    range is an fma chain from zero and the partials are added in range order."""
    nb = s.shape[1]
    kb = 8 if fmt == FMT_Q4_0 else 4
    nst = -(-nb // kb)
    S = max(1, min(S, 8, nst))  # the library clamps the same way
    total = np.zeros((X.shape[0], w.shape[0]), dtype=np.float32)
    for z in range(S):
        b0, b1 = z * nst // S * kb, min((z + 1) * nst // S * kb, nb)
        part = oracle_rows(oracle, fmt, np.ascontiguousarray(w[:, b0:b1]), np.ascontiguousarray(s[:, b0:b1]),
                           np.ascontiguousarray(X[:, 32 * b0: 32 * b1]))
        total = (total + part).astype(np.float32)
    return total


@pytest.fixture
def splits():
    """Sets the "gemm_splits" option for one test and restores it."""
    prev = []

    def set_(v):
        prev.append(ops.set_option("gemm_splits", v))

    yield set_
    if prev:
        ops.set_option("gemm_splits", prev[0])


def run_gemm(torch, fmt, w, s, X):
    y = ops.gemm(fmt, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half(), torch.from_numpy(X).cuda())
    torch.cuda.synchronize()
    return y.cpu().numpy()


SHAPES = [(128, 64, 256), (300, 70, 288), (64, 8, 4096), (1000, 130, 1024), (4096, 64, 4096), (256, 16, 96),
          (130, 33, 11008)]


@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_unsplit_bit_exact_vs_oracle(cuda, oracle, splits, fmt, M, N, K):
    splits(1)
    w, s = weights(fmt, M, K, seed=80 + M)
    X = synth.activation(K, seed=81, n=N) * 2
    np.testing.assert_array_equal(run_gemm(cuda, fmt, w, s, X), oracle_rows(oracle, fmt, w, s, X))
    assert ops.device_error() == 0


@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
@pytest.mark.parametrize("S", [2, 3, 8])
@pytest.mark.parametrize("M,N,K", [(256, 16, 4096), (300, 70, 2048), (128, 128, 1024)])
def test_gemm_split_k_bit_exact_vs_oracle(cuda, oracle, splits, fmt, S, M, N, K):
    splits(S)
    w, s = weights(fmt, M, K, seed=60 + S)
    X = synth.activation(K, seed=61, n=N)
    np.testing.assert_array_equal(run_gemm(cuda, fmt, w, s, X), oracle_split(oracle, fmt, w, s, X, S))
    assert ops.device_error() == 0


@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
def test_gemm_automatic_split_is_deterministic_and_within_rounding(cuda, oracle, fmt):
    w, s = weights(fmt, 1024, 4096, seed=70)
    X = synth.activation(4096, seed=71, n=8)
    a = run_gemm(cuda, fmt, w, s, X)
    b = run_gemm(cuda, fmt, w, s, X)
    np.testing.assert_array_equal(a, b)
    ref = oracle_rows(oracle, fmt, w, s, X)
    assert np.abs(a - ref).max() <= 1e-5 * np.abs(ref).max()
    assert ops.device_error() == 0


@pytest.mark.parametrize("N", [8, 64, 512])
@pytest.mark.parametrize("M,K", [(4096, 4096), (11008, 4096), (4096, 11008)])
def test_gemm_7b_shapes_match_the_matvec(cuda, oracle, N, M, K):
    # the 7B prefill shapes of the benchmark config: every row against the GPU matvec
    # (1e-4 bound) and the first and last rows against the oracle
    torch = cuda
    w, s = weights(FMT_Q4_0, M, K, seed=90)
    X = synth.activation(K, seed=91, n=N)
    dw, ds, dX = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half(), torch.from_numpy(X).cuda()
    img = ops.act_image_dev(dX)
    y = ops.gemm_image(FMT_Q4_0, dw, ds, img, K).cpu().numpy()
    for n in range(0, N, max(1, N // 8)):
        ref = ops.matvec_image(FMT_Q4_0, dw, ds, img[n], K).cpu().numpy()
        assert np.abs(y[n] - ref).max() <= 1e-4 * np.abs(ref).max()
    for n in (0, N - 1):  # automatic K split: within fp32 rounding of the oracle
        ref = oracle.matmul_q4q8(w, s, X[n])
        assert np.abs(y[n] - ref).max() <= 1e-5 * np.abs(ref).max()
    assert ops.device_error() == 0


@pytest.mark.parametrize("M,K", [(10240, 8192), (57344, 8192)])
def test_gemm_70b_batch_shapes_match_the_matvec(cuda, M, K):
    # 70B batch-32 projections whose tile counts (80, 448) make the launch split K
    # over 3 and 2 cluster ranks to even out waves: rows against the GPU matvec
    # (1e-4 bound), and two calls give the same bits
    torch = cuda
    w, s = weights(FMT_Q4_0, M, K, seed=92)
    N = 32
    X = synth.activation(K, seed=93, n=N)
    dw, ds, dX = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half(), torch.from_numpy(X).cuda()
    img = ops.act_image_dev(dX)
    y = ops.gemm_image(FMT_Q4_0, dw, ds, img, K)
    y2 = ops.gemm_image(FMT_Q4_0, dw, ds, img, K)
    assert torch.equal(y, y2)
    y = y.cpu().numpy()
    for n in (0, 7, 19, 31):
        ref = ops.matvec_image(FMT_Q4_0, dw, ds, img[n], K).cpu().numpy()
        assert np.abs(y[n] - ref).max() <= 1e-4 * np.abs(ref).max()
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
