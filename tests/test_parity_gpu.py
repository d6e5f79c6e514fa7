"""GPU parity: the sm_100a kernels against the CPU oracle, through the C ABI.

Bars (from the task's north star):
  * Q8_0 activation bytes and scales: bit-exact.
  * per-(row, block) int32 dot sums: bit-exact.
  * y: max |y - y_oracle| <= 1e-4 * ||y_oracle||_inf  (YTOL in conftest).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import refharness
from asmllm_b200 import native, ops, synth
from asmllm_b200.native import FMT_Q4_0, FMT_Q8_0
from conftest import YTOL, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["tma", "ldg"])
def kernel_path(request, cuda):
    """Runs a test on the bulk-copy pipeline kernel and on the register-streaming one."""
    prev = ops.set_option("tma", 1 if request.param == "tma" else 0)
    yield request.param
    ops.set_option("tma", prev)
    assert ops.device_error() == 0

SHAPES_SMALL = [(1, 32), (5, 64), (7, 96), (33, 4096), (129, 4096), (257, 1024), (1000, 11008)]
SHAPES_7B = list(synth.SHAPES_7B.values())


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def special_x(K):
    """Activation with every edge case of the quantize in some block."""
    x = synth.activation(K, seed=3).copy()
    nb = K // 32
    if nb >= 8:
        x[0:32] = 0.0                                     # zero block
        x[32:64] *= 1e-30                                 # tiny but normal
        x[64] = np.nan                                    # NaN block
        x[96] = np.inf                                    # inf block
        x[128:160] = np.float32(2.0) ** -127              # 127/amax overflows
        x[129] = -x[129]
        x[160:192] = np.linspace(-127, 127, 32).astype(np.float32)
        x[192:224] = np.array([62.5, 63.5, -2.5, 0.5, 1.5, 126.5, -0.5, 127.0] * 4, dtype=np.float32)
    return x


def assert_quant_equal(xq, xd, rq, rd):
    assert np.array_equal(xq, rq), f"{np.count_nonzero(xq != rq)} int8 values differ"
    nan_a, nan_b = np.isnan(xd), np.isnan(rd)
    assert np.array_equal(nan_a, nan_b)
    assert np.array_equal(xd[~nan_a].view(np.uint32), rd[~nan_b].view(np.uint32))


# --------------------------------------------------------------------------
# Drop-in contract: the reference harness's own checks on its fixture
# --------------------------------------------------------------------------

@pytest.mark.parametrize("kernel,tol", refharness.KERNELS)
def test_reference_harness(cuda, golden, kernel, tol):
    status, err = refharness.run_kernel_test(kernel, tol, golden, native.lib())
    assert status == "PASS", (kernel, err)


def test_reference_harness_fixture_matches_oracle(cuda, golden, oracle):
    # The drop-in asm_matmul_q4 is the NEON Q4_0 x Q8_0 semantics, not numpy's fp32-x.
    q, s, x = golden["q4_matmul_qweights"], golden["q4_matmul_scales"], golden["q4_matmul_x"]
    assert rel_err(ops.matmul_q4(q, s, x), oracle.matmul_q4q8(q, s, x)) <= YTOL
    assert rel_err(ops.matmul_q4_avx512(q, s, x), oracle.matmul_q4f32_avx512(q, s, x)) <= YTOL
    q8, s8 = golden["q8_matmul_qweights"], golden["q8_matmul_scales"]
    assert rel_err(ops.matmul_q8(q8, s8, x), oracle.matmul_q8f32_avx2(q8, s8, x)) <= YTOL
    assert rel_err(ops.matmul_q8q8(q8, s8, x), oracle.matmul_q8q8(q8, s8, x)) <= YTOL


# --------------------------------------------------------------------------
# Activation quantize: bit-exact
# --------------------------------------------------------------------------

@pytest.mark.parametrize("K", [32, 64, 256, 4096, 11008, 28672])
def test_quantize_bit_exact_device(cuda, oracle, K):
    x = special_x(K)
    rq, rd = oracle.quantize_q8_0(x)
    xq, xd = ops.quantize_q8_0_dev(dev(cuda, x))
    assert_quant_equal(xq.cpu().numpy(), xd.cpu().numpy(), rq, rd)


def test_quantize_bit_exact_host_abi(cuda, oracle):
    x = special_x(4096)
    rq, rd = oracle.quantize_q8_0(x)
    xq, xd = ops.quantize_q8_0(x)
    assert_quant_equal(xq, xd, rq, rd)


def test_quantize_batched_rows(cuda, oracle):
    X = synth.activation(4096, seed=7, n=8)
    X[3, :32] = 0.0
    xq, xd = ops.quantize_q8_0_dev(dev(cuda, X))
    for n in range(8):
        rq, rd = oracle.quantize_q8_0(X[n])
        assert_quant_equal(xq[n].cpu().numpy(), xd[n].cpu().numpy(), rq, rd)


def test_quantize_random_bulk(cuda, oracle):
    # 2^22 values from several scales: the quantize is exact on all of them.
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(1 << 22) * np.exp(rng.uniform(-30, 30, 1 << 22))).astype(np.float32)
    rq, rd = oracle.quantize_q8_0(x)
    xq, xd = ops.quantize_q8_0_dev(dev(cuda, x))
    assert_quant_equal(xq.cpu().numpy(), xd.cpu().numpy(), rq, rd)


def split_image(img, K):
    """(xq int8 [K], d fp32 [K/32], qsum int32 [K/32]) from one activation image row."""
    nb = K // 32
    raw = np.asarray(img, dtype=np.uint8).reshape(-1)
    xq = raw[: nb * 48].reshape(nb, 48)[:, :32].reshape(-1).view(np.int8)
    pairs = raw[nb * 48: nb * 56].view(np.uint32).reshape(nb, 2)
    return xq, pairs[:, 0].copy().view(np.float32), pairs[:, 1].copy().view(np.int32)


@pytest.mark.parametrize("K", [32, 64, 96, 4096, 11008, 28672])
def test_activation_image_bit_exact(cuda, oracle, K):
    x = special_x(K)
    rq, rd = oracle.quantize_q8_0(x)
    img = ops.act_image_dev(dev(cuda, x)).cpu().numpy()[0]
    assert img.size == ops.act_image_bytes(K) and img.size % 16 == 0
    xq, d, qsum = split_image(img, K)
    assert_quant_equal(xq, d, rq, rd)
    assert np.array_equal(qsum, oracle.block_qsum(rq))


def test_activation_image_batched(cuda, oracle):
    X = synth.activation(11008, seed=8, n=5)
    imgs = ops.act_image_dev(dev(cuda, X)).cpu().numpy()
    for n in range(5):
        xq, d, _ = split_image(imgs[n], 11008)
        rq, rd = oracle.quantize_q8_0(X[n])
        assert_quant_equal(xq, d, rq, rd)


@pytest.mark.parametrize("M,K", [(5, 64), (129, 4096), (4096, 11008), (32000, 4096)])
@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
def test_image_path_equals_fused_path(cuda, kernel_path, fmt, M, K):
    # Same int8 image either way, same kernel arithmetic: identical y.
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=13)
    x = synth.activation(K, seed=14)
    dw, ds, dx = dev(cuda, w), dev(cuda, s).half(), dev(cuda, x)
    y_fused = ops.matvec(fmt, dw, ds, dx)
    img = ops.act_image_dev(dx)
    y_img = ops.matvec_image(fmt, dw, ds, img, K)
    assert cuda.equal(y_fused, y_img)


# --------------------------------------------------------------------------
# Block sums: bit-exact (the matvec kernel's own debug instantiation)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("M,K", SHAPES_SMALL + [(4096, 4096)])
@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
def test_block_sums_bit_exact(cuda, oracle, kernel_path, fmt, M, K):
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=M + K)
    x = special_x(K) if K >= 256 else synth.activation(K, seed=2)
    xq, _ = oracle.quantize_q8_0(x)
    ref = (oracle.q4q8_block_sums if fmt == FMT_Q4_0 else oracle.q8q8_block_sums)(w, xq, M, K)
    _, isums = ops.block_sums_dev(fmt, dev(cuda, w), dev(cuda, s), dev(cuda, x))
    assert np.array_equal(isums.cpu().numpy(), ref)


# --------------------------------------------------------------------------
# Matvec outputs within 1e-4 * ||y||_inf
# --------------------------------------------------------------------------

def _oracle_y(oracle, fmt, fp32_act, w, s, x):
    if fmt == FMT_Q4_0:
        return (oracle.matmul_q4f32_avx2 if fp32_act else oracle.matmul_q4q8)(w, s, x)
    return (oracle.matmul_q8f32_avx2 if fp32_act else oracle.matmul_q8q8)(w, s, x)


@pytest.mark.parametrize("M,K", SHAPES_SMALL + SHAPES_7B)
@pytest.mark.parametrize("fmt,fp32_act", [(FMT_Q4_0, False), (FMT_Q8_0, False), (FMT_Q4_0, True), (FMT_Q8_0, True)])
def test_matvec_parity(cuda, oracle, kernel_path, fmt, fp32_act, M, K):
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=M * 7 + K)
    x = synth.activation(K, seed=K)
    ref = _oracle_y(oracle, fmt, fp32_act, w, s, x)
    dw, ds, dx = dev(cuda, w), dev(cuda, s), dev(cuda, x)
    y = ops.matvec(fmt, dw, ds, dx, fp32_activations=fp32_act).cpu().numpy()
    assert rel_err(y, ref) <= YTOL
    if not fp32_act:  # fp16 scale plane: same values, same result
        y16 = ops.matvec(fmt, dw, ds.half(), dx).cpu().numpy()
        assert np.array_equal(y16, y)


@pytest.mark.parametrize("M,K", [(129, 4096), (4096, 11008), (11008, 4096)])
@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
def test_static_weights_same_result(cuda, kernel_path, fmt, M, K):
    # Weights declared static are streamed before the previous kernel finishes;
    # the result must not change.  The preceding kernel here writes x.
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=17)
    x = synth.activation(K, seed=18)
    dw, ds, dx = dev(cuda, w), dev(cuda, s).half(), dev(cuda, x)
    cuda.cuda.synchronize()
    ref = ops.matvec(fmt, dw, ds, dx).clone()
    ops.mark_static(dw, ds)
    try:
        for _ in range(3):
            x2 = dx * 1.0  # a kernel right before the matvec (writes the activation)
            y = ops.matvec(fmt, dw, ds, x2)
            img = ops.act_image_dev(x2 * 1.0)
            y2 = ops.matvec_image(fmt, dw, ds, img, K)
            assert cuda.equal(y, ref) and cuda.equal(y2, ref)
    finally:
        ops.unmark_static(dw, ds)


@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
def test_matvec_edge_activations(cuda, oracle, kernel_path, fmt):
    M, K = 300, 4096
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=9)
    x = special_x(K)
    x[64] = 0.0  # drop the NaN block so y stays finite
    x[96] = 1.0  # and the inf block
    ref = _oracle_y(oracle, fmt, False, w, s, x)
    y = ops.matvec(fmt, dev(cuda, w), dev(cuda, s), dev(cuda, x)).cpu().numpy()
    assert rel_err(y, ref) <= YTOL


def test_nan_activation_propagates(cuda, oracle):
    M, K = 64, 128
    w, s = synth.q4_0_weights(M, K, seed=4)
    x = synth.activation(K)
    x[5] = np.nan
    ref = oracle.matmul_q4q8(w, s, x)
    y = ops.matvec(FMT_Q4_0, dev(cuda, w), dev(cuda, s), dev(cuda, x)).cpu().numpy()
    assert np.isnan(ref).all() and np.isnan(y).all()


def test_zero_k_gives_zero(cuda):
    y = ops.matmul_q4(np.zeros((3, 0, 16), np.uint8), np.zeros((3, 0), np.float32), np.zeros(0, np.float32))
    assert y.shape == (3,) and not y.any()


# --------------------------------------------------------------------------
# The synchronous ABI: host, device and registered pointers agree
# --------------------------------------------------------------------------

@pytest.mark.parametrize("fmt,name", [(FMT_Q4_0, "asm_matmul_q4"), (FMT_Q8_0, "asm_matmul_q8q8"),
                                      (FMT_Q4_0, "asm_matmul_q4_avx512"), (FMT_Q8_0, "asm_matmul_q8")])
def test_sync_abi_pointer_kinds(cuda, oracle, fmt, name):
    M, K = 4096, 4096
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=21)
    x = synth.activation(K, seed=22)
    L = native.lib()
    f = getattr(L, name)

    def call(pw, ps, px, py):
        f(pw, ps, px, py, M, K)
        native.check()

    y_host = np.zeros(M, np.float32)
    call(w.ctypes.data, s.ctypes.data, x.ctypes.data, y_host.ctypes.data)
    dw, ds, dx = dev(cuda, w), dev(cuda, s), dev(cuda, x)
    dy = cuda.zeros(M, dtype=cuda.float32, device="cuda")
    call(dw.data_ptr(), ds.data_ptr(), dx.data_ptr(), dy.data_ptr())
    assert np.array_equal(dy.cpu().numpy(), y_host)
    # pinned host x / y (the end-to-end path of the benchmark)
    px = cuda.from_numpy(x).pin_memory()
    py = cuda.zeros(M, dtype=cuda.float32).pin_memory()
    call(w.ctypes.data, s.ctypes.data, px.data_ptr(), py.data_ptr())
    assert np.array_equal(py.numpy(), y_host)
    # registered (resident) weights, fp16 scale plane
    ops.register_weights(w, s, fmt)
    try:
        y_reg = np.zeros(M, np.float32)
        call(w.ctypes.data, s.ctypes.data, x.ctypes.data, y_reg.ctypes.data)
        cnt = ctypes.c_int(0)
        assert L.asm_weights_resident_bytes(ctypes.byref(cnt)) > 0 and cnt.value == 1
        assert np.array_equal(y_reg, y_host)
    finally:
        ops.unregister_weights(w)
    fp32_act = name in ("asm_matmul_q4_avx512", "asm_matmul_q8")
    assert rel_err(y_host, _oracle_y(oracle, fmt, fp32_act, w, s, x)) <= YTOL


def test_mt_entries_and_threadpool(cuda, golden):
    ops.threadpool_init(8)
    assert ops.threadpool_get_num_threads() == 8
    q, s, x = golden["q4_matmul_qweights"], golden["q4_matmul_scales"], golden["q4_matmul_x"]
    assert np.array_equal(ops.matmul_q4_mt(q, s, x, 8), ops.matmul_q4(q, s, x))
    q8, s8 = golden["q8_matmul_qweights"], golden["q8_matmul_scales"]
    y8 = ops.matmul_q8(q8, s8, x)
    assert np.array_equal(ops.matmul_q8_mt(q8, s8, x, 3), y8)
    yd = np.zeros(4, np.float32)
    native.lib().asm_threadpool_dispatch_q8(q8.ctypes.data, s8.ctypes.data, x.ctypes.data, yd.ctypes.data, 4, 64)
    native.check()
    assert np.array_equal(yd, y8)
    ops.threadpool_shutdown()
    assert ops.threadpool_get_num_threads() == 0
    # usable again after shutdown
    assert np.array_equal(ops.matmul_q4(q, s, x), ops.matmul_q4_mt(q, s, x, 2))


def test_deterministic(cuda, kernel_path):
    M, K = 11008, 4096
    w, s = synth.q4_0_weights(M, K)
    x = synth.activation(K)
    dw, ds, dx = dev(cuda, w), dev(cuda, s), dev(cuda, x)
    a = ops.matvec(FMT_Q4_0, dw, ds, dx)
    b = ops.matvec(FMT_Q4_0, dw, ds, dx)
    assert cuda.equal(a, b)


# --------------------------------------------------------------------------
# Errors are reported, never launched
# --------------------------------------------------------------------------

def test_async_rejects_host_pointers(cuda):
    w, s = synth.q4_0_weights(8, 64)
    x = synth.activation(64)
    y = np.zeros(8, np.float32)
    rc = native.lib().asm_matmul_q4_async(w.ctypes.data, s.ctypes.data, x.ctypes.data, y.ctypes.data, 8, 64, None)
    assert rc == native.ASM_E_NOT_DEVICE
    native.last_error()


def test_misaligned_device_pointers_are_rejected(cuda):
    M, K = 16, 128
    dw = cuda.zeros(M * K // 2 + 16, dtype=cuda.uint8, device="cuda")
    ds = cuda.zeros(M * K // 32, dtype=cuda.float32, device="cuda")
    dx = cuda.zeros(K + 4, dtype=cuda.float32, device="cuda")
    dy = cuda.zeros(M, dtype=cuda.float32, device="cuda")
    L = native.lib()
    rc = L.asm_matmul_q4_async(dw.data_ptr() + 8, ds.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, None)
    assert rc == native.ASM_E_INVALID and "aligned" in native.last_error()[1]
    rc = L.asm_matmul_q4_async(dw.data_ptr(), ds.data_ptr(), dx.data_ptr() + 4, dy.data_ptr(), M, K, None)
    assert rc == native.ASM_E_INVALID and "aligned" in native.last_error()[1]
    L.asm_matmul_q4(dw.data_ptr(), ds.data_ptr(), dx.data_ptr() + 4, dy.data_ptr(), M, K)
    assert native.last_error()[0] == native.ASM_E_INVALID
    cuda.cuda.synchronize()


def test_k_beyond_maximum_is_rejected(cuda):
    kmax = ops.max_k(FMT_Q4_0, False)
    assert kmax >= 131072 - 32
    K = kmax + 32
    dw = cuda.zeros((1, K // 32, 16), dtype=cuda.uint8, device="cuda")
    ds = cuda.zeros((1, K // 32), dtype=cuda.float32, device="cuda")
    dx = cuda.zeros(K, dtype=cuda.float32, device="cuda")
    with pytest.raises(native.AsmError) as e:
        ops.matvec(FMT_Q4_0, dw, ds, dx)
    assert e.value.code == native.ASM_E_UNSUPPORTED


# --------------------------------------------------------------------------
# GGUF block split (reference generate.py:91-119)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
@pytest.mark.parametrize("f16", [True, False])
def test_gguf_split(cuda, fmt, f16):
    M, K = 77, 4096
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=5)
    raw = synth.gguf_blocks(w, s)
    nblk = M * (K // 32)
    qs, sc = ops.gguf_split_dev(fmt, dev(cuda, raw), nblk, scales_f16=f16)
    assert np.array_equal(qs.cpu().numpy().reshape(w.shape), w)
    assert np.array_equal(sc.float().cpu().numpy().reshape(s.shape), s)


# --------------------------------------------------------------------------
# Q5_0 x fp32 (asm_matmul_q5, row f4)
# --------------------------------------------------------------------------

def q5_weights(M, K, seed):
    rng = np.random.default_rng(seed)
    ql = rng.integers(0, 256, (M, K // 32, 16), dtype=np.uint8)
    qh = rng.integers(0, 256, (M, K // 32, 4), dtype=np.uint8)
    s = np.abs(rng.standard_normal((M, K // 32), dtype=np.float32) * np.float32(0.02))
    return ql, qh, s.astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("M,K", [(1, 32), (37, 96), (4096, 4096), (11008, 4096), (4096, 11008)])
def test_q5_matvec_matches_oracle(cuda, oracle, M, K):
    torch = cuda
    ql, qh, s = q5_weights(M, K, seed=70 + M)
    x = synth.activation(K, seed=71)
    ref = oracle.matmul_q5f32_avx2(ql, qh, s, x)
    y = native_q5_dev(torch, ql, qh, s, x)
    assert rel_err(y, ref) <= YTOL
    yh = np.zeros(M, dtype=np.float32)  # synchronous entry, host buffers
    native.lib().asm_matmul_q5(ql.ctypes.data, qh.ctypes.data, s.ctypes.data, x.ctypes.data, yh.ctypes.data, M, K)
    native.check()
    assert rel_err(yh, ref) <= YTOL


def native_q5_dev(torch, ql, qh, s, x):
    dl, dh, ds, dx = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (ql, qh, s, x))
    y = torch.full((ql.shape[0],), float("nan"), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = native.lib().asm_matmul_q5_async(dl.data_ptr(), dh.data_ptr(), ds.data_ptr(), dx.data_ptr(), y.data_ptr(),
                                          ql.shape[0], x.shape[0], st)
    native.check(rc)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_q5_rejects_bad_arguments(cuda):
    torch = cuda
    ql = torch.zeros((4, 1, 16), dtype=torch.uint8, device="cuda")
    x = torch.zeros(32, device="cuda")
    y = torch.zeros(4, device="cuda")
    L = native.lib()
    rc = L.asm_matmul_q5_async(ql.data_ptr(), ql.data_ptr() + 1, x.data_ptr(), x.data_ptr(), y.data_ptr(), 4, 32, None)
    assert rc == native.ASM_E_INVALID and "aligned" in native.last_error()[1]
    rc = L.asm_matmul_q5_async(ql.data_ptr(), ql.data_ptr(), x.data_ptr(), x.data_ptr(), y.data_ptr(), 4, 33, None)
    assert rc == native.ASM_E_INVALID and "K=33" in native.last_error()[1]


@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
def test_long_k_prepass_equals_fused_prologue(cuda, fmt):
    # K >= "image_min_k": x is quantized once by a pre-pass kernel instead of in every CTA;
    # the image bytes are the same, so y is bit-identical
    torch = cuda
    M, K = 300, 11008
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=17)
    dw, ds = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half()
    x = torch.from_numpy(synth.activation(K, seed=18)).cuda()
    prev = ops.set_option("image_min_k", 0)
    try:
        a = ops.matvec(fmt, dw, ds, x)
        ops.set_option("image_min_k", 8192)
        b = ops.matvec(fmt, dw, ds, x)
    finally:
        ops.set_option("image_min_k", prev)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    # the pre-pass scratch comes from the library's pool eagerly and from graph
    # memory under stream capture: both give the same bytes
    out = torch.empty_like(b)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.matvec(fmt, dw, ds, x, out=out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, b)
    for _ in range(3):  # eager calls with a synchronize between them reuse the pool
        c = ops.matvec(fmt, dw, ds, x)
        torch.cuda.synchronize()
        assert torch.equal(c, b)
    del g
    assert ops.device_error() == 0


@pytest.mark.parametrize("mapping", [0, 1, 2, 3])
@pytest.mark.parametrize("M,K", [(1000, 4096), (4096, 11008)])
def test_sync_abi_pinned_buffers_used_in_place(cuda, M, K, mapping):
    # pinned host x / y go to the kernels as mapped host memory (no staging
    # copies; option "sync_map" bit 0 = x, bit 1 = y); every choice equals
    # the staged (pageable) path bit for bit
    torch = cuda
    w, s = synth.q4_0_weights(M, K, seed=21)
    x = synth.activation(K, seed=22)
    hx = torch.from_numpy(x.copy()).pin_memory()
    hy = torch.zeros(M, dtype=torch.float32).pin_memory()
    prev = ops.set_option("sync_map", mapping)
    try:
        native.lib().asm_matmul_q4(w.ctypes.data, s.ctypes.data, hx.data_ptr(), hy.data_ptr(), M, K)
        native.check()
    finally:
        ops.set_option("sync_map", prev)
    np.testing.assert_array_equal(hy.numpy(), ops.matmul_q4(w, s, x))
