"""GPU checks of the reference's decode-glue entry points (asm_rmsnorm,
asm_rope, asm_softmax, asm_attention, asm_silu_hadamard) and of
asm_threadpool_dispatch_q5, called through the C ABI with ctypes as the
reference's generation driver calls them (src/runtime/generate.py:221-316).

Bars: RMSNorm bit-exact against the reference's numpy outputs (numpy's
pairwise summation order is restated in the kernel); softmax, RoPE and
SiLU * up bit-exact against the restatement with float64 transcendentals
(oracle/glue_oracle.py), which itself is within a few ulps of numpy;
attention within the harness tolerance 1e-5 (its dot products follow BLAS
order in numpy)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import GOLDEN, rel_err

from oracle import glue_oracle as G

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L(cuda):
    from asmllm_b200 import native

    return native.lib()


def _check():
    from asmllm_b200 import native

    native.check()


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def rmsnorm(L, x, w, eps=1e-5):
    y = np.zeros_like(x)
    L.asm_rmsnorm(x.ctypes.data, w.ctypes.data, y.ctypes.data, x.shape[0], eps)
    _check()
    return y


def test_rmsnorm_is_bit_exact_vs_reference_numpy(L, golden):
    with np.load(GOLDEN / "decode_glue.npz") as d:  # dim 4096, the reference's ref_rmsnorm output
        assert np.array_equal(_bits(rmsnorm(L, d["norm_x"], d["norm_w"])), _bits(d["norm_y"]))
    y = rmsnorm(L, golden["rmsnorm_x"], golden["rmsnorm_weight"], float(golden["rmsnorm_eps"]))
    assert np.array_equal(_bits(y), _bits(golden["rmsnorm_expected"]))


@pytest.mark.parametrize("n", [1, 7, 8, 100, 129, 288, 1000, 11008, 28672, 65537])
def test_rmsnorm_matches_numpy_at_every_size_class(L, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    ref = ((x / np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + 1e-5)) * w).astype(np.float32)  # ops.py:114-115
    assert np.array_equal(_bits(rmsnorm(L, x, w)), _bits(ref))


def test_device_pointers_give_the_same_bits(L, cuda):
    torch = cuda
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 4096).astype(np.float32)
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    dy = torch.empty(4096, device="cuda")
    L.asm_rmsnorm(dx.data_ptr(), dw.data_ptr(), dy.data_ptr(), 4096, 1e-5)
    _check()
    assert np.array_equal(_bits(dy.cpu().numpy()), _bits(rmsnorm(L, x, w)))
    # mixed: host x, device y
    dy.zero_()
    L.asm_softmax(x.ctypes.data, dy.data_ptr(), 4096)
    _check()
    assert np.array_equal(_bits(dy.cpu().numpy()), _bits(G.softmax(x)))


def test_softmax_bit_exact_vs_restatement_and_close_to_numpy(L, golden):
    with np.load(GOLDEN / "decode_glue.npz") as d:
        cases = [(d["softmax_x"], d["softmax_y"]), (golden["softmax_x"], golden["softmax_expected"])]
    rng = np.random.default_rng(9)
    cases += [((rng.standard_normal(n) * 8).astype(np.float32), None) for n in (1, 5, 128, 129, 1025, 100000)]
    for x, ref in cases:
        y = np.zeros_like(x)
        L.asm_softmax(x.ctypes.data, y.ctypes.data, x.shape[0])
        _check()
        assert np.array_equal(_bits(y), _bits(G.softmax(x)))
        if ref is not None:
            assert np.max(np.abs(y - ref)) <= 1e-6 * float(np.max(ref))


def test_rope_bit_exact_vs_restatement_and_close_to_numpy(L, golden):
    with np.load(GOLDEN / "decode_glue.npz") as d:
        for i, p in enumerate(d["rope_pos"]):
            for h in range(d["rope_q"].shape[0]):
                q, k = d["rope_q"][h].copy(), d["rope_k"][h].copy()
                L.asm_rope(q.ctypes.data, k.ctypes.data, 128, int(p), 10000.0)
                _check()
                assert np.array_equal(_bits(q), _bits(G.rope(d["rope_q"][h], 128, int(p))))
                assert np.array_equal(_bits(k), _bits(G.rope(d["rope_k"][h], 128, int(p))))
                # numpy's fp32 pow is an ulp off for some frequencies; pos multiplies it
                tol = (int(p) + 1) * 3e-7 * float(np.abs(d["rope_q"][h]).max())
                assert np.max(np.abs(q - d["rope_q_out"][i, h])) <= tol
    q, k = golden["rope_q"].copy(), golden["rope_k"].copy()
    L.asm_rope(q.ctypes.data, k.ctypes.data, 32, int(golden["rope_pos"]), 10000.0)
    _check()
    assert np.max(np.abs(q - golden["rope_q_expected"])) <= 1e-5
    assert np.max(np.abs(k - golden["rope_k_expected"])) <= 1e-5


def test_silu_hadamard_bit_exact_vs_restatement(L):
    rng = np.random.default_rng(11)
    for n in (1, 33, 11008, 100003):
        gate = (rng.standard_normal(n) * 4).astype(np.float32)
        up = rng.standard_normal(n).astype(np.float32)
        g = gate.copy()
        L.asm_silu_hadamard(g.ctypes.data, up.ctypes.data, n)
        _check()
        assert np.array_equal(_bits(g), _bits(G.silu_hadamard(gate, up)))
        ref = (gate / (1.0 + np.exp(-gate))) * up  # generate.py:370 in numpy fp32
        assert np.max(np.abs(g - ref)) <= 2e-6 * max(1.0, float(np.abs(ref).max()))


def test_attention_within_harness_tolerance(L, golden):
    q, k, v = (np.ascontiguousarray(golden[f"attention_{n}"]) for n in "qkv")
    y = np.zeros_like(q)
    L.asm_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, y.ctypes.data, q.shape[0], q.shape[1],
                    1.0 / np.sqrt(q.shape[1]))
    _check()
    assert np.max(np.abs(y - golden["attention_expected"])) <= 1e-5
    rng = np.random.default_rng(13)
    for seq, hd in ((1, 128), (37, 64), (512, 128)):
        q, k, v = (rng.standard_normal((seq, hd)).astype(np.float32) for _ in range(3))
        y = np.zeros_like(q)
        L.asm_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, y.ctypes.data, seq, hd, 1.0 / np.sqrt(hd))
        _check()
        assert np.max(np.abs(y - G.attention(q, k, v, 1.0 / np.sqrt(hd)))) <= 1e-5


def test_glue_entries_report_bad_arguments(L):
    from asmllm_b200 import native

    q = np.zeros(6, dtype=np.float32)
    L.asm_rope(q.ctypes.data, q.ctypes.data, 5, 0, 10000.0)  # odd head_dim
    code, msg = native.last_error()
    assert code == 1 and "even" in msg
    L.asm_softmax(q.ctypes.data, q.ctypes.data, 0)
    assert native.last_error()[0] != 0
    L.asm_rmsnorm(None, None, None, 4, 1e-5)
    assert native.last_error()[0] == 1
    L.asm_silu_hadamard(q.ctypes.data, q.ctypes.data, 0)  # n = 0: nothing to do
    assert native.last_error()[0] == 0


def test_threadpool_dispatch_q5_equals_matmul_q5(L, golden):
    ql, qh, s, x = (np.ascontiguousarray(golden[f"q5_matmul_{n}"]) for n in ("ql", "qh", "scales", "x"))
    M, K = ql.shape[0], x.shape[0]
    y1, y2 = np.zeros(M, dtype=np.float32), np.zeros(M, dtype=np.float32)
    L.asm_matmul_q5(ql.ctypes.data, qh.ctypes.data, s.ctypes.data, x.ctypes.data, y1.ctypes.data, M, K)
    L.asm_threadpool_dispatch_q5(ql.ctypes.data, qh.ctypes.data, s.ctypes.data, x.ctypes.data, y2.ctypes.data, M, K)
    _check()
    assert np.array_equal(y1, y2)
    assert np.max(np.abs(y2 - golden["q5_matmul_expected"])) <= 1e-2  # test_runner.py:35


def test_forward_token_replayed_through_the_c_abi_matches_the_decode_oracle(L, cuda):
    """AsmEngineForward.forward_token (generate.py:261-326) call by call:
    asm_rmsnorm, three asm_matmul_q4, asm_rope per head, numpy attention
    scores with asm_softmax, asm_matmul_q4 (o), asm_rmsnorm, two asm_matmul_q4,
    asm_silu_hadamard, asm_matmul_q4 (down); host numpy buffers throughout, as
    the reference passes them.  Compared with the decode oracle's restatement
    of the same step (fp32 KV, the reference's), teacher-forced."""
    from asmllm_b200 import decode as D
    from oracle import decode_oracle as DO

    shape = D.LlamaShape(n_layers=2, dim=256, n_heads=2, n_kv_heads=2, head_dim=128, ffn=512, vocab=300)
    dec = D.LlamaDecoder(shape, ctx=16, seed=21)
    try:
        W = dec.host_weights()
    finally:
        dec.close()
    for Lw in W["layers"]:  # gate/up come de-interleaved as strided views: the C ABI wants contiguous rows
        for key in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
            Lw[key] = tuple(np.ascontiguousarray(a) for a in Lw[key])
    W["lm_head"] = tuple(np.ascontiguousarray(a) for a in W["lm_head"])
    nh, hd, dim, ffn = shape.n_heads, shape.head_dim, shape.dim, shape.ffn
    ctx = 16
    kc = [np.zeros((ctx, nh, hd), dtype=np.float32) for _ in range(shape.n_layers)]
    vc = [np.zeros((ctx, nh, hd), dtype=np.float32) for _ in range(shape.n_layers)]

    def mm(w, x, M, K):
        y = np.zeros(M, dtype=np.float32)
        L.asm_matmul_q4(w[0].ctypes.data, w[1].ctypes.data, np.ascontiguousarray(x).ctypes.data, y.ctypes.data, M, K)
        return y

    def forward_token(tok, pos):
        x = W["embed"][tok].astype(np.float32).copy()
        for li, Lw in enumerate(W["layers"]):
            xn = np.zeros_like(x)
            L.asm_rmsnorm(x.ctypes.data, Lw["attn_norm"].ctypes.data, xn.ctypes.data, dim, shape.eps)
            q, k, v = mm(Lw["wq"], xn, dim, dim), mm(Lw["wk"], xn, dim, dim), mm(Lw["wv"], xn, dim, dim)
            qh, kh = q.reshape(nh, hd), k.reshape(nh, hd)
            for h in range(nh):
                L.asm_rope(qh[h].ctypes.data, kh[h].ctypes.data, hd, pos, 10000.0)
            kc[li][pos], vc[li][pos] = kh, v.reshape(nh, hd)
            att = np.zeros((nh, hd), dtype=np.float32)
            for h in range(nh):
                scores = np.ascontiguousarray((qh[h] @ kc[li][:pos + 1, h].T) / np.sqrt(hd, dtype=np.float32))
                probs = np.zeros_like(scores)
                L.asm_softmax(scores.ctypes.data, probs.ctypes.data, pos + 1)
                att[h] = probs @ vc[li][:pos + 1, h]
            x += mm(Lw["wo"], att.reshape(-1), dim, dim)
            fn = np.zeros_like(x)
            L.asm_rmsnorm(x.ctypes.data, Lw["ffn_norm"].ctypes.data, fn.ctypes.data, dim, shape.eps)
            gate, up = mm(Lw["w_gate"], fn, ffn, dim), mm(Lw["w_up"], fn, ffn, dim)
            L.asm_silu_hadamard(gate.ctypes.data, up.ctypes.data, ffn)
            x += mm(Lw["w_down"], gate, dim, ffn)
        xn = np.zeros_like(x)
        L.asm_rmsnorm(x.ctypes.data, W["final_norm"].ctypes.data, xn.ctypes.data, dim, shape.eps)
        _check()
        return mm(W["lm_head"], xn, shape.vocab, dim)

    # the oracle with the reference's fp32 cache and RoPE table of this library's kernel
    W2 = dict(W)
    W2["rope"] = np.stack([np.stack(G.rope_table(hd, p, 10000.0), axis=1) for p in range(ctx)])
    orc = DO.DecodeOracle(shape, W2, ctx=ctx, kv_dtype=np.float32)
    seq = [3, 141, 59, 26, 53, 58, 97, 93]
    errs = []
    for pos, tok in enumerate(seq):
        errs.append(rel_err(forward_token(tok, pos), orc.forward_token(tok, pos)))
    # fp32 summation order only, unless a one-ulp difference moved a Q8_0 rounding (decode bars)
    assert max(errs) <= 2e-2 and min(errs) <= 1e-5, errs
