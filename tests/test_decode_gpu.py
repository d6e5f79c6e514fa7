"""Decode-step parity on the GPU: the fused matvec modes, the attention kernel
and whole batch-1 decode (asmllm_b200.decode.LlamaDecoder) against the CPU
restatement of the reference's forward_token (oracle/decode_oracle.py).

Bars: integer/byte work (KV append, argmax, token/position bookkeeping, the
Q8_0 image of a value the GPU produced) is bit-exact; a fused matvec whose
inputs quantize identically is bit-identical to the unfused kernel; float
results are within the stated tolerances.  Decode logits are compared with
teacher forcing (both sides consume the same tokens).  Steps agree to fp32
summation order (STEP_TOL * max|logit|) unless a one-ulp difference in a
normalised activation moved one Q8_0 rounding somewhere in the network, which
the quantized network carries forward (into the KV cache too): such steps
differ by up to DECODE_TOL * max|logit| -- on the 512-wide test models a
single moved rounding is worth up to ~1e-2, at 7B widths ~1e-3.  A systematic
error (RoPE, scaling, layout) would leave no step at STEP_TOL, so at least
one step must be there.
"""
from __future__ import annotations

import contextlib

import numpy as np
import pytest

from asmllm_b200 import decode as D
from asmllm_b200 import native, ops, synth
from asmllm_b200.native import FMT_Q4_0, FMT_Q8_0
from conftest import YTOL, rel_err

pytestmark = pytest.mark.gpu

DECODE_TOL = 2e-2
WIDE_DECODE_TOL = 5e-3
STEP_TOL = 1e-5
SMALL = D.LlamaShape(n_layers=2, dim=512, n_heads=4, n_kv_heads=4, head_dim=128, ffn=1536, vocab=1000)
SMALL_GQA = D.LlamaShape(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1536, vocab=1000)


def check_decode_errors(errs, tol=DECODE_TOL):
    assert max(errs) <= tol, errs
    assert min(errs) <= STEP_TOL, errs


@pytest.fixture(scope="module")
def DO(oracle):
    from oracle import decode_oracle
    return decode_oracle


def dev_weights(torch, fmt, M, K, seed):
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=seed)
    return torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half()


@contextlib.contextmanager
def row_stages():
    """Plain matvecs on the row-stage kernel: the kernel the fused decode-step
    matvecs take, so the comparisons below are of one summation order."""
    prev = ops.set_option("mv_kernel", 2)
    try:
        yield
    finally:
        ops.set_option("mv_kernel", prev)


def image_parts(img, nb):
    """(int8 values [nb, 32], (d, qsum) bytes [nb, 8]) of a Q8_0 activation image
    (the 16 pad bytes of each 48-byte slot carry nothing)."""
    raw = img.reshape(-1).cpu().numpy()
    return raw[: nb * 48].reshape(nb, 48)[:, :32].copy(), raw[nb * 48: nb * 56].reshape(nb, 8).copy()


def exact_inputs(K, seed):
    """x in multiples of 1/8 and w in 1 + multiples of 1/64: every sum of squares
    is exact, so the GPU's RMSNorm equals numpy's bit for bit."""
    rng = np.random.default_rng(seed)
    x = (rng.integers(-64, 65, K) / 8).astype(np.float32)
    w = (1 + rng.integers(-8, 9, K) / 64).astype(np.float32)
    return x, w


# ---------------------------------------------------------------- fused matvecs
@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
@pytest.mark.parametrize("M,K", [(1536, 512), (12288, 4096), (4096, 11008)])
def test_norm_prologue_equals_unfused_on_normed_x(cuda, DO, fmt, M, K):
    torch = cuda
    dw, ds = dev_weights(torch, fmt, M, K, seed=40)
    x, nw = exact_inputs(K, 41)
    xn = DO.rmsnorm(x, nw, 1e-5)
    with row_stages():
        y_plain = ops.matvec(fmt, dw, ds, torch.from_numpy(xn).cuda())
    y = torch.full((M,), float("nan"), device="cuda")
    ops.fused_matvec(fmt, dw, ds, native.EPI_STORE, x=torch.from_numpy(x).cuda(), norm_w=torch.from_numpy(nw).cuda(),
                     eps=1e-5, y=y)
    torch.cuda.synchronize()
    assert torch.equal(y, y_plain)
    assert ops.device_error() == 0


def test_norm_prologue_random_input_within_tolerance(cuda, DO, oracle):
    torch = cuda
    M, K = 12288, 4096
    w, s = synth.q4_0_weights(M, K, seed=42)
    x = 3 * synth.activation(K, seed=43)
    nw = (1 + 0.01 * synth.activation(K, seed=44)).astype(np.float32)
    y = torch.empty(M, device="cuda")
    ops.fused_matvec(FMT_Q4_0, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half(), native.EPI_STORE,
                     x=torch.from_numpy(x).cuda(), norm_w=torch.from_numpy(nw).cuda(), eps=1e-5, y=y)
    ref = oracle.matmul_q4q8(w, s, DO.rmsnorm(x, nw, 1e-5), M, K)
    assert rel_err(y.cpu().numpy(), ref) <= 10 * YTOL


@pytest.mark.parametrize("K", [4096, 11008])
def test_residual_epilogue(cuda, K):
    torch = cuda
    M = 4096
    dw, ds = dev_weights(torch, FMT_Q4_0, M, K, seed=45)
    x = torch.from_numpy(synth.activation(K, seed=46)).cuda()
    y0 = torch.from_numpy(100 * synth.activation(M, seed=47)).cuda()
    img = ops.act_image_dev(x)
    with row_stages():
        plain = ops.matvec_image(FMT_Q4_0, dw, ds, img, K)
        plain_x = ops.matvec(FMT_Q4_0, dw, ds, x)
    y = y0.clone()
    ops.fused_matvec(FMT_Q4_0, dw, ds, native.EPI_RESIDUAL, image=img, y=y)
    torch.cuda.synchronize()
    assert torch.equal(y, y0 + plain)
    y = y0.clone()
    ops.fused_matvec(FMT_Q4_0, dw, ds, native.EPI_RESIDUAL, x=x, y=y)  # quantizing prologue
    torch.cuda.synchronize()
    assert torch.equal(y, y0 + plain_x)


@pytest.mark.parametrize("ffn,K", [(1536, 512), (11008, 4096)])
def test_swiglu_epilogue(cuda, DO, ffn, K):
    torch = cuda
    gw, gs = dev_weights(torch, FMT_Q4_0, ffn, K, seed=48)
    uw, us = dev_weights(torch, FMT_Q4_0, ffn, K, seed=49)
    w = torch.stack([gw, uw], 1).reshape(2 * ffn, K // 32, 16).contiguous()
    s = torch.stack([gs, us], 1).reshape(2 * ffn, K // 32).contiguous()
    x, nw = exact_inputs(K, 50)
    dx, dnw = torch.from_numpy(x).cuda(), torch.from_numpy(nw).cuda()
    h = torch.full((ffn,), float("nan"), device="cuda")
    img = torch.zeros(ops.act_image_bytes(ffn), dtype=torch.uint8, device="cuda")
    counters = torch.zeros(ffn // 32, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the counters must come back to zero for the next launch
        ops.fused_matvec(FMT_Q4_0, w, s, native.EPI_SWIGLU, x=dx, norm_w=dnw, eps=1e-5, y=h, h=h, image_out=img,
                         counters=counters)
        torch.cuda.synchronize()
        assert not counters.any()
    xn = torch.from_numpy(DO.rmsnorm(x, nw, 1e-5)).cuda()
    g = ops.matvec(FMT_Q4_0, gw, gs, xn)
    u = ops.matvec(FMT_Q4_0, uw, us, xn)
    ref = (g / (1.0 + torch.exp(-g))) * u
    assert rel_err(h.cpu().numpy(), ref.cpu().numpy()) <= 1e-6
    # the image is the Q8_0 quantization of the GPU's own h, bit for bit
    got, want = image_parts(img, ffn // 32), image_parts(ops.act_image_dev(h), ffn // 32)
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[1], want[1])
    assert ops.device_error() == 0


def test_argmax_epilogue_token_and_position(cuda):
    torch = cuda
    M, K = 32000, 4096
    dw, ds = dev_weights(torch, FMT_Q4_0, M, K, seed=51)
    x = torch.from_numpy(synth.activation(K, seed=52)).cuda()
    nw = torch.ones(K, device="cuda")
    logits = torch.empty(M, device="cuda")
    best = torch.zeros(1, dtype=torch.int64, device="cuda")
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    tokens = torch.full((16,), -5, dtype=torch.int32, device="cuda")
    pos = torch.tensor([3], dtype=torch.int32, device="cuda")
    kw = dict(x=x, norm_w=nw, eps=1e-5, y=logits, best=best, done=done, tokens=tokens, pos=pos, max_tokens=16)
    ops.fused_matvec(FMT_Q4_0, dw, ds, native.EPI_ARGMAX, n_prompt=2, **kw)
    torch.cuda.synchronize()
    assert int(pos.item()) == 4 and best.item() == 0 and done.item() == 0
    assert int(tokens[4].item()) == int(torch.argmax(logits).item())
    # inside the prompt (p + 1 < n_prompt) the stored id is kept
    ops.fused_matvec(FMT_Q4_0, dw, ds, native.EPI_ARGMAX, n_prompt=8, **kw)
    torch.cuda.synchronize()
    assert int(pos.item()) == 5 and int(tokens[5].item()) == -5


def test_argmax_ties_pick_first_row(cuda):
    torch = cuda
    M, K = 1000, 512
    w = torch.full((M, K // 32, 16), 0x88, dtype=torch.uint8, device="cuda")  # every weight is 0
    s = torch.full((M, K // 32), 0.5, dtype=torch.float16, device="cuda")
    logits = torch.empty(M, device="cuda")
    tokens = torch.tensor([0, 77, 0, 0], dtype=torch.int32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.fused_matvec(FMT_Q4_0, w, s, native.EPI_ARGMAX, x=torch.ones(K, device="cuda"),
                     norm_w=torch.ones(K, device="cuda"), y=logits, best=torch.zeros(1, dtype=torch.int64, device="cuda"),
                     done=torch.zeros(1, dtype=torch.int32, device="cuda"), tokens=tokens, pos=pos, max_tokens=4)
    torch.cuda.synchronize()
    assert not logits.any() and int(tokens[1].item()) == 0 and int(pos.item()) == 1


def test_fused_rejects_bad_descriptors(cuda):
    torch = cuda
    dw, ds = dev_weights(torch, FMT_Q4_0, 96, 512, seed=53)
    y = torch.empty(96, device="cuda")
    with pytest.raises(native.AsmError, match="M % 64"):
        ops.fused_matvec(FMT_Q4_0, dw, ds, native.EPI_SWIGLU, x=torch.ones(512, device="cuda"), y=y,
                         h=y, image_out=torch.zeros(4096, dtype=torch.uint8, device="cuda"),
                         counters=torch.zeros(4, dtype=torch.int32, device="cuda"))
    with pytest.raises(native.AsmError, match="device pointer"):
        ops.fused_matvec(FMT_Q4_0, dw, ds, native.EPI_STORE, x=torch.ones(512), y=y)
    with pytest.raises(TypeError):
        ops.fused_matvec(FMT_Q4_0, dw, ds.float(), native.EPI_STORE, x=torch.ones(512, device="cuda"), y=y)


# ---------------------------------------------------------------- attention
@pytest.mark.parametrize("n_heads,n_kv,pos", [(32, 32, 0), (32, 32, 142), (8, 2, 37), (64, 8, 511)])
def test_attention_kernel(cuda, DO, oracle, n_heads, n_kv, pos):
    torch = cuda
    ctx, hd = 512, 128
    rng = np.random.default_rng(60 + pos)
    qkv = (3 * rng.standard_normal((n_heads + 2 * n_kv) * hd)).astype(np.float32)
    kc = np.zeros((ctx, n_kv, hd), np.float16)
    vc = np.zeros((ctx, n_kv, hd), np.float16)
    kc[:pos] = rng.standard_normal((pos, n_kv, hd)) * 3
    vc[:pos] = rng.standard_normal((pos, n_kv, hd))
    tab = D.rope_table(ctx, hd, 10000.0)
    dk, dv = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    img = torch.zeros(ops.act_image_bytes(n_heads * hd), dtype=torch.uint8, device="cuda")
    sqrt_hd = float(np.sqrt(np.float32(hd), dtype=np.float32))
    ops.attention_decode(torch.from_numpy(qkv).cuda(), dk, dv, torch.from_numpy(tab).cuda(),
                         torch.tensor([pos], dtype=torch.int32, device="cuda"), img, n_heads, n_kv, ctx, sqrt_hd)
    torch.cuda.synchronize()
    q = DO.rope(qkv[: n_heads * hd].reshape(n_heads, hd), tab[pos])
    k = DO.rope(qkv[n_heads * hd:(n_heads + n_kv) * hd].reshape(n_kv, hd), tab[pos])
    v = qkv[(n_heads + n_kv) * hd:].reshape(n_kv, hd)
    kc[pos], vc[pos] = k.astype(np.float16), v.astype(np.float16)
    # KV append: bit-exact (RoPE products rounded as numpy does, then fp16)
    np.testing.assert_array_equal(dk.cpu().numpy(), kc)
    np.testing.assert_array_equal(dv.cpu().numpy(), vc)
    g = n_heads // n_kv
    out = np.zeros((n_heads, hd), np.float32)
    for h in range(n_heads):
        K_ = kc[: pos + 1, h // g].astype(np.float32)
        V_ = vc[: pos + 1, h // g].astype(np.float32)
        out[h] = DO.softmax((q[h] @ K_.T) / np.float32(sqrt_hd)) @ V_
    out = out.reshape(-1)
    # the image: per block d within 1e-5 and int8 values within one step of
    # the oracle's quantization of the numpy output (most identical)
    nb = n_heads * hd // 32
    raw = img.cpu().numpy()
    gq = raw[: nb * 48].reshape(nb, 48)[:, :32].view(np.int8).astype(np.int32)
    gd = raw[nb * 48: nb * 56].view(np.float32).reshape(nb, 2)[:, 0]
    rq, rd = oracle.quantize_q8_0(out)
    rq = rq.reshape(nb, 32).astype(np.int32)
    np.testing.assert_allclose(gd, rd, rtol=1e-5, atol=0)
    assert np.abs(gq - rq).max() <= 1 and np.mean(gq != rq) < 0.01
    assert ops.device_error() == 0


# ---------------------------------------------------------------- whole decode
def step_logits(torch, dec, n):
    """n eager steps, the logits after each."""
    out = []
    for _ in range(n):
        dec.step()
        torch.cuda.synchronize()
        out.append(dec.logits.cpu().numpy().copy())
    return out


@pytest.mark.parametrize("shape", [SMALL, SMALL_GQA], ids=["mha", "gqa"])
def test_decode_matches_oracle_teacher_forced(cuda, DO, shape):
    torch = cuda
    dec = D.LlamaDecoder(shape, ctx=64, seed=11)
    try:
        prompt = [3, 141, 59, 26, 535]
        n_new = 12
        toks = dec.generate(prompt, n_new)
        dec.reset(prompt)
        gl = step_logits(torch, dec, len(prompt) - 1 + n_new)
        assert dec.tokens[len(prompt):len(prompt) + n_new].cpu().tolist() == toks
        orc = DO.DecodeOracle(shape, dec.host_weights(), ctx=64)
        otoks, ol = orc.generate(prompt, n_new, forced=toks)
        errs = [rel_err(a, b) for a, b in zip(gl, ol)]
        check_decode_errors(errs)
        # the GPU's choice is the oracle's argmax wherever the oracle's top-2 margin is clear
        for i, t in enumerate(toks):
            lg = ol[len(prompt) - 1 + i]
            top2 = np.sort(lg)[-2:]
            if top2[1] - top2[0] > 2 * DECODE_TOL * np.abs(lg).max():
                assert t == otoks[i]
        assert ops.device_error() == 0
    finally:
        dec.close()


def test_graph_replay_equals_eager_and_is_deterministic(cuda):
    torch = cuda
    dec = D.LlamaDecoder(SMALL, ctx=64, seed=12)
    try:
        prompt = [9, 8, 7]
        a = dec.generate(prompt, 20, chunk=16)  # 22 steps: one 16-step graph + 6 one-step graphs
        la = dec.logits.clone()
        b = dec.generate(prompt, 20, chunk=16)
        assert a == b and torch.equal(la, dec.logits)
        dec.reset(prompt)
        dec.step(len(prompt) - 1 + 20)
        torch.cuda.synchronize()
        assert dec.tokens[3:23].cpu().tolist() == a and torch.equal(la, dec.logits)
        assert dec.position() == 22
    finally:
        dec.close()


def test_decode_7b_shapes_two_layers_vs_oracle(cuda, DO):
    torch = cuda
    shape = D.LlamaShape(n_layers=2, dim=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000)
    dec = D.LlamaDecoder(shape, ctx=16, seed=13)
    try:
        prompt = [31999, 0, 12345]
        toks = dec.generate(prompt, 2)
        dec.reset(prompt)
        gl = step_logits(torch, dec, 4)
        orc = DO.DecodeOracle(shape, dec.host_weights(), ctx=16)
        _, ol = orc.generate(prompt, 2, forced=toks)
        errs = [rel_err(a, b) for a, b in zip(gl, ol)]
        check_decode_errors(errs, WIDE_DECODE_TOL)
    finally:
        dec.close()


def test_position_out_of_range_sets_error_and_skips(cuda):
    torch = cuda
    dec = D.LlamaDecoder(SMALL, ctx=8, seed=14)
    try:
        dec.generate([1, 2], 6)  # positions 0..6
        assert ops.device_error() == 0
        dec.step(2)  # positions 7 (last slot) and 8 (out of range: flagged, no access)
        torch.cuda.synchronize()
        err = ops.device_error()
        assert err & native.DEVERR_DECODE_RANGE
        assert ops.device_error() == 0  # read clears
        toks = dec.generate([1, 2], 3)  # the engine is usable afterwards
        assert len(toks) == 3 and ops.device_error() == 0
    finally:
        dec.close()


def test_sync_entry_reports_and_consumes_kernel_error_bits(cuda):
    # the synchronous entries learn of a kernel's error report through a mapped
    # host word (no copy back per call); the bits come from the device word
    torch = cuda
    rng = np.random.default_rng(3)
    M, K = 64, 256
    qw = rng.integers(0, 256, (M, K // 32, 16), dtype=np.uint8)
    sc = np.abs(rng.normal(0, 0.02, (M, K // 32))).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    y0 = ops.matmul_q4(qw, sc, x)  # also sets up the device state and its error word
    dec = D.LlamaDecoder(SMALL, ctx=8, seed=14)
    try:
        dec.generate([1, 2], 6)
        dec.step(2)  # position 8 is out of range: the argmax epilogue reports it
        torch.cuda.synchronize()
        with pytest.raises(native.AsmError, match="error bits 0x2"):
            ops.matmul_q4(qw, sc, x)
        assert ops.device_error() == 0  # consumed by the synchronous entry
        np.testing.assert_array_equal(ops.matmul_q4(qw, sc, x), y0)
        # bits already consumed through asm_device_error are not reported again
        dec.step(1)
        torch.cuda.synchronize()
        assert ops.device_error() & native.DEVERR_DECODE_RANGE
        np.testing.assert_array_equal(ops.matmul_q4(qw, sc, x), y0)
    finally:
        dec.close()


# ---------------------------------------------------------------- persistent engine
@pytest.mark.parametrize("shape", [SMALL, SMALL_GQA], ids=["mha", "gqa"])
def test_persistent_engine_agrees_with_per_launch_engine(cuda, shape):
    # The two engines add a row's block products in different fp32 orders
    # (the persistent kernel splits a row over two warps), so they agree to
    # fp32 rounding: compared teacher-forced on the same token sequence, each
    # engine bit-deterministic on its own.
    torch = cuda
    dec = D.LlamaDecoder(shape, ctx=64, seed=15)
    try:
        prompt = [5, 600, 7, 8]
        g = dec.generate(prompt, 14, engine="graph")
        seq = prompt + g  # every position teacher-forced (all of seq is "prompt")
        out = {}
        for eng in ("graph", "persistent", "persistent"):
            dec.reset(seq)
            dec.run(len(seq) - 1, engine=eng)
            torch.cuda.synchronize()
            lg, kc = dec.logits.clone(), dec.k_cache[:, :len(seq) - 1].float().clone()
            if eng in out:  # the same engine again: bit for bit
                assert torch.equal(lg, out[eng][0]) and torch.equal(kc, out[eng][1])
            out[eng] = (lg, kc)
        (lg_g, kc_g), (lg_p, kc_p) = out["graph"], out["persistent"]
        assert rel_err(lg_p.cpu().numpy(), lg_g.cpu().numpy()) <= DECODE_TOL
        assert rel_err(kc_p.cpu().numpy(), kc_g.cpu().numpy()) <= DECODE_TOL
        assert dec.position() == len(seq) - 1 and ops.device_error() == 0
        # persistent: the same steps split over several launches, bit for bit
        dec.reset(prompt)
        p = dec.generate(prompt, 14, engine="persistent")
        lp = dec.logits.clone()
        dec.reset(prompt)
        for n in (1, 4, 12):
            dec.run(n, engine="persistent")
        torch.cuda.synchronize()
        assert dec.tokens[4:18].cpu().tolist() == p and torch.equal(dec.logits, lp)
        assert not dec.best.any() and not dec.counters.any()
    finally:
        dec.close()


def test_persistent_engine_7b_shapes_matches_oracle(cuda, DO):
    torch = cuda
    shape = D.LlamaShape(n_layers=2, dim=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000)
    dec = D.LlamaDecoder(shape, ctx=16, seed=13)
    try:
        prompt = [31999, 0, 12345]
        toks = dec.generate(prompt, 3, engine="persistent")
        lg = dec.logits.cpu().numpy().copy()
        orc = DO.DecodeOracle(shape, dec.host_weights(), ctx=16)
        _, ol = orc.generate(prompt, 3, forced=toks)
        assert rel_err(lg, ol[-1]) <= WIDE_DECODE_TOL
        # the per-launch engine on the same (teacher-forced) sequence
        dec.reset(prompt + toks[:-1])
        dec.run(len(prompt) + 2, engine="graph")
        torch.cuda.synchronize()
        assert rel_err(dec.logits.cpu().numpy(), ol[-1]) <= WIDE_DECODE_TOL
        assert ops.device_error() == 0
    finally:
        dec.close()


def test_persistent_engine_refuses_runs_past_the_cache(cuda):
    torch = cuda
    dec = D.LlamaDecoder(SMALL, ctx=8, seed=16)
    try:
        dec.generate([1, 2], 3, engine="persistent")  # position 4 afterwards
        assert ops.device_error() == 0
        dec.run(5, engine="persistent")  # would need positions 4..8: refused on the device, nothing done
        torch.cuda.synchronize()
        assert ops.device_error() & native.DEVERR_DECODE_RANGE
        assert dec.position() == 4
        dec.run(3, engine="persistent")  # positions 4..6 fit (the last id lands in tokens[7])
        torch.cuda.synchronize()
        assert dec.position() == 7 and ops.device_error() == 0
    finally:
        dec.close()


def test_gguf_round_trip_decodes_identically(cuda, tmp_path):
    # the model written as GGUF (Q4_0 linear weights, F32 embedding and norms), read
    # back with one upload + device split per tensor, decodes bit for bit the same
    torch = cuda
    dec = D.LlamaDecoder(SMALL_GQA, ctx=32, seed=17)
    try:
        prompt = [4, 8, 15]
        toks = dec.generate(prompt, 6, engine="graph")
        lg = dec.logits.clone()
        toks_p = dec.generate(prompt, 6, engine="persistent")
        lg_p = dec.logits.clone()
        dec.to_gguf(tmp_path / "m.gguf")
    finally:
        dec.close()
    back = D.LlamaDecoder.from_gguf(tmp_path / "m.gguf", ctx=32)
    try:
        assert back.shape == SMALL_GQA and back.fmt == FMT_Q4_0
        assert back.generate(prompt, 6, engine="graph") == toks
        assert torch.equal(back.logits, lg)
        assert back.generate(prompt, 6, engine="persistent") == toks_p
        assert torch.equal(back.logits, lg_p)
    finally:
        back.close()
