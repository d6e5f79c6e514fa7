"""Batched decode on the GPU (asmllm_b200.batch_decode.BatchDecoder): the
activation tiles, the per-row glue kernels and whole batched decode against
the CPU restatement of the reference's forward_token (oracle/decode_oracle.py),
one oracle per sequence.

Bars: layout and integer work (tiles from an image, argmax keys, token and
position bookkeeping, attention whose arithmetic is the batch-1 kernel's) is
bit-exact; RMSNorm + quantize agrees with the oracle's quantize of the
oracle's RMSNorm to one Q8_0 step; decode logits follow the batch-1 decode
tolerances (see tests/test_decode_gpu.py) with teacher forcing."""
from __future__ import annotations

import numpy as np
import pytest

from asmllm_b200 import batch_decode as BD
from asmllm_b200 import decode as D
from asmllm_b200 import ops, synth
from asmllm_b200.native import FMT_Q4_0, FMT_Q8_0
from conftest import rel_err

pytestmark = pytest.mark.gpu

DECODE_TOL = 2e-2
STEP_TOL = 1e-5
SMALL_GQA = D.LlamaShape(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1536, vocab=1000)
PERM = np.array([4 * c + j for c in range(4) for j in (0, 2, 1, 3, 16, 18, 17, 19)])


@pytest.fixture(scope="module")
def DO(oracle):
    from oracle import decode_oracle
    return decode_oracle


def tiles_expected(q, d, np_):
    """Activation tiles (bytes) from int8 quants q [N, nb, 32] and scales d [N, nb] (numpy)."""
    N, nb, _ = q.shape
    plane = np.zeros((nb, np_ // 8, 4, 8, 8), dtype=np.float16)  # [b][n/8][k/8][n%8][k%8]
    for n in range(N):
        v = q[n][:, PERM].astype(np.float16).reshape(nb, 4, 8)
        plane[:, n // 8, :, n % 8, :] = v
    dpl = np.zeros((nb, np_), dtype=np.float32)
    dpl[:, :N] = d.T
    return np.concatenate([plane.reshape(-1).view(np.uint8), dpl.reshape(-1).view(np.uint8)])


def tiles_parts(raw, N, nb, np_):
    """(quants [N, nb, 32] in element order, scales [N, nb]) read back from tile bytes."""
    plane = raw[: nb * np_ * 64].view(np.float16).reshape(nb, np_ // 8, 4, 8, 8)
    q = np.zeros((N, nb, 32), dtype=np.float32)
    for n in range(N):
        q[n][:, PERM] = plane[:, n // 8, :, n % 8, :].reshape(nb, 32)
    d = raw[nb * np_ * 64:].view(np.float32).reshape(nb, np_)[:, :N].T
    return q, d


@pytest.mark.parametrize("N,K", [(1, 256), (5, 4096), (16, 512), (33, 1024), (130, 288)])
def test_tiles_from_image_layout(cuda, oracle, N, K):
    torch = cuda
    X = synth.activation(K, seed=N, n=N) * 3
    img = ops.act_image_dev(torch.from_numpy(X).cuda())
    tiles = ops.act_tiles_from_image(img, K).cpu().numpy()
    qd = [oracle.quantize_q8_0(x) for x in X]
    q = np.stack([a.reshape(-1, 32) for a, _ in qd])
    d = np.stack([b for _, b in qd])
    np_ = ops.act_tiles_bytes(N, K) // (K // 32) // 68
    np.testing.assert_array_equal(tiles, tiles_expected(q, d, np_))


@pytest.mark.parametrize("fmt", [FMT_Q4_0, FMT_Q8_0])
def test_gemm_tiles_equals_gemm_image(cuda, fmt):
    torch = cuda
    M, K, N = 384, 1024, 40
    w, s = (synth.q4_0_weights if fmt == FMT_Q4_0 else synth.q8_0_weights)(M, K, seed=5)
    dw, ds = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half()
    img = ops.act_image_dev(torch.from_numpy(synth.activation(K, seed=6, n=N)).cuda())
    a = ops.gemm_image(fmt, dw, ds, img, K)
    b = ops.gemm_tiles(fmt, dw, ds, ops.act_tiles_from_image(img, K), N)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert ops.device_error() == 0


@pytest.mark.parametrize("mode", ["norm", "delta", "embed", "plain"])
def test_rows_norm_tiles(cuda, oracle, DO, mode):
    torch = cuda
    B, dim, vocab, P = 6, 1024, 50, 4
    rng = np.random.default_rng(7)
    x = rng.standard_normal((B, dim)).astype(np.float32)
    delta = rng.standard_normal((B, dim)).astype(np.float32)
    emb = rng.standard_normal((vocab, dim)).astype(np.float32)
    w = (1 + 0.01 * rng.standard_normal(dim)).astype(np.float32)
    tokens = rng.integers(0, vocab, (B, P)).astype(np.int32)
    pos = 2
    dx = torch.from_numpy(x).cuda()
    tiles = torch.zeros(ops.act_tiles_bytes(B, dim), dtype=torch.uint8, device="cuda")
    kw = {}
    if mode == "delta":
        kw["delta"] = torch.from_numpy(delta).cuda()
        src = (x + delta).astype(np.float32)
    elif mode == "embed":
        kw.update(embed=torch.from_numpy(emb).cuda(), tokens=torch.from_numpy(tokens).cuda(),
                  pos=torch.tensor([pos], dtype=torch.int32, device="cuda"))
        src = emb[tokens[:, pos]]
    else:
        src = x
    norm = None if mode == "plain" else torch.from_numpy(w).cuda()
    ops.rows_norm_tiles(dx, tiles, norm, 1e-5, **kw)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dx.cpu().numpy(), src)  # the residual stream as updated
    q, d = tiles_parts(tiles.cpu().numpy(), B, dim // 32, ops.act_tiles_bytes(B, dim) // (dim // 32) // 68)
    ref = src if mode == "plain" else np.stack([DO.rmsnorm(r, w, 1e-5) for r in src])
    got = (q * d[:, :, None]).reshape(B, dim)
    # the quantize of a value within fp32 summation order of the oracle's norm: one Q8_0 step at most
    assert np.all(np.abs(got - ref) <= np.repeat(d, 32, axis=1) * 1.0001 + 1e-7)
    if mode == "plain":  # no norm: the quantize itself is bit-exact
        for r in range(B):
            rq, rd = oracle.quantize_q8_0(src[r])
            np.testing.assert_array_equal(q[r].reshape(-1), rq.astype(np.float32))
            np.testing.assert_array_equal(d[r], rd)
    assert ops.device_error() == 0


def test_rows_swiglu_tiles(cuda, oracle):
    torch = cuda
    B, ffn = 3, 1536
    gu = np.random.default_rng(8).standard_normal((B, 2 * ffn)).astype(np.float32) * 3
    tiles = torch.zeros(ops.act_tiles_bytes(B, ffn), dtype=torch.uint8, device="cuda")
    ops.rows_swiglu_tiles(torch.from_numpy(gu).cuda(), tiles)
    torch.cuda.synchronize()
    g, u = gu[:, 0::2], gu[:, 1::2]
    h = ((g / (np.float32(1.0) + np.exp(-g))) * u).astype(np.float32)
    q, d = tiles_parts(tiles.cpu().numpy(), B, ffn // 32, 16)
    got = (q * d[:, :, None]).reshape(B, ffn)
    assert np.all(np.abs(got - h) <= np.repeat(d, 32, axis=1) * 1.0001 + 1e-7)
    assert ops.device_error() == 0


def test_attention_batch_equals_batch1_kernel(cuda):
    torch = cuda
    B, nh, nkv, ctx, pos = 3, 8, 2, 64, 37
    hd = 128
    rng = np.random.default_rng(9)
    qkv = torch.from_numpy(rng.standard_normal((B, (nh + 2 * nkv) * hd)).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.standard_normal((B, ctx, nkv, hd)).astype(np.float16)).cuda()
    vc = torch.from_numpy(rng.standard_normal((B, ctx, nkv, hd)).astype(np.float16)).cuda()
    kc1, vc1 = kc.clone(), vc.clone()
    rope = torch.from_numpy(D.rope_table(ctx, hd, 10000.0)).cuda()
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    sq = float(np.sqrt(np.float32(hd), dtype=np.float32))
    tiles = torch.zeros(ops.act_tiles_bytes(B, nh * hd), dtype=torch.uint8, device="cuda")
    ops.attention_batch(qkv, kc, vc, rope, p, tiles, nh, nkv, ctx, sq)
    imgs = torch.zeros((B, ops.act_image_bytes(nh * hd)), dtype=torch.uint8, device="cuda")
    for r in range(B):
        ops.attention_decode(qkv[r], kc1[r], vc1[r], rope, p, imgs[r], nh, nkv, ctx, sq)
    ref = ops.act_tiles_from_image(imgs, nh * hd)
    torch.cuda.synchronize()
    assert torch.equal(tiles, ref)
    assert torch.equal(kc, kc1) and torch.equal(vc, vc1)  # the same K/V appended at pos
    assert ops.device_error() == 0


def test_rows_argmax_and_advance(cuda):
    torch = cuda
    B, V, P, T = 4, 3000, 3, 10
    rng = np.random.default_rng(10)
    lg = rng.standard_normal((B, V)).astype(np.float32)
    lg[1, 17] = lg[1, 2999] = 50.0  # ties: the first index wins
    lg[2, 5] = np.nan  # NaN is ignored
    dl = torch.from_numpy(lg).cuda()
    keys = torch.zeros(B, dtype=torch.int64, device="cuda")
    ops.rows_argmax(dl, keys, offset=100)
    idx = ops.key_index(keys).cpu().numpy()
    ref = np.array([np.nanargmax(r) for r in lg]) + 100
    np.testing.assert_array_equal(idx, ref)
    # two vocabulary halves combine with an int64 max
    k0 = torch.zeros(B, dtype=torch.int64, device="cuda")
    k1 = torch.zeros(B, dtype=torch.int64, device="cuda")
    ops.rows_argmax(dl[:, :1500], k0, offset=0)
    ops.rows_argmax(dl[:, 1500:], k1, offset=1500)
    np.testing.assert_array_equal(ops.key_index(torch.maximum(k0, k1)).cpu().numpy(), ref - 100)
    tokens = torch.zeros((B, T), dtype=torch.int32, device="cuda")
    pos = torch.tensor([P - 2], dtype=torch.int32, device="cuda")
    ops.rows_advance(keys, tokens, pos, P)  # inside the prompt: nothing written
    assert int(pos.item()) == P - 1 and not tokens.any()
    ops.rows_advance(keys, tokens, pos, P)
    torch.cuda.synchronize()
    assert int(pos.item()) == P
    np.testing.assert_array_equal(tokens[:, P].cpu().numpy(), ref)
    assert ops.device_error() == 0


def test_batch_decode_matches_oracle_teacher_forced(cuda, DO):
    torch = cuda
    shape, B = SMALL_GQA, 3
    prompts = np.array([[3, 141, 59, 26], [7, 7, 900, 1], [500, 2, 33, 999]])
    n_new = 6
    dec = BD.BatchDecoder(shape, B, ctx=32, seed=11)
    try:
        toks = dec.generate(prompts, n_new)
        dec.reset(prompts)
        gl = []
        for _ in range(prompts.shape[1] - 1 + n_new):
            dec.step()
            torch.cuda.synchronize()
            gl.append(dec.logits.cpu().numpy().copy())
        np.testing.assert_array_equal(dec.tokens[:, 4:4 + n_new].cpu().numpy(), toks)  # eager = graphs
        assert ops.device_error() == 0
    finally:
        dec.close()
    one = D.LlamaDecoder(shape, ctx=32, seed=11)  # the same unit-seeded model
    hw = one.host_weights()
    one.close()
    for b in range(B):
        orc = DO.DecodeOracle(shape, hw, ctx=32)
        otoks, ol = orc.generate(list(prompts[b]), n_new, forced=list(toks[b]))
        errs = [rel_err(g[b], o) for g, o in zip(gl, ol)]
        assert max(errs) <= DECODE_TOL and min(errs) <= STEP_TOL, (b, errs)
        for i, t in enumerate(toks[b]):
            lg = ol[prompts.shape[1] - 1 + i]
            top2 = np.sort(lg)[-2:]
            if top2[1] - top2[0] > 2 * DECODE_TOL * np.abs(lg).max():
                assert t == otoks[i]


def test_batch_decode_rows_are_independent(cuda):
    # a sequence's tokens do not depend on the other rows of the batch
    torch = cuda
    shape = SMALL_GQA
    p = np.array([[11, 12, 13], [400, 401, 402]])
    a = BD.BatchDecoder(shape, 2, ctx=32, seed=4)
    b = BD.BatchDecoder(shape, 1, ctx=32, seed=4)
    try:
        ta = a.generate(p, 8)
        tb = b.generate(p[1:], 8)
        la, lb = a.logits[1].cpu().numpy(), b.logits[0].cpu().numpy()
        assert rel_err(la, lb) <= 1e-5 or (ta[1] == tb[0]).all()
        assert ops.device_error() == 0
    finally:
        a.close()
        b.close()
