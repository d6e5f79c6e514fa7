"""CPU checks of the decode-step restatement (oracle/decode_oracle.py) and of
the host side of asmllm_b200.decode: the glue ops against the reference's own
outputs (tests/golden/decode_glue.npz, made by make_golden.py from
tests/reference/ops.py), the RoPE table, the descriptor layout, and a tiny
model decoded twice on the CPU."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from asmllm_b200 import decode as D
from asmllm_b200 import native
from conftest import GOLDEN


@pytest.fixture(scope="module")
def glue():
    return dict(np.load(GOLDEN / "decode_glue.npz"))


@pytest.fixture(scope="module")
def DO(oracle):
    from oracle import decode_oracle
    return decode_oracle


def test_rmsnorm_matches_reference_bit_exact(glue, DO):
    y = DO.rmsnorm(glue["norm_x"], glue["norm_w"], 1e-5)
    np.testing.assert_array_equal(y, glue["norm_y"])


def test_rope_table_matches_reference_bit_exact(glue, DO):
    tab = D.rope_table(512, 128, 10000.0)
    assert tab.shape == (512, 64, 2) and tab.dtype == np.float32
    for i, p in enumerate(glue["rope_pos"]):
        np.testing.assert_array_equal(DO.rope(glue["rope_q"], tab[p]), glue["rope_q_out"][i])
        np.testing.assert_array_equal(DO.rope(glue["rope_k"], tab[p]), glue["rope_k_out"][i])


def test_softmax_matches_reference(glue, DO):
    np.testing.assert_array_equal(DO.softmax(glue["softmax_x"]), glue["softmax_y"])


def test_descriptor_layout_matches_header():
    # asm_fused_matvec_t on LP64: 2 int32, 15 pointers, float + 3 int32, 2 int64,
    # 4 int32, 8 + 2 pointers
    assert ctypes.sizeof(native.FusedMatvec) == 256
    assert native.FusedMatvec.eps.offset == 128 and native.FusedMatvec.M.offset == 144
    assert native.FusedMatvec.xchg.offset == 176
    text = (GOLDEN.parent.parent / "include" / "asmllm.h").read_text()
    body = text[text.index("typedef struct asm_fused_matvec"):text.index("} asm_fused_matvec_t;")]
    body = re.sub(r"/\*.*?\*/", " ", body, flags=re.S)  # declarations only
    names = [f for f, _ in native.FusedMatvec._fields_]
    pos = [body.index(f" {n};") if f" {n};" in body else body.index(f" {n},") if f" {n}," in body
           else body.index(f"*{n};") if f"*{n};" in body else body.index(f" {n}[") for n in names]
    assert pos == sorted(pos), "field order differs from include/asmllm.h"


def test_rows_descriptor_layout_matches_header():
    # asm_rows_t on LP64: 2 int32, 5 pointers, 2 int32, pointer, float + int32, pointer
    assert ctypes.sizeof(native.Rows) == 80
    assert native.Rows.norm_w.offset == 56 and native.Rows.tiles.offset == 72
    text = (GOLDEN.parent.parent / "include" / "asmllm.h").read_text()
    body = text[text.index("typedef struct asm_rows {"):text.index("} asm_rows_t;")]
    body = re.sub(r"/\*.*?\*/", " ", body, flags=re.S)
    names = [f for f, _ in native.Rows._fields_]
    pos = [body.index(f" {n};") if f" {n};" in body else body.index(f"*{n};") for n in names]
    assert pos == sorted(pos), "field order differs from include/asmllm.h"


def test_shape_bytes():
    assert D.LLAMA_7B.weight_bytes() == 3_716_481_024
    assert D.LLAMA2_70B.weight_bytes() == 38_651_166_720
    assert D.LLAMA_7B.qkv_rows == 12288 and D.LLAMA2_70B.qkv_rows == 10240
    assert D.LLAMA_7B.kv_bytes(0) == 32 * 2 * 4096 * 2


def tiny_weights(shape, seed=3):
    """Host weights in the layout LlamaDecoder.host_weights() returns."""
    rng = np.random.default_rng(seed)

    def q4(M, K):
        return (rng.integers(0, 256, (M, K // 32, 16), dtype=np.uint8),
                np.abs(rng.normal(0, 0.02, (M, K // 32))).astype(np.float16).astype(np.float32))

    s = shape
    qd, kvd = s.n_heads * s.head_dim, s.n_kv_heads * s.head_dim
    layers = []
    for _ in range(s.n_layers):
        layers.append({"wq": q4(qd, s.dim), "wk": q4(kvd, s.dim), "wv": q4(kvd, s.dim), "wo": q4(s.dim, qd),
                       "w_gate": q4(s.ffn, s.dim), "w_up": q4(s.ffn, s.dim), "w_down": q4(s.dim, s.ffn),
                       "attn_norm": (1 + 0.01 * rng.standard_normal(s.dim)).astype(np.float32),
                       "ffn_norm": (1 + 0.01 * rng.standard_normal(s.dim)).astype(np.float32)})
    return {"layers": layers, "embed": rng.standard_normal((s.vocab, s.dim)).astype(np.float32),
            "final_norm": (1 + 0.01 * rng.standard_normal(s.dim)).astype(np.float32),
            "lm_head": q4(s.vocab, s.dim), "rope": D.rope_table(32, s.head_dim, s.theta)}


TINY = D.LlamaShape(n_layers=2, dim=256, n_heads=2, n_kv_heads=1, head_dim=128, ffn=512, vocab=300)


def test_decode_oracle_is_deterministic_and_greedy(DO):
    W = tiny_weights(TINY)
    a = DO.DecodeOracle(TINY, W, ctx=32, nthreads=1)
    toks, logits = a.generate([5, 17, 250], 6)
    assert len(toks) == 6 and len(logits) == 2 + 6
    assert all(0 <= t < TINY.vocab for t in toks)
    for i, t in enumerate(toks):  # each generated id is the argmax of the step that made it
        assert t == int(np.argmax(logits[2 + i]))
    b = DO.DecodeOracle(TINY, W, ctx=32, nthreads=2)
    toks2, logits2 = b.generate([5, 17, 250], 6)
    assert toks2 == toks
    for x, y in zip(logits, logits2):
        np.testing.assert_array_equal(x, y)


def test_decode_oracle_grouped_kv_reads_shared_head(DO):
    # With one KV head for two query heads, both heads attend over the same cache rows.
    W = tiny_weights(TINY, seed=4)
    o = DO.DecodeOracle(TINY, W, ctx=32, nthreads=1)
    o.forward_token(7, 0)
    o.forward_token(8, 1)
    assert o.kc.shape[2] == 1 and np.any(o.kc[0, 1] != 0) and not np.any(o.kc[0, 2])
