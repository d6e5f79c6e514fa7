"""CPU restatement of the reference's batch-1 decode step (numpy + the C oracle).

TEST INFRASTRUCTURE ONLY.  Imported by tests/ and bench.py's reference arm as
the checker -- never by the shipped package ``asmllm_b200``.

Restates ``AsmEngineForward.forward_token`` (THRISHAL12345/asmllm
src/runtime/generate.py:255-326) with the model shape as a parameter:

  * every matvec is ``asm_matmul_q4`` (generate.py:227-231) with the NEON
    Q4_0 x Q8_0 semantics the north star names -- here the C restatement
    ``ref_matmul_q4q8`` / ``ref_matmul_q8q8`` of oracle/asmllm_oracle.c;
  * RMSNorm as ``ref_rmsnorm`` (tests/reference/ops.py:103-116):
    (x / sqrt(mean(x^2) + eps)) * w in float32;
  * RoPE as ``ref_rope`` (ops.py:119-141) on interleaved pairs, with the
    (cos, sin) table the decoder uses (same numpy expressions);
  * the KV cache is fp16 by default (the config the path is measured on); the
    reference keeps fp32 (generate.py:252-253), kv_dtype=np.float32 -- k and v
    are rounded to the cache dtype when stored and read back as float32;
  * attention per head: scores = q.K^T / float32(sqrt(hd)) (generate.py:292),
    softmax = exp(s - max) / sum (ops.py:144-153), out = p.V;
  * silu(gate) * up = (gate / (1 + exp(-gate))) * up (generate.py:370);
  * the lm_head is a Q4_0 matvec after the final RMSNorm; the next token is
    the first argmax (generate.py:410).

Grouped KV heads (n_kv_heads < n_heads) map query head h to KV head
h // (n_heads / n_kv_heads), as Llama-2-70B does.
"""
from __future__ import annotations

import numpy as np

from . import oracle as _o


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float32)
    rms = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + np.float32(eps))
    return ((x / rms) * w).astype(np.float32)


def rope(v: np.ndarray, cs: np.ndarray) -> np.ndarray:
    """v: [..., hd]; cs: [hd/2, 2] (cos, sin) of this position."""
    x0, x1 = v[..., 0::2], v[..., 1::2]
    c, s = cs[:, 0], cs[:, 1]
    out = np.empty_like(v)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def softmax(s: np.ndarray) -> np.ndarray:
    e = np.exp(s - np.max(s))
    return e / np.sum(e)


class DecodeOracle:
    """One model's decode state on the CPU; weights from LlamaDecoder.host_weights()."""

    def __init__(self, shape, weights: dict, ctx: int, fmt: int = 2, nthreads: int | None = None,
                 kv_dtype=np.float16):
        self.s = shape
        self.w = weights
        self.fmt = fmt
        self.ctx = ctx
        self.nthreads = nthreads or _o.host_threads()
        L, nkv, hd = shape.n_layers, shape.n_kv_heads, shape.head_dim
        self.kc = np.zeros((L, ctx, nkv, hd), dtype=kv_dtype)  # fp16: the measured config; fp32: the reference's
        self.vc = np.zeros((L, ctx, nkv, hd), dtype=kv_dtype)
        self.sqrt_hd = np.sqrt(np.float32(hd), dtype=np.float32)

    def matvec(self, w, x: np.ndarray) -> np.ndarray:
        qs, sc = w
        M, K = sc.shape[0], sc.shape[1] * 32
        kind = _o.K_Q4Q8 if self.fmt == 2 else _o.K_Q8Q8
        if self.nthreads > 1 and M >= 1024:
            return _o.matmul_mt(kind, qs, sc, x.astype(np.float32), M, K, self.nthreads)
        f = _o.matmul_q4q8 if self.fmt == 2 else _o.matmul_q8q8
        return f(qs, sc, x.astype(np.float32), M, K)

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        s, W = self.s, self.w
        nh, nkv, hd = s.n_heads, s.n_kv_heads, s.head_dim
        group = nh // nkv
        cs = W["rope"][pos]
        x = W["embed"][token].astype(np.float32).copy()
        for li, L in enumerate(W["layers"]):
            xn = rmsnorm(x, L["attn_norm"], s.eps)
            q = self.matvec(L["wq"], xn).reshape(nh, hd)
            k = self.matvec(L["wk"], xn).reshape(nkv, hd)
            v = self.matvec(L["wv"], xn).reshape(nkv, hd)
            q = rope(q, cs)
            k = rope(k, cs)
            self.kc[li, pos] = k.astype(self.kc.dtype)
            self.vc[li, pos] = v.astype(self.vc.dtype)
            att = np.zeros((nh, hd), dtype=np.float32)
            for h in range(nh):
                j = h // group
                K = self.kc[li, : pos + 1, j].astype(np.float32)
                V = self.vc[li, : pos + 1, j].astype(np.float32)
                scores = (q[h] @ K.T) / self.sqrt_hd
                att[h] = softmax(scores) @ V
            x = x + self.matvec(L["wo"], att.reshape(-1))
            xn = rmsnorm(x, L["ffn_norm"], s.eps)
            gate = self.matvec(L["w_gate"], xn)
            up = self.matvec(L["w_up"], xn)
            hsw = (gate / (np.float32(1.0) + np.exp(-gate))) * up
            x = x + self.matvec(L["w_down"], hsw.astype(np.float32))
        xn = rmsnorm(x, W["final_norm"], s.eps)
        return self.matvec(W["lm_head"], xn)

    def generate(self, prompt, n_new: int, forced=None):
        """Greedy decode as generate.py:399-411; returns (tokens, per-step logits).
        With `forced`, the inputs after the prompt are those ids (teacher forcing)
        instead of the argmax."""
        logits_all = []
        out = []
        cur = int(prompt[0])
        n = len(prompt) - 1 + n_new
        for p in range(n):
            lg = self.forward_token(cur, p)
            logits_all.append(lg)
            nxt = int(np.argmax(lg))
            if p + 1 < len(prompt):
                cur = int(prompt[p + 1])
            else:
                out.append(nxt)
                cur = int(forced[len(out) - 1]) if forced is not None else nxt
        return out, logits_all
