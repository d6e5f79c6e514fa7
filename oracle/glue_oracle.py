"""CPU restatement of the decode-glue kernels (numpy; float64 transcendentals).

TEST INFRASTRUCTURE ONLY.  Imported by tests/ as the checker -- never by the
shipped package ``asmllm_b200``.

Restates, operation by operation in fp32, the reference's numpy definitions
(THRISHAL12345/asmllm tests/reference/ops.py:103-170, generate.py:370) the
way the library's GPU kernels evaluate them:

  * ``pairwise_sum`` -- numpy's own summation order for a contiguous fp32
    reduction (numpy/_core/src/umath/loops_utils.h.src, pairwise_sum: running
    sums for n < 8; eight interleaved running sums combined
    ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) plus the n % 8 tail for n <= 128;
    otherwise halves at n2 = n/2 rounded down to a multiple of 8).  It is
    pinned against numpy.sum / numpy.mean (tests/test_glue_oracle.py), and
    ``rmsnorm`` against the reference's ref_rmsnorm outputs bit for bit;
  * exp / sin / cos / pow in float64, rounded once to fp32 -- as the
    reference's x86 kernels use the x87 unit (rope_avx2.asm:98,
    softmax_avx2.asm:75-87).  numpy's fp32 versions are not correctly
    rounded, so ``softmax``, ``rope`` and ``silu_hadamard`` agree with the
    reference's numpy outputs to about one ulp, not bit for bit.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def pairwise_sum(a) -> np.float32:
    a = np.asarray(a, dtype=np.float32)
    n = a.shape[0]
    if n < 8:
        r = f32(0.0)
        for v in a:
            r = f32(r + v)
        return r
    if n <= 128:
        m = n - n % 8
        r = a[:8].copy()
        for i in range(8, m, 8):
            r = (r + a[i:i + 8]).astype(np.float32)
        res = f32(f32(f32(r[0] + r[1]) + f32(r[2] + r[3])) + f32(f32(r[4] + r[5]) + f32(r[6] + r[7])))
        for i in range(m, n):
            res = f32(res + a[i])
        return res
    n2 = n // 2
    n2 -= n2 % 8
    return f32(pairwise_sum(a[:n2]) + pairwise_sum(a[n2:]))


def rmsnorm(x, w, eps) -> np.ndarray:
    """(x / sqrt(mean(x^2) + eps)) * w (ops.py:103-116)."""
    x = np.asarray(x, dtype=np.float32)
    ms = f32(pairwise_sum((x * x).astype(np.float32)) / f32(x.shape[0]))
    rms = np.sqrt(f32(ms + f32(eps)), dtype=np.float32)
    return ((x / rms).astype(np.float32) * np.asarray(w, dtype=np.float32)).astype(np.float32)


def exp_r(x) -> np.ndarray:
    return np.exp(np.asarray(x, dtype=np.float64)).astype(np.float32)


def softmax(x) -> np.ndarray:
    """exp(x - max) / sum (ops.py:144-153), exp rounded from float64."""
    x = np.asarray(x, dtype=np.float32)
    e = exp_r((x - np.max(x)).astype(np.float32))
    return (e / pairwise_sum(e)).astype(np.float32)


def rope_table(head_dim: int, pos: int, theta: float):
    """(cos, sin) per pair: angle = pos * (1 / theta^(2i / hd)) in fp32 steps (ops.py:119-128)."""
    e = (np.arange(0, head_dim, 2, dtype=np.float32) / f32(head_dim)).astype(np.float32)
    p = np.power(np.float64(f32(theta)), e.astype(np.float64)).astype(np.float32)
    freq = (f32(1.0) / p).astype(np.float32)
    ang = (f32(pos) * freq).astype(np.float32)
    return np.cos(ang.astype(np.float64)).astype(np.float32), np.sin(ang.astype(np.float64)).astype(np.float32)


def rope(v, head_dim: int, pos: int, theta: float = 10000.0) -> np.ndarray:
    """Interleaved-pair rotation (ops.py:130-141)."""
    c, s = rope_table(head_dim, pos, theta)
    v = np.asarray(v, dtype=np.float32)
    x0, x1 = v[..., 0::2], v[..., 1::2]
    out = np.empty_like(v)
    out[..., 0::2] = (x0 * c).astype(np.float32) - (x1 * s).astype(np.float32)
    out[..., 1::2] = (x0 * s).astype(np.float32) + (x1 * c).astype(np.float32)
    return out


def silu_hadamard(gate, up) -> np.ndarray:
    """(gate / (1 + exp(-gate))) * up (generate.py:370)."""
    g = np.asarray(gate, dtype=np.float32)
    t = (f32(1.0) + exp_r(-g)).astype(np.float32)
    return ((g / t).astype(np.float32) * np.asarray(up, dtype=np.float32)).astype(np.float32)


def attention(q, k, v, scale) -> np.ndarray:
    """softmax(q k^T * scale) v per query row (ops.py:156-170), in float64."""
    q, k, v = (np.asarray(a, dtype=np.float64) for a in (q, k, v))
    s = (q @ k.T) * float(scale)
    s = np.exp(s - s.max(axis=1, keepdims=True))
    return ((s / s.sum(axis=1, keepdims=True)) @ v).astype(np.float32)
