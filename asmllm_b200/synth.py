"""Seeded synthetic inputs with the distributions of the benchmark configurations.

No model file or dataset is involved: weights and activations are drawn as
the benchmark configurations describe them --
  Q4_0: nibbles uniform 0..15, block scale d = fp16(|N(0, 0.02)|);
  Q8_0: int8 uniform -127..127, d = fp16(|N(0, 0.002)|);
  x:    fp32 N(0, 1).
Scales are returned as fp32 arrays holding fp16 values (the reference ABI
takes fp32 scales, src/runtime/generate.py:94-98 widens GGUF's fp16), so the
fp16 repack of the resident layout is lossless.
Seeds: 0 for weights, 1 for activations unless given.
"""
from __future__ import annotations

import numpy as np

SHAPES_7B = {
    "attn_4096x4096": (4096, 4096),
    "ffn_up_11008x4096": (11008, 4096),
    "ffn_down_4096x11008": (4096, 11008),
    "lm_head_32000x4096": (32000, 4096),
}


def q4_0_weights(M: int, K: int, seed: int = 0):
    """(qs uint8 [M, K/32, 16], scales fp32 [M, K/32])."""
    rng = np.random.default_rng(seed)
    nb = K // 32
    qs = rng.integers(0, 256, size=(M, nb, 16), dtype=np.uint8)
    d = np.abs(rng.standard_normal((M, nb), dtype=np.float32) * np.float32(0.02))
    return qs, d.astype(np.float16).astype(np.float32)


def q8_0_weights(M: int, K: int, seed: int = 0):
    """(qs int8 [M, K/32, 32], scales fp32 [M, K/32])."""
    rng = np.random.default_rng(seed)
    nb = K // 32
    qs = rng.integers(-127, 128, size=(M, nb, 32), dtype=np.int8)
    d = np.abs(rng.standard_normal((M, nb), dtype=np.float32) * np.float32(0.002))
    return qs, d.astype(np.float16).astype(np.float32)


def activation(K: int, seed: int = 1, n: int | None = None):
    rng = np.random.default_rng(seed)
    shape = (K,) if n is None else (n, K)
    return rng.standard_normal(shape, dtype=np.float32)


def gguf_blocks(qs: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Interleave a qs plane and scales into raw GGUF blocks (fp16 d first)."""
    nblk = scales.size
    qb = qs.reshape(nblk, -1).view(np.uint8)
    d = scales.reshape(nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    return np.ascontiguousarray(np.concatenate([d, qb], axis=1)).reshape(-1)
