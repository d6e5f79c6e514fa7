#!/usr/bin/env python3
"""Regenerates the golden fixtures in this folder from the reference itself.

Run in a container where the reference project (THRISHAL12345/asmllm) is
checked out; pass its root as the first argument or via ASMLLM_REFERENCE_ROOT.
It imports the reference's own Python (no copy of it lives in this repo):

  * tools/reference_gen.py:31-112  generate_reference_data(seed=42) -- the
    fixture tests/correctness/test_runner.py feeds every kernel (the matvecs
    and the glue kernels rmsnorm / rope / softmax / attention);
  * tests/reference/ops.py:33-64   ref_q4_matmul / ref_q8_matmul -- the numpy
    fp32 expectations the reference harness compares against;
  * the input recipes of bench/harness/bench_matmul_q4.py:76-80,
    bench_mt_throughput.py:54-58 and bench_quant_formats.py:68-80 (numpy
    RandomState(42)), whose numpy outputs are stored as expectations.  Inputs
    of the large recipes are not stored: tests regenerate them from the same
    legacy RandomState stream and check the stored SHA-256 of the bytes.

  * tests/reference/ops.py:103-153 ref_rmsnorm / ref_rope / ref_softmax --
    the decode-step glue of generate.py:255-326, on seeded inputs
    (np.random.default_rng(7)) at the 7B shapes (dim 4096, head_dim 128).

  * src/runtime/generate.py:38-88 load_gguf_tensors_and_vocab -- the
    reference's GGUF parser, run on tiny.gguf (a small GGUF v3 file written
    here by asmllm_b200.gguf.write_gguf: metadata of several types, a token
    list, Q4_0 / Q8_0 / F32 tensors); its tensor table, data offset and
    vocabulary are stored in tiny_gguf_ref.json.

Outputs: reference_seed42.npz (small fixture, all arrays),
bench_recipes.npz (expected y vectors + input digests), decode_glue.npz,
tiny.gguf and tiny_gguf_ref.json.
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bench_matmul_q4_inputs(M=4096, K=4096):
    """Input recipe of bench/harness/bench_matmul_q4.py:76-80."""
    rng = np.random.RandomState(42)
    nb = K // 32
    q = rng.randint(0, 256, size=(M, nb, 16), dtype=np.uint8)
    s = rng.uniform(0.5, 1.5, size=(M, nb)).astype(np.float32)
    x = rng.randn(K).astype(np.float32)
    return q, s, x


def bench_mt_inputs(M=4096, K=4096):
    """Input recipe of bench/harness/bench_mt_throughput.py:54-58."""
    rng = np.random.RandomState(42)
    nb = K // 32
    q = rng.randint(0, 256, size=(M, nb, 16), dtype=np.uint8)
    s = rng.uniform(0.05, 0.25, size=(M, nb)).astype(np.float32)
    x = rng.randn(K).astype(np.float32)
    return q, s, x


def bench_quant_formats_inputs(M=1024, K=4096):
    """Input recipe of bench/harness/bench_quant_formats.py:68-80 (Q4 and Q8 parts)."""
    rng = np.random.RandomState(42)
    nb = K // 32
    x = rng.randn(K).astype(np.float32)
    q4 = rng.randint(0, 256, size=(M, nb, 16), dtype=np.uint8)
    s4 = rng.uniform(0.5, 1.5, size=(M, nb)).astype(np.float32)
    q8 = rng.randint(-127, 128, size=(M, nb, 32), dtype=np.int8)
    s8 = rng.uniform(0.1, 0.9, size=(M, nb)).astype(np.float32)
    return x, q4, s4, q8, s8


def main() -> None:
    root = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ASMLLM_REFERENCE_ROOT", ""))
    if not (root / "tools" / "reference_gen.py").exists():
        raise SystemExit("usage: make_golden.py <reference project root>")
    sys.path.insert(0, str(root))
    from tools.reference_gen import generate_reference_data  # noqa: E402
    from tests.reference.ops import ref_q4_matmul, ref_q8_matmul  # noqa: E402

    data = generate_reference_data(seed=42)
    keep = {k: v for k, v in data.items()
            if k.startswith(("q4_matmul", "q8_matmul", "q5_matmul", "rmsnorm", "rope", "softmax", "attention"))}
    np.savez_compressed(HERE / "reference_seed42.npz", **keep)

    out = {}
    q, s, x = bench_matmul_q4_inputs()
    out["bench_q4_y"] = ref_q4_matmul(q, s, x).astype(np.float32)
    out["bench_q4_sha"] = np.array([_sha(q), _sha(s), _sha(x)])
    q, s, x = bench_mt_inputs()
    out["bench_mt_y"] = ref_q4_matmul(q, s, x).astype(np.float32)
    out["bench_mt_sha"] = np.array([_sha(q), _sha(s), _sha(x)])
    x, q4, s4, q8, s8 = bench_quant_formats_inputs()
    out["bench_qf_q4_y"] = ref_q4_matmul(q4, s4, x).astype(np.float32)
    out["bench_qf_q8_y"] = ref_q8_matmul(q8, s8, x).astype(np.float32)
    out["bench_qf_sha"] = np.array([_sha(x), _sha(q4), _sha(s4), _sha(q8), _sha(s8)])
    np.savez_compressed(HERE / "bench_recipes.npz", **out)

    from tests.reference.ops import ref_rmsnorm, ref_rope, ref_softmax  # noqa: E402
    rng = np.random.default_rng(7)
    g = {}
    g["norm_x"] = (3.0 * rng.standard_normal(4096)).astype(np.float32)
    g["norm_w"] = (1.0 + 0.01 * rng.standard_normal(4096)).astype(np.float32)
    g["norm_y"] = ref_rmsnorm(g["norm_x"], g["norm_w"], eps=1e-5)
    g["rope_pos"] = np.array([0, 1, 17, 142, 511], dtype=np.int64)
    g["rope_q"] = rng.standard_normal((4, 128)).astype(np.float32)
    g["rope_k"] = rng.standard_normal((4, 128)).astype(np.float32)
    qs, ks = [], []
    for p in g["rope_pos"]:
        qr, kr = ref_rope(g["rope_q"], g["rope_k"], head_dim=128, pos=int(p), theta=10000.0)
        qs.append(qr)
        ks.append(kr)
    g["rope_q_out"], g["rope_k_out"] = np.stack(qs), np.stack(ks)
    g["softmax_x"] = (8.0 * rng.standard_normal(143)).astype(np.float32)
    g["softmax_y"] = ref_softmax(g["softmax_x"])
    np.savez_compressed(HERE / "decode_glue.npz", **g)

    import json

    sys.path.insert(0, str(HERE.parent.parent))
    from asmllm_b200 import gguf as G  # noqa: E402
    from src.runtime.generate import load_gguf_tensors_and_vocab  # noqa: E402
    rng = np.random.default_rng(5)
    q4 = rng.integers(0, 256, (4, 2, 16), dtype=np.uint8)
    s4 = np.abs(rng.standard_normal((4, 2))).astype(np.float16).astype(np.float32)
    q8 = rng.integers(-127, 128, (3, 1, 32), dtype=np.int8)
    s8 = np.abs(rng.standard_normal((3, 1))).astype(np.float16).astype(np.float32)
    f = rng.standard_normal(32).astype(np.float32)
    G.write_gguf(HERE / "tiny.gguf",
                 {"general.architecture": "llama", "llama.block_count": 1, "llama.rope.freq_base": 10000.0,
                  "general.name": "tiny", "tokenizer.ggml.tokens": ["<s>", "</s>", "a", "b"],
                  "tokenizer.ggml.scores": [0.0, 0.5, 1.0, 1.5], "general.file_type": 2},
                 [("blk.0.attn_q.weight", (64, 4), G.GGML_Q4_0, G.blocks_from_planes(q4, s4)),
                  ("blk.0.attn_k.weight", (32, 3), G.GGML_Q8_0, G.blocks_from_planes(q8, s8)),
                  ("output_norm.weight", (32,), G.GGML_F32, f.tobytes())])
    tensors, data_offset, data, vocab = load_gguf_tensors_and_vocab(str(HERE / "tiny.gguf"))
    with open(HERE / "tiny_gguf_ref.json", "w") as fh:
        json.dump({"tensors": {k: [list(v[0]), v[1], v[2]] for k, v in tensors.items()},
                   "data_offset": data_offset, "data_len": len(data), "vocab": vocab}, fh, indent=1)
    print("wrote the fixtures in", HERE)


if __name__ == "__main__":
    main()
