"""GGUF reading and writing (asmllm_b200.gguf), pinned to the reference's own
parser: tests/golden/tiny.gguf was written by write_gguf and parsed by the
reference's load_gguf_tensors_and_vocab (src/runtime/generate.py:38-88);
tiny_gguf_ref.json holds what that parser found."""
from __future__ import annotations

import json

import numpy as np

from asmllm_b200 import gguf as G
from conftest import GOLDEN


def test_reader_matches_the_reference_parser():
    ref = json.loads((GOLDEN / "tiny_gguf_ref.json").read_text())
    gg = G.GGUFFile(GOLDEN / "tiny.gguf")
    assert gg.version == 3
    assert {k: [list(t.dims), t.type, t.offset] for k, t in gg.tensors.items()} == ref["tensors"]
    assert gg.data_offset == ref["data_offset"]
    assert gg.metadata["tokenizer.ggml.tokens"] == ref["vocab"]
    size = (GOLDEN / "tiny.gguf").stat().st_size
    assert size - gg.data_offset == ref["data_len"]


def test_tensor_bytes_round_trip(tmp_path):
    rng = np.random.default_rng(9)
    q4 = rng.integers(0, 256, (8, 3, 16), dtype=np.uint8)
    s4 = np.abs(rng.standard_normal((8, 3))).astype(np.float16).astype(np.float32)
    q8 = rng.integers(-127, 128, (5, 2, 32), dtype=np.int8)
    s8 = np.abs(rng.standard_normal((5, 2))).astype(np.float16).astype(np.float32)
    f = rng.standard_normal((2, 32)).astype(np.float32)
    md = {"general.architecture": "llama", "i": -7, "big": 2**40, "x": 0.25, "flag": True, "name": "m",
          "ints": [1, 2, 3], "floats": [0.5, 1.5], "strs": ["a", "bc"]}
    p = tmp_path / "t.gguf"
    G.write_gguf(p, md, [("q4", (96, 8), G.GGML_Q4_0, G.blocks_from_planes(q4, s4)),
                         ("q8", (64, 5), G.GGML_Q8_0, G.blocks_from_planes(q8, s8)),
                         ("f", (32, 2), G.GGML_F32, f.tobytes())], alignment=64)
    gg = G.GGUFFile(p)
    assert gg.alignment == 64 and gg.data_offset % 64 == 0
    for k, v in md.items():
        got = gg.metadata[k]
        assert got == v if not isinstance(v, float) else abs(got - v) < 1e-7
    assert gg.metadata["floats"] == [0.5, 1.5]
    # the reference's host split (generate.py:91-106): fp16 d first, then the quants
    raw = np.asarray(gg.raw("q4")).reshape(8, 3, 18)
    np.testing.assert_array_equal(raw[:, :, 2:], q4)
    np.testing.assert_array_equal(raw[:, :, :2].copy().view(np.float16).reshape(8, 3).astype(np.float32), s4)
    raw8 = np.asarray(gg.raw("q8")).reshape(5, 2, 34)
    np.testing.assert_array_equal(raw8[:, :, 2:].view(np.int8), q8)
    np.testing.assert_array_equal(gg.array("f"), f)
    t = gg.tensors["q4"]
    assert (t.rows, t.cols, t.nbytes) == (8, 96, 8 * 3 * 18)
