"""CPU checks of the decode-glue restatement (oracle/glue_oracle.py) against
numpy itself and the reference's own outputs (tests/golden/)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN

from oracle import glue_oracle as G


def ulps(a, b):
    """Largest distance in units in the last place between two fp32 arrays."""
    a = np.asarray(a, dtype=np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, dtype=np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return int(np.max(np.abs(a - b))) if a.size else 0


@pytest.mark.parametrize("n", [1, 5, 7, 8, 9, 15, 16, 63, 64, 100, 127, 128, 129, 143, 255, 256, 288, 1000,
                               4096, 4097, 8192, 11008, 28672])
def test_pairwise_sum_is_numpys_order(n):
    rng = np.random.default_rng(n)
    for _ in range(4):
        a = (rng.standard_normal(n) * rng.uniform(0.1, 100)).astype(np.float32)
        assert G.pairwise_sum(a).view(np.uint32) == np.sum(a).view(np.uint32)
        sq = (a * a).astype(np.float32)
        assert np.float32(G.pairwise_sum(sq) / np.float32(n)).view(np.uint32) == np.mean(sq).view(np.uint32)


def test_rmsnorm_restatement_is_bit_exact_vs_reference_outputs(golden):
    with np.load(GOLDEN / "decode_glue.npz") as d:
        y = G.rmsnorm(d["norm_x"], d["norm_w"], 1e-5)
        assert np.array_equal(y.view(np.uint32), d["norm_y"].view(np.uint32))
    y = G.rmsnorm(golden["rmsnorm_x"], golden["rmsnorm_weight"], float(golden["rmsnorm_eps"]))
    assert np.array_equal(y.view(np.uint32), golden["rmsnorm_expected"].view(np.uint32))


def test_transcendental_steps_are_within_an_ulp_or_two_of_numpy(golden):
    # numpy's fp32 exp / sin / cos are not correctly rounded; the restatement
    # (float64 rounded once, as the x87 path of the reference's x86 kernels)
    # stays within a few ulps of the reference's numpy outputs.
    with np.load(GOLDEN / "decode_glue.npz") as d:
        assert ulps(G.softmax(d["softmax_x"]), d["softmax_y"]) <= 4
        for i, p in enumerate(d["rope_pos"]):
            # numpy's fp32 pow is off by an ulp for some of the 64 frequencies;
            # the angle pos * freq carries that error times pos
            for v, ref in ((d["rope_q"], d["rope_q_out"][i]), (d["rope_k"], d["rope_k_out"][i])):
                out = G.rope(v, 128, int(p))
                assert np.max(np.abs(out - ref)) <= (int(p) + 1) * 3e-7 * float(np.abs(v).max())
    assert ulps(G.softmax(golden["softmax_x"]), golden["softmax_expected"]) <= 4
    q = G.rope(golden["rope_q"], 32, int(golden["rope_pos"]))
    assert np.max(np.abs(q - golden["rope_q_expected"])) <= 1e-6
    att = G.attention(golden["attention_q"], golden["attention_k"], golden["attention_v"],
                      1.0 / np.sqrt(golden["attention_q"].shape[1]))
    assert np.max(np.abs(att - golden["attention_expected"])) <= 1e-5
