"""Shared fixtures.  `-m gpu` tests need a CUDA device; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(autouse=True)
def no_pending_library_error():
    """A test that provokes a library error must read it (native.last_error());
    one left pending would be raised by the next test's first check()."""
    yield
    native = sys.modules.get("asmllm_b200.native")
    if native is not None and getattr(native, "_lib", None) is not None:
        code, msg = native.last_error()
        assert code == 0, f"test left a pending library error: {code} {msg}"


@pytest.fixture(scope="session")
def golden():
    """The reference's seed-42 fixture (tools/reference_gen.py), saved by tests/golden/make_golden.py."""
    with np.load(GOLDEN / "reference_seed42.npz") as d:
        return {k: d[k] for k in d.files}


@pytest.fixture(scope="session")
def bench_recipes():
    with np.load(GOLDEN / "bench_recipes.npz") as d:
        return {k: d[k] for k in d.files}


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.lib()
    return O


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def rel_err(y, ref):
    """max |y - ref| / max |ref| (the parity metric; 0/0 counts as exact)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    num = float(np.max(np.abs(y - ref))) if y.size else 0.0
    den = float(np.max(np.abs(ref))) if ref.size else 0.0
    if den == 0.0:
        return 0.0 if num == 0.0 else float("inf")
    return num / den


# Parity tolerance for fp32 outputs (max |err| <= 1e-4 * ||y||_inf).
YTOL = 1e-4
