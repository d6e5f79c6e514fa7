"""__graft_entry__.smoke() in a fresh process, as a deployment check runs it.

smoke() checks one small call of every kernel family against the oracle
(quantize and block sums bit for bit, the matvec and the sync ABI within the
y tolerance, three decode steps, the tensor-core product bit for bit unsplit
and within tolerance with its automatic K split).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_smoke_in_a_fresh_process():
    env = dict(os.environ, PYTHONPATH=str(ROOT) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.smoke()"], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "smoke ok" in r.stdout
