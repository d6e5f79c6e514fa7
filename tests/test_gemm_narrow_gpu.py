"""The batched product for a few tokens (asm_gemm_narrow_async, N <= 8): every
activation row's result equals the warp-ring matvec of that row bit for bit
(same lanes, same block order, same reduction), and stays within the parity
tolerance of the oracle."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import YTOL, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", [2, 8], ids=["q4_0", "q8_0"])
@pytest.mark.parametrize("N", [1, 2, 3, 8])
@pytest.mark.parametrize("M,K", [(512, 4096), (301, 11008), (64, 256), (1000, 1024)])
def test_narrow_rows_equal_matvec(cuda, oracle, fmt, N, M, K):
    torch = cuda
    from asmllm_b200 import ops, synth

    w, s = (synth.q4_0_weights if fmt == 2 else synth.q8_0_weights)(M, K, seed=M + K + N)
    dw, ds = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half()
    X = torch.stack([torch.from_numpy(synth.activation(K, seed=100 + n)) for n in range(N)]).cuda()
    img = ops.act_image_dev(X)
    Y = ops.gemm_narrow(fmt, dw, ds, img, K)
    torch.cuda.synchronize()
    sf = s.astype(np.float16).astype(np.float32)
    for n in range(N):
        ref = ops.matvec(fmt, dw, ds, X[n], independent=True)
        assert torch.equal(Y[n], ref), n
        o = oracle.matmul_q4q8(w, sf, X[n].cpu().numpy()) if fmt == 2 else oracle.matmul_q8q8(w, sf, X[n].cpu().numpy())
        assert rel_err(Y[n].cpu().numpy(), o) <= YTOL
    assert ops.device_error() == 0


def test_narrow_rejects_more_than_eight_tokens(cuda):
    torch = cuda
    from asmllm_b200 import native, ops

    K, M = 256, 16
    dw = torch.zeros((M, K // 32, 16), dtype=torch.uint8, device="cuda")
    ds = torch.zeros((M, K // 32), dtype=torch.float16, device="cuda")
    img = ops.act_image_dev(torch.zeros((9, K), device="cuda"))
    with pytest.raises(native.AsmError):
        ops.gemm_narrow(2, dw, ds, img, K)
