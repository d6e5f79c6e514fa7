"""Row-split matvec (rank r holds rows [r*M, (r+1)*M), y all-gathered by peer
stores inside the matvec plus one wait kernel per step) and the bounded
exchange waits, on one GPU.

Two ranks are emulated on one GPU with local buffers standing in for the
peers' gather buffers: rank 0's matvec, then rank 1's, then each rank's wait.
Every word a wait reads was written by a kernel that completed before it
started, so nothing waits on a kernel running beside it.  The timeout tests
give the wait a word nobody writes and a short limit (option "xchg_wait_us"):
the kernel must give up, set the exchange-timeout bit and return."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import YTOL, rel_err

pytestmark = pytest.mark.gpu


def _emulated_step(torch, ops, native, fmt, shards, xs, ys, bufs, seqs, dones, packed):
    """One step of tp = len(shards) ranks on this GPU: every rank's matvecs, then every rank's wait."""
    L = native.lib()
    tp = len(shards)
    for r in range(tp):
        for j, (w, s) in enumerate(shards[r]):
            M = w.shape[0]
            xchg = (ctypes.c_void_p * 8)(*[bufs[j][q].data_ptr() for q in range(tp)], *([0] * (8 - tp)))
            flags = ops.MV_PACKED if packed else 0
            native.check(L.asm_matvec_rowsplit_async(
                fmt, w.data_ptr(), None if packed else s.data_ptr(), xs[j].data_ptr(), ys[r][j].data_ptr(), M,
                xs[j].shape[0], tp, r, xchg, seqs[r].data_ptr(), flags, None))
    for r in range(tp):
        wt = native.RowsplitWait()
        wt.n, wt.tp, wt.rank = len(xs), tp, r
        for j in range(len(xs)):
            wt.own[j] = bufs[j][r].data_ptr()
            wt.y_full[j] = ys[r][j].data_ptr()
            wt.M[j] = shards[r][j][0].shape[0]
        wt.seq, wt.done = seqs[r].data_ptr(), dones[r].data_ptr()
        native.check(L.asm_rowsplit_wait_async(ctypes.byref(wt), None))


@pytest.mark.parametrize("packed", [True, False], ids=["packed", "planes"])
@pytest.mark.parametrize("tp", [1, 2, 3])
def test_rowsplit_matches_unsplit_matvec(cuda, oracle, tp, packed):
    torch = cuda
    from asmllm_b200 import native, ops, synth

    fmt = native.FMT_Q4_0
    shapes = [(768, 4096), (256, 11008)]  # rows per rank, K
    shards, full_w = [[] for _ in range(tp)], []
    for j, (M, K) in enumerate(shapes):
        w, s = synth.q4_0_weights(tp * M, K, seed=40 + j)
        full_w.append((w, s))
        for r in range(tp):
            dw = torch.from_numpy(w[r * M:(r + 1) * M]).cuda()
            ds = torch.from_numpy(s[r * M:(r + 1) * M]).cuda().half()
            shards[r].append((ops.pack_rows(fmt, dw, ds), None) if packed else (dw, ds))
    xs = [torch.from_numpy(synth.activation(K, seed=50 + j)).cuda() for j, (_, K) in enumerate(shapes)]
    ys = [[torch.full((tp * M,), float("nan"), device="cuda") for M, _ in shapes] for _ in range(tp)]
    bufs = [[torch.zeros(2 * tp * M, dtype=torch.int64, device="cuda") for _ in range(tp)] for M, _ in shapes]
    seqs = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(tp)]
    dones = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(tp)]
    for step in range(3):  # both parities of the buffers, the counter advancing
        for r in range(tp):
            for y in ys[r]:
                y.fill_(float("nan"))
        _emulated_step(torch, ops, native, fmt, shards, xs, ys, bufs, seqs, dones, packed)
        torch.cuda.synchronize()
        assert ops.device_error() == 0
        for j, (M, K) in enumerate(shapes):
            # each shard's rows are the plain matvec's rows bit for bit, on every rank
            # (independent launches: the warp-ring kernel, as the row-split matvec)
            plain = torch.cat([ops.matvec_packed(fmt, shards[r][j][0], xs[j]) if packed
                               else ops.matvec(fmt, *shards[r][j], xs[j], independent=True) for r in range(tp)])
            for r in range(tp):
                assert torch.equal(ys[r][j], plain), (step, r, j)
            if step == 0:
                w, s = full_w[j]
                ref = oracle.matmul_q4q8(w, s.astype(np.float16).astype(np.float32), xs[j].cpu().numpy())
                assert rel_err(ys[0][j].cpu().numpy(), ref) <= YTOL
        assert all(int(q.item()) == step + 1 for q in seqs) or tp == 1


def test_rowsplit_wait_times_out_when_a_peer_never_writes(cuda):
    torch = cuda
    from asmllm_b200 import native, ops, synth

    fmt, tp, M, K = native.FMT_Q4_0, 2, 512, 4096
    w, s = synth.q4_0_weights(M, K, seed=7)
    packed = ops.pack_rows(fmt, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half())
    x = torch.from_numpy(synth.activation(K, seed=8)).cuda()
    y = torch.zeros(tp * M, device="cuda")
    own = torch.zeros(2 * tp * M, dtype=torch.int64, device="cuda")
    peer = torch.zeros(2 * tp * M, dtype=torch.int64, device="cuda")  # "rank 1": nobody runs it
    seq, done = torch.zeros(1, dtype=torch.int32, device="cuda"), torch.zeros(1, dtype=torch.int32, device="cuda")
    L = native.lib()
    assert ops.device_error() == 0
    prev = ops.set_option("xchg_wait_us", 2000)
    try:
        xchg = (ctypes.c_void_p * 8)(own.data_ptr(), peer.data_ptr(), *([0] * 6))
        native.check(L.asm_matvec_rowsplit_async(fmt, packed.data_ptr(), None, x.data_ptr(), y.data_ptr(), M, K, tp,
                                                 0, xchg, seq.data_ptr(), ops.MV_PACKED, None))
        wt = native.RowsplitWait()
        wt.n, wt.tp, wt.rank = 1, tp, 0
        wt.own[0], wt.y_full[0], wt.M[0] = own.data_ptr(), y.data_ptr(), M
        wt.seq, wt.done = seq.data_ptr(), done.data_ptr()
        native.check(L.asm_rowsplit_wait_async(ctypes.byref(wt), None))
        torch.cuda.synchronize()
        err = ops.device_error()
    finally:
        ops.set_option("xchg_wait_us", prev)
    assert err & native.DEVERR_XCHG_TIMEOUT
    # this rank's own rows were computed and the words for "rank 1" were stored
    assert torch.equal(y[:M], ops.matvec_packed(fmt, packed, x))
    assert int((peer[2 * M:3 * M] >> 32).min().item()) == 1  # [parity 1][source rank 0]: sequence 1
    # the library is still usable: the next plain matvec runs and reports nothing
    ops.matvec_packed(fmt, packed, x)
    torch.cuda.synchronize()
    assert ops.device_error() == 0


@pytest.mark.parametrize("K,kernel", [(4096, 1), (8192, 2)], ids=["warp-ring", "row-stage"])
def test_tp_residual_exchange_times_out_when_a_peer_never_writes(cuda, K, kernel):
    """A tp = 2 row-parallel projection (the decode step's o / down) whose peer exchange
    buffer is a local buffer nobody writes: the kernel's bounded wait must run out."""
    torch = cuda
    from asmllm_b200 import native, ops, synth

    M = 1024
    w, s = synth.q4_0_weights(M, K, seed=9)
    dw, ds = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda().half()
    x = torch.from_numpy(synth.activation(K, seed=10)).cuda()
    resid = torch.ones(M, device="cuda")
    own = torch.zeros(2 * 2 * M, dtype=torch.int64, device="cuda")
    peer = torch.zeros(2 * 2 * M, dtype=torch.int64, device="cuda")
    ar_seq, ar_done = torch.zeros(1, dtype=torch.int32, device="cuda"), torch.zeros(1, dtype=torch.int32, device="cuda")
    d = native.FusedMatvec()
    d.fmt, d.epilogue = native.FMT_Q4_0, native.EPI_RESIDUAL
    d.qweights, d.scales, d.x, d.y = dw.data_ptr(), ds.data_ptr(), x.data_ptr(), resid.data_ptr()
    d.M, d.K = M, K
    d.tp, d.tp_rank, d.xchg_rows = 2, 0, M
    d.xchg[0], d.xchg[1] = own.data_ptr(), peer.data_ptr()
    d.ar_seq, d.ar_done = ar_seq.data_ptr(), ar_done.data_ptr()
    assert ops.device_error() == 0
    prev = ops.set_option("xchg_wait_us", 2000)
    prev_kernel = ops.set_option("mv_kernel", kernel)  # 1: warp rings, 2: row stages
    try:
        native.check(native.lib().asm_fused_matvec_async(ctypes.byref(d), None))
        torch.cuda.synchronize()
        err = ops.device_error()
    finally:
        ops.set_option("xchg_wait_us", prev)
        ops.set_option("mv_kernel", prev_kernel)
    assert err & native.DEVERR_XCHG_TIMEOUT
    # the partials went out: rank 0's rows in "rank 1's" buffer, [parity 1][source rank 0], sequence 1
    assert int((peer[2 * M:3 * M] >> 32).min().item()) == 1
    # with the missing partial read as 0 the residual stream got this rank's rows
    ref = torch.ones(M, device="cuda") + ops.matvec(native.FMT_Q4_0, dw, ds, x)
    assert rel_err(resid.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
    assert ops.device_error() == 0
