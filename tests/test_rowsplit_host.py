"""Host side of the row-split matvec, on CPU with the gloo backend (world size
2): the shard ranges, the exchange of IPC handles in rank order, and the
property the GPU path relies on -- each rank's rows computed alone and laid
out at rank * M concatenate to the unsplit matvec (the oracle, bit for bit:
a row's products do not depend on the other rows)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from asmllm_b200 import rowsplit, synth


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        handles = rowsplit.exchange_handles(bytes([65 + rank]) * 64)
        from oracle import oracle as O  # the CPU restatement (test infrastructure)

        M_total, K = 96, 256
        w, s = synth.q4_0_weights(M_total, K, seed=5)
        x = synth.activation(K, seed=6)
        a, b = rowsplit.shard_range(M_total, world, rank)
        mine = O.matmul_q4q8(w[a:b], s[a:b], x)  # this rank's rows alone
        full = [None] * world
        dist.all_gather_object(full, (a, mine))
        if rank == 0:
            out.put((handles, full, O.matmul_q4q8(w, s, x)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_gather_handles_and_rows():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        handles, parts, ref = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    assert handles == [b"A" * 64, b"B" * 64]  # rank order
    y = np.empty_like(ref)
    for a, rows in parts:
        y[a:a + len(rows)] = rows
    assert np.array_equal(y, ref)


def test_shard_ranges_cover_the_rows_once():
    for tp in (1, 2, 3, 4, 8):
        M = 4096 * tp
        got = [rowsplit.shard_range(M, tp, r) for r in range(tp)]
        assert got[0][0] == 0 and got[-1][1] == M
        assert all(got[r][1] == got[r + 1][0] for r in range(tp - 1))
        assert all(b - a == 4096 for a, b in got)
    with pytest.raises(ValueError):
        rowsplit.shard_range(10, 3, 0)
    with pytest.raises(ValueError):
        rowsplit.shard_range(8, 2, 2)
    assert rowsplit.gather_buffer_bytes(4096, 8) == 2 * 8 * 4096 * 8
