"""Host side of tensor-parallel decode, on CPU with the gloo backend
(world size 2): the shard plan, the unit-seeded weights (the shards of a
2-rank model concatenate to the 1-rank model), and the all-gather the
decoder uses to exchange its IPC handles."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from asmllm_b200 import decode as D

SMALL = D.LlamaShape(n_layers=1, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024, vocab=512)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = D.shard_plan(SMALL, world, rank)
        W = D.make_weights(SMALL, sh, 11, D.FMT_Q4_0, torch.device("cpu"))
        L = W["layers"][0]
        mine = {k: (L[k][0].clone(), L[k][1].clone()) for k in ("wqkv", "wo", "wgu", "wdown")}
        mine["lm_head"] = W["lm_head"]
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        handles = [None] * world
        dist.all_gather_object(handles, bytes([rank]) * 64)  # as the decoder exchanges its 64-byte IPC handles
        if rank == 0:  # numpy copies: tensors would travel as shared memory of an exiting process
            out.put(([{k: tuple(t.numpy() for t in v) for k, v in g.items()} for g in gathered], handles))
    finally:
        dist.destroy_process_group()


def test_shard_plan_splits():
    sh = D.shard_plan(D.LLAMA2_70B, 8, 5)
    assert sh.heads == range(40, 48) and sh.kv_heads == range(5, 6)
    assert sh.ffn == range(17920, 21504) and sh.vocab == range(20000, 24000)
    for tp in (1, 2, 4, 8):
        parts = [D.shard_plan(D.LLAMA2_70B, tp, r) for r in range(tp)]
        assert sum(len(p.heads) for p in parts) == 64 and sum(len(p.ffn) for p in parts) == 28672
    with pytest.raises(ValueError):
        D.shard_plan(D.LLAMA_7B, 2, 0)  # FFN 11008 / 2 is not a whole number of 256-row units
    with pytest.raises(ValueError):
        D.shard_plan(D.LLAMA2_70B, 16, 0)


def test_two_rank_shards_concatenate_to_the_one_rank_model():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, handles = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert handles == [bytes([0]) * 64, bytes([1]) * 64]
    gathered = [{k: tuple(torch.from_numpy(a) for a in v) for k, v in g.items()} for g in gathered]
    full = D.make_weights(SMALL, D.shard_plan(SMALL, 1, 0), 11, D.FMT_Q4_0, torch.device("cpu"))
    L = full["layers"][0]
    hd, nh, nkv = SMALL.head_dim, SMALL.n_heads, SMALL.n_kv_heads
    for i in (0, 1):  # quants, scales
        # q/k/v rows: each rank holds [its q heads; its k heads; its v heads]
        q_rows = torch.cat([g["wqkv"][i][: nh // 2 * hd] for g in gathered])
        k_rows = torch.cat([g["wqkv"][i][nh // 2 * hd: (nh // 2 + nkv // 2) * hd] for g in gathered])
        v_rows = torch.cat([g["wqkv"][i][(nh // 2 + nkv // 2) * hd:] for g in gathered])
        assert torch.equal(torch.cat([q_rows, k_rows, v_rows]), L["wqkv"][i])
        assert torch.equal(torch.cat([g["wo"][i] for g in gathered], 1), L["wo"][i])
        assert torch.equal(torch.cat([g["wgu"][i] for g in gathered]), L["wgu"][i])
        assert torch.equal(torch.cat([g["wdown"][i] for g in gathered], 1), L["wdown"][i])
        assert torch.equal(torch.cat([g["lm_head"][i] for g in gathered]), full["lm_head"][i])
