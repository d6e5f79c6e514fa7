"""Batched greedy decode: B sequences of one Llama-style model in lockstep.

The reference decodes one sequence at a time (THRISHAL12345/asmllm
src/runtime/generate.py:255-326, AsmEngineForward.forward_token; its seven
matvecs per layer are asm_matmul_q4 calls, generate.py:227-231).  Here the
B sequences share every weight read: each projection is one tensor-core
batched product over the B token rows (asm_gemm_tiles_async), and the glue
between them runs per row (asm_rows_norm_tiles_async,
asm_attention_batch_async, asm_rows_swiglu_tiles_async, asm_rows_argmax_async,
asm_rows_advance_async).  Every step is a fixed sequence of launches reading
the position from the device, captured once into CUDA graphs.

Tensor parallelism (tp > 1, one process per GPU): the same Megatron split as
the batch-1 decoder (q/k/v, gate/up and the lm_head by rows; o and down by
columns), with an NCCL all-reduce of the [B, dim] partial rows after each
row-parallel projection and a max all-reduce of the per-row argmax keys
(signed-orderable (value, index) words) after the lm_head.  The weights are
the unit-seeded ones of asmllm_b200.decode.make_weights, so the model is the
same for every tp and equals the batch-1 decoder's model for the same seed.
"""
from __future__ import annotations

import numpy as np

from . import ops
from .decode import LlamaShape, make_weights, rope_table, shard_plan
from .native import FMT_Q4_0


class BatchDecoder:
    def __init__(self, shape: LlamaShape, batch: int, ctx: int = 512, max_tokens: int | None = None, seed: int = 0,
                 fmt: int = FMT_Q4_0, device=None, tp: int = 1, tp_rank: int = 0, group=None, weights=None):
        import torch

        self.torch = torch
        self.shape = s = shape
        self.B = B = int(batch)
        self.fmt = fmt
        self.ctx = ctx
        self.max_tokens = max_tokens or ctx
        if B < 1:
            raise ValueError("batch must be >= 1")
        if s.head_dim != 128:
            raise ValueError("head_dim must be 128")
        self.shard = sh = shard_plan(s, tp, tp_rank)
        self.tp, self.tp_rank, self.group = tp, tp_rank, group
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        # weights handed in (e.g. a batch-1 decoder's) stay under their owner's static declaration
        self._owns = weights is None
        W = weights if weights is not None else make_weights(s, sh, seed, fmt, dev)
        self.layers, self.final_norm, self.lm_head, self.embed = W["layers"], W["final_norm"], W["lm_head"], W["embed"]
        if self._owns:
            for L in self.layers:
                for k in ("wqkv", "wo", "wgu", "wdown"):
                    ops.mark_static(*L[k])
            ops.mark_static(*self.lm_head)
        hd = s.head_dim
        self.nh, self.nkv, self.ffn = len(sh.heads), len(sh.kv_heads), len(sh.ffn)
        self.vocab_l = len(sh.vocab)
        self.rope = torch.from_numpy(rope_table(ctx, hd, s.theta)).to(dev)
        # per layer: [B][ctx][n_kv][hd] fp16, each sequence's cache contiguous
        self.k_cache = [torch.zeros((B, ctx, self.nkv, hd), dtype=torch.float16, device=dev)
                        for _ in range(s.n_layers)]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        self.x = torch.zeros((B, s.dim), device=dev)
        self.qkv = torch.zeros((B, (self.nh + 2 * self.nkv) * hd), device=dev)
        self.delta = torch.zeros((B, s.dim), device=dev)
        self.gu = torch.zeros((B, 2 * self.ffn), device=dev)
        self.logits = torch.zeros((B, self.vocab_l), device=dev)
        self.keys = torch.zeros(B, dtype=torch.int64, device=dev)
        self.t_dim = torch.zeros(ops.act_tiles_bytes(B, s.dim), dtype=torch.uint8, device=dev)
        self.t_attn = torch.zeros(ops.act_tiles_bytes(B, self.nh * hd), dtype=torch.uint8, device=dev)
        self.t_h = torch.zeros(ops.act_tiles_bytes(B, self.ffn), dtype=torch.uint8, device=dev)
        self.tokens = torch.zeros((B, self.max_tokens), dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        # the reference divides the scores by np.sqrt(head_dim, dtype=np.float32)
        self.sqrt_hd = float(np.sqrt(np.float32(hd), dtype=np.float32))
        self.n_prompt = 0
        self._graphs = {}

    # ------------------------------------------------------------------ steps
    def _all_reduce(self, t, op):
        import torch.distributed as dist

        dist.all_reduce(t, op=op, group=self.group)

    def launch_step(self) -> None:
        """One decode step for all B rows on the current stream."""
        import torch.distributed as dist

        s, fmt, B = self.shape, self.fmt, self.B
        for li, L in enumerate(self.layers):
            if li == 0:
                ops.rows_norm_tiles(self.x, self.t_dim, L["attn_norm"], s.eps, embed=self.embed, tokens=self.tokens,
                                    pos=self.pos)
            else:
                ops.rows_norm_tiles(self.x, self.t_dim, L["attn_norm"], s.eps, delta=self.delta)
            ops.gemm_tiles(fmt, *L["wqkv"], self.t_dim, B, out=self.qkv)
            ops.attention_batch(self.qkv, self.k_cache[li], self.v_cache[li], self.rope, self.pos, self.t_attn,
                                self.nh, self.nkv, self.ctx, self.sqrt_hd)
            ops.gemm_tiles(fmt, *L["wo"], self.t_attn, B, out=self.delta)
            if self.tp > 1:
                self._all_reduce(self.delta, dist.ReduceOp.SUM)
            ops.rows_norm_tiles(self.x, self.t_dim, L["ffn_norm"], s.eps, delta=self.delta)
            ops.gemm_tiles(fmt, *L["wgu"], self.t_dim, B, out=self.gu)
            ops.rows_swiglu_tiles(self.gu, self.t_h)
            ops.gemm_tiles(fmt, *L["wdown"], self.t_h, B, out=self.delta)
            if self.tp > 1:
                self._all_reduce(self.delta, dist.ReduceOp.SUM)
        ops.rows_norm_tiles(self.x, self.t_dim, self.final_norm, s.eps, delta=self.delta)
        ops.gemm_tiles(fmt, *self.lm_head, self.t_dim, B, out=self.logits)
        ops.rows_argmax(self.logits, self.keys, offset=self.shard.vocab.start)
        if self.tp > 1:
            self._all_reduce(self.keys, dist.ReduceOp.MAX)
        ops.rows_advance(self.keys, self.tokens, self.pos, self.n_prompt)

    @property
    def launches_per_step(self) -> int:
        return 7 * self.shape.n_layers + 5

    def reset(self, prompts) -> None:
        """Loads B prompts of one length; the next step runs position 0."""
        prompts = np.asarray(prompts, dtype=np.int64)
        if prompts.ndim != 2 or prompts.shape[0] != self.B:
            raise ValueError(f"prompts must be [B={self.B}, length]")
        P = prompts.shape[1]
        if not 1 <= P <= self.max_tokens:
            raise ValueError("prompt length must be in [1, max_tokens]")
        if P != self.n_prompt:  # n_prompt is part of the captured launches
            self.n_prompt = P
            self._graphs = {}
        t = np.zeros((self.B, self.max_tokens), dtype=np.int32)
        t[:, :P] = prompts
        self.tokens.copy_(self.torch.from_numpy(t))
        self.pos.zero_()

    def step(self, n: int = 1) -> None:
        for _ in range(n):
            self.launch_step()

    def _graph(self, k: int):
        g = self._graphs.get(k)
        if g is None:
            torch = self.torch
            saved_pos, saved_tok = self.pos.clone(), self.tokens.clone()
            self.launch_step()  # one eager step: kernel attributes, NCCL communicators
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(k):
                    self.launch_step()
            torch.cuda.synchronize()
            self.pos.copy_(saved_pos)
            self.tokens.copy_(saved_tok)
            self._graphs[k] = g
        return g

    def run(self, n: int, chunk: int = 16) -> None:
        while n >= chunk:
            self._graph(chunk).replay()
            n -= chunk
        for _ in range(n):
            self._graph(1).replay()

    def generate(self, prompts, n_new: int, chunk: int = 16) -> np.ndarray:
        """Greedy decode of B prompts (teacher-forced through the prompt, then
        n_new generated tokens each); returns [B, n_new] token ids."""
        prompts = np.asarray(prompts)
        if prompts.shape[1] + n_new > self.max_tokens:
            raise ValueError("prompt + n_new exceeds max_tokens")
        self.reset(prompts)
        self.run(prompts.shape[1] - 1 + n_new, chunk)
        self.torch.cuda.synchronize()
        P = prompts.shape[1]
        return self.tokens[:, P: P + n_new].cpu().numpy()

    def position(self) -> int:
        return int(self.pos.item())

    def close(self) -> None:
        self._graphs = {}
        if self._owns:
            for L in self.layers:
                for k in ("wqkv", "wo", "wgu", "wdown"):
                    ops.unmark_static(*L[k])
            ops.unmark_static(*self.lm_head)
