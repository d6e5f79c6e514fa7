"""Batch-1 Llama decode on one B200 through the fused C-ABI entries.

The reference decodes one token at a time in
``AsmEngineForward.forward_token`` (THRISHAL12345/asmllm
src/runtime/generate.py:255-326) and picks the next token with a numpy
argmax (generate.py:410-411).  ``LlamaDecoder`` runs the same step as five
launches per layer plus one for the lm_head:

  1. q/k/v matvec (rows [wq; wk; wv]) with RMSNorm + Q8_0 quantize in its
     prologue (layer 0: the source row is the token's embedding, copied to
     the residual stream x by CTA 0);
  2. RoPE + fp16 KV append + attention, output quantized to a Q8_0 image;
  3. o matvec from that image, residual add into x in its epilogue;
  4. gate/up matvec (rows interleaved gate_0, up_0, gate_1, ...) with RMSNorm
     in its prologue and silu(gate)*up + Q8_0 quantize in its epilogue;
  5. down matvec from that image, residual add into x;
  and the lm_head matvec with the final RMSNorm in its prologue and the
  argmax in its epilogue, which writes the next token id and advances the
  position.

The position and the token ids live in device memory, so one captured CUDA
graph of a step replays for every token with no host round trip.  The
default engine goes further: the same program runs as ONE persistent
cooperative kernel for all the steps of a run (asm_decode_run_async), each CTA
streaming its share of every weight matrix through a shared-memory ring
without stopping between operations; the two engines agree bit for bit.  Weights
are random-init in GGUF Q4_0 (or Q8_0) form with fp16 scales, generated on
the device from a seed; norm weights are 1 + N(0, 0.01) fp32.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import native, ops
from .native import FMT_Q4_0, FMT_Q8_0, FusedMatvec


@dataclass(frozen=True)
class LlamaShape:
    n_layers: int
    dim: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-5
    theta: float = 10000.0

    @property
    def qkv_rows(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def weight_bytes(self, fmt: int = FMT_Q4_0) -> int:
        """GGUF-size bytes of every linear weight read per token (18 B or 34 B per block)."""
        bb = 18 if fmt == FMT_Q4_0 else 34
        per_layer = (self.qkv_rows * self.dim + self.dim * self.n_heads * self.head_dim
                     + 2 * self.ffn * self.dim + self.dim * self.ffn) // 32 * bb
        return self.n_layers * per_layer + self.vocab * self.dim // 32 * bb

    def kv_bytes(self, pos: int) -> int:
        """fp16 KV bytes the attention of one token at position pos reads (all layers)."""
        return self.n_layers * 2 * (pos + 1) * self.n_kv_heads * self.head_dim * 2


LLAMA_7B = LlamaShape(n_layers=32, dim=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008, vocab=32000)
LLAMA2_70B = LlamaShape(n_layers=80, dim=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=32000)


def rope_table(ctx: int, head_dim: int, theta: float) -> np.ndarray:
    """fp32 [ctx][head_dim/2][2] = (cos, sin) of pos * freq_i, computed with the
    reference's numpy expressions (tests/reference/ops.py:125-128) in float32."""
    freqs = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    angles = np.arange(ctx, dtype=np.float32)[:, None] * freqs[None, :]
    assert freqs.dtype == np.float32 and angles.dtype == np.float32
    return np.ascontiguousarray(np.stack([np.cos(angles), np.sin(angles)], axis=-1))


def _random_weights(torch, fmt, M, K, gen, dev):
    """GGUF-style random block weights: Q4_0 nibbles U[0,15] with d = |N(0,0.02)|,
    or Q8_0 int8 U[-127,127] with d = |N(0,0.002)|; fp16 scales."""
    nb = K // 32
    if fmt == FMT_Q4_0:
        qs = torch.randint(0, 256, (M, nb, 16), dtype=torch.uint8, device=dev, generator=gen)
        d = torch.randn((M, nb), device=dev, generator=gen).abs_().mul_(0.02).half()
    else:
        qs = torch.randint(-127, 128, (M, nb, 32), dtype=torch.int8, device=dev, generator=gen)
        d = torch.randn((M, nb), device=dev, generator=gen).abs_().mul_(0.002).half()
    return qs, d


LM_UNIT = 16    # lm_head rows per generation unit
FFN_UNIT = 256  # gate/up rows (and down-proj columns) per generation unit


def _unit_seed(seed: int, layer: int, kind: int, index: int) -> int:
    """Seed of one generation unit (a head, an FFN chunk, an lm_head chunk):
    the random model does not depend on how it is sharded."""
    h = (seed * 0x9E3779B97F4A7C15 + 0x632BE59BD9B4E019) & 0xFFFFFFFFFFFFFFFF
    for v in (layer + 1, kind + 1, index + 1):
        h = ((h ^ v) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h & 0x7FFFFFFFFFFFFFFF


_Q, _K, _V, _O, _G, _U, _D, _NA, _NF, _LM, _FN, _EMB = range(12)


def _f32_short(v) -> float:
    """A float32 metadata value as the shortest decimal that rounds to it
    (GGUF stores 1e-5 as float32 9.99999974e-06; the model shape keeps 1e-05)."""
    return float(str(np.float32(v)))


@dataclass(frozen=True)
class Shard:
    """This rank's slice of a tensor-parallel model (Megatron-style split)."""
    tp: int
    rank: int
    heads: range      # query heads (column-parallel q, row-parallel o)
    kv_heads: range
    ffn: range        # FFN rows (column-parallel gate/up, row-parallel down)
    vocab: range      # lm_head rows


def shard_plan(shape: LlamaShape, tp: int, rank: int) -> Shard:
    s = shape
    if not 1 <= tp <= 8 or not 0 <= rank < tp:
        raise ValueError("tp must be in [1, 8] and 0 <= rank < tp")
    if s.n_heads % tp or s.n_kv_heads % tp:
        raise ValueError(f"{s.n_heads} query / {s.n_kv_heads} KV heads do not split over {tp} ranks")
    if (s.ffn // tp) % FFN_UNIT or s.ffn % tp:
        raise ValueError(f"FFN {s.ffn} / {tp} is not a multiple of {FFN_UNIT}")
    if (s.n_heads // tp * s.head_dim) % 256:
        raise ValueError("each rank's n_heads * head_dim must be a multiple of 256")
    if tp > 1 and s.vocab % (tp * LM_UNIT):  # one rank: the last unit may be partial
        raise ValueError(f"vocab {s.vocab} is not a multiple of {tp} * {LM_UNIT}")
    def part(n):
        return range(rank * n // tp, (rank + 1) * n // tp)
    return Shard(tp, rank, part(s.n_heads), part(s.n_kv_heads), part(s.ffn), part(s.vocab))


def make_weights(shape: LlamaShape, sh: Shard, seed: int, fmt: int, dev) -> dict:
    """This rank's weights (torch tensors on `dev`): per layer wqkv (rows
    [q heads; k heads; v heads]), wo (its heads' columns), wgu (its FFN rows,
    gate/up interleaved), wdown (its FFN columns), norms; plus the lm_head
    rows of its vocabulary slice, the final norm and the whole embedding.
    Every unit (head, FFN chunk, vocabulary chunk, norm) has its own seed."""
    import torch

    s = shape
    gen = torch.Generator(device=dev)
    hd, nb_dim = s.head_dim, s.dim // 32
    bpb = 16 if fmt == FMT_Q4_0 else 32

    def rows(layer, kind, index, n, K):  # n rows of K columns
        gen.manual_seed(_unit_seed(seed, layer, kind, index))
        return _random_weights(torch, fmt, n, K, gen, dev)

    def cols(layer, kind, index, M, n):  # M rows of n columns (a column block)
        return rows(layer, kind, index, M, n)

    def cat_rows(parts):
        return (torch.cat([p[0] for p in parts]).contiguous(), torch.cat([p[1] for p in parts]).contiguous())

    def cat_cols(parts):
        return (torch.cat([p[0] for p in parts], 1).contiguous(), torch.cat([p[1] for p in parts], 1).contiguous())

    def vec(layer, kind, n, scale=0.01, base=1.0):
        gen.manual_seed(_unit_seed(seed, layer, kind, 0))
        return base + scale * torch.randn(n, device=dev, generator=gen)

    nh_l, nkv_l, ffn_l = len(sh.heads), len(sh.kv_heads), len(sh.ffn)
    layers = []
    for li in range(s.n_layers):
        L = {}
        L["wqkv"] = cat_rows([rows(li, _Q, h, hd, s.dim) for h in sh.heads]
                             + [rows(li, _K, j, hd, s.dim) for j in sh.kv_heads]
                             + [rows(li, _V, j, hd, s.dim) for j in sh.kv_heads])
        L["wo"] = cat_cols([cols(li, _O, h, s.dim, hd) for h in sh.heads])
        c0, c1 = sh.ffn.start // FFN_UNIT, sh.ffn.stop // FFN_UNIT
        g = cat_rows([rows(li, _G, c, FFN_UNIT, s.dim) for c in range(c0, c1)])
        u = cat_rows([rows(li, _U, c, FFN_UNIT, s.dim) for c in range(c0, c1)])
        # rows gate_0, up_0, gate_1, up_1, ...: a pair is finished by one warp
        L["wgu"] = (torch.stack([g[0], u[0]], 1).reshape(2 * ffn_l, nb_dim, bpb).contiguous(),
                    torch.stack([g[1], u[1]], 1).reshape(2 * ffn_l, nb_dim).contiguous())
        del g, u
        L["wdown"] = cat_cols([cols(li, _D, c, s.dim, FFN_UNIT) for c in range(c0, c1)])
        L["attn_norm"] = vec(li, _NA, s.dim)
        L["ffn_norm"] = vec(li, _NF, s.dim)
        layers.append(L)
    final_norm = vec(-1, _FN, s.dim)
    lm_head = cat_rows([rows(-1, _LM, c, LM_UNIT, s.dim)
                        for c in range(sh.vocab.start // LM_UNIT, -(-sh.vocab.stop // LM_UNIT))])
    if lm_head[0].shape[0] != len(sh.vocab):  # partial last unit (one rank only)
        lm_head = tuple(t[: len(sh.vocab)].contiguous() for t in lm_head)
    gen.manual_seed(_unit_seed(seed, -1, _EMB, 0))
    return {"layers": layers, "final_norm": final_norm, "lm_head": lm_head,
            "embed": torch.randn((s.vocab, s.dim), device=dev, generator=gen)}


class LlamaDecoder:
    """Random-init Llama-style model resident on one GPU (or this rank's slice
    of it, tp > 1), decoded at batch 1.

    Tensor parallelism: q/k/v, gate/up and the lm_head are split by rows
    (heads, FFN rows, vocabulary), o and down by columns; the row-parallel
    projections exchange their partial rows over NVLink inside the matvec
    kernel (peer stores into every rank's exchange buffer, each rank sums in
    rank order), and the lm_head ranks exchange their maxima.  Every rank
    holds the full residual stream, embedding and norms.  The weights are
    generated per unit (head, 256-row FFN chunk, 16-row vocabulary chunk)
    from `seed`, so the model is the same whatever tp is.
    """

    def __init__(self, shape: LlamaShape, ctx: int = 512, max_tokens: int | None = None, seed: int = 0,
                 fmt: int = FMT_Q4_0, device=None, tp: int = 1, tp_rank: int = 0, group=None, weights=None):
        import torch

        self.torch = torch
        self.shape = s = shape
        self.fmt = fmt
        self.ctx = ctx
        self.max_tokens = max_tokens or ctx
        if s.head_dim != 128:
            raise ValueError("head_dim must be 128")
        if s.dim % 256 or s.ffn % 256 or (s.n_heads * s.head_dim) % 256:
            raise ValueError("dim, ffn and n_heads*head_dim must be multiples of 256 (whole fp16 scale rows)")
        self.shard = sh = shard_plan(s, tp, tp_rank)
        self.tp, self.tp_rank = tp, tp_rank
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        W = weights if weights is not None else make_weights(s, sh, seed, fmt, dev)
        self.layers, self.final_norm, self.lm_head, self.embed = W["layers"], W["final_norm"], W["lm_head"], W["embed"]
        hd = s.head_dim
        nh_l, nkv_l, ffn_l = len(sh.heads), len(sh.kv_heads), len(sh.ffn)
        for L in self.layers:
            for k in ("wqkv", "wo", "wgu", "wdown"):
                ops.mark_static(*L[k])
        ops.mark_static(*self.lm_head)

        self.rope = torch.from_numpy(rope_table(ctx, s.head_dim, s.theta)).to(dev)
        self.k_cache = torch.zeros((s.n_layers, ctx, nkv_l, s.head_dim), dtype=torch.float16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.x = torch.zeros(s.dim, device=dev)
        self.qkv = torch.zeros((nh_l + 2 * nkv_l) * hd, device=dev)
        self.img_attn = torch.zeros(ops.act_image_bytes(nh_l * hd), dtype=torch.uint8, device=dev)
        self.h = torch.zeros(ffn_l, device=dev)
        self.img_h = torch.zeros(ops.act_image_bytes(ffn_l), dtype=torch.uint8, device=dev)
        self.counters = torch.zeros(ffn_l // 32, dtype=torch.int32, device=dev)
        self.logits = torch.zeros(len(sh.vocab), device=dev)
        self.best = torch.zeros(2, dtype=torch.int64, device=dev)
        self.done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(self.max_tokens, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ar_seq = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ar_done = torch.zeros(1, dtype=torch.int32, device=dev)
        # the reference divides the scores by np.sqrt(head_dim, dtype=np.float32)
        self.sqrt_hd = float(np.sqrt(np.float32(s.head_dim), dtype=np.float32))
        self.n_prompt = 0
        self._descs = None
        self._graphs = {}
        self._handle = None
        self._xchg_own = None
        self._xchg_peers = []
        self._xchg = [0] * 8
        if tp > 1:
            self._open_exchange(group)

    def _open_exchange(self, group):
        """Exchange buffers: one per rank (CUDA IPC), every rank maps all of them."""
        import torch.distributed as dist

        L = native.lib()
        nbytes = 2 * self.tp * self.shape.dim * 8
        ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        native.check(L.asm_ipc_alloc(nbytes, ctypes.byref(ptr), handle))
        self._xchg_own = ptr
        handles = [None] * self.tp
        dist.all_gather_object(handles, handle.raw, group=group)
        for r, hr in enumerate(handles):
            if r == self.tp_rank:
                self._xchg[r] = ptr.value
                continue
            peer = ctypes.c_void_p()
            native.check(L.asm_ipc_open(hr, ctypes.byref(peer)))
            self._xchg_peers.append(peer)
            self._xchg[r] = peer.value
        dist.barrier(group=group)

    def _tp_fields(self, d, epi):
        if self.tp > 1 and epi in (native.EPI_RESIDUAL, native.EPI_ARGMAX):
            d.tp, d.tp_rank, d.xchg_rows = self.tp, self.tp_rank, self.shape.dim
            d.vocab_offset = self.shard.vocab.start if epi == native.EPI_ARGMAX else 0
            for r in range(self.tp):
                d.xchg[r] = self._xchg[r]
            d.ar_seq, d.ar_done = self.ar_seq.data_ptr(), self.ar_done.data_ptr()

    # ------------------------------------------------------------------ launches
    def _mv(self, w, epi, M, K, **kw) -> FusedMatvec:
        d = FusedMatvec()
        d.fmt, d.epilogue = self.fmt, epi
        d.qweights, d.scales = w[0].data_ptr(), w[1].data_ptr()
        d.M, d.K = M, K
        d.eps = self.shape.eps
        d.vocab, d.max_tokens, d.n_prompt = self.shape.vocab, self.max_tokens, self.n_prompt
        d.tokens, d.pos = self.tokens.data_ptr(), self.pos.data_ptr()
        for k, v in kw.items():
            setattr(d, k, v.data_ptr() if hasattr(v, "data_ptr") else v)
        self._tp_fields(d, epi)
        return d

    def _build(self):
        s, sh = self.shape, self.shard
        nh_l, nkv_l, ffn_l = len(sh.heads), len(sh.kv_heads), len(sh.ffn)
        qdim = nh_l * s.head_dim
        kv_layer = nkv_l * s.head_dim * self.ctx
        descs = []
        for li, L in enumerate(self.layers):
            src = dict(embed=self.embed, x_copy=self.x) if li == 0 else dict(x=self.x)
            descs.append(("mv", self._mv(L["wqkv"], native.EPI_STORE, (nh_l + 2 * nkv_l) * s.head_dim, s.dim,
                                         norm_w=L["attn_norm"], y=self.qkv, **src)))
            descs.append(("attn", (self.qkv.data_ptr(), self.k_cache.data_ptr() + 2 * li * kv_layer,
                                   self.v_cache.data_ptr() + 2 * li * kv_layer, self.rope.data_ptr(),
                                   self.pos.data_ptr(), self.img_attn.data_ptr(), nh_l, nkv_l,
                                   s.head_dim, self.ctx, self.sqrt_hd)))
            descs.append(("mv", self._mv(L["wo"], native.EPI_RESIDUAL, s.dim, qdim, image=self.img_attn, y=self.x)))
            descs.append(("mv", self._mv(L["wgu"], native.EPI_SWIGLU, 2 * ffn_l, s.dim, x=self.x,
                                         norm_w=L["ffn_norm"], y=self.h, h=self.h, image_out=self.img_h,
                                         counters=self.counters)))
            descs.append(("mv", self._mv(L["wdown"], native.EPI_RESIDUAL, s.dim, ffn_l, image=self.img_h, y=self.x)))
        descs.append(("mv", self._mv(self.lm_head, native.EPI_ARGMAX, len(sh.vocab), s.dim, x=self.x,
                                     norm_w=self.final_norm, y=self.logits, best=self.best, done=self.done)))
        self._descs = descs

    @property
    def launches_per_step(self) -> int:
        return 5 * self.shape.n_layers + 1

    def launch_step(self, stream=None):
        """Enqueue one decode step (token at *pos -> logits, next token, pos+1)."""
        if self._descs is None:
            self._build()
        L = native.lib()
        st = ctypes.c_void_p(stream if stream is not None else self.torch.cuda.current_stream().cuda_stream)
        for kind, d in self._descs:
            if kind == "mv":
                rc = L.asm_fused_matvec_async(ctypes.byref(d), st)
            else:
                rc = L.asm_attention_decode_async(*d, st)
            if rc:
                native.check(rc)

    # ------------------------------------------------------------------ state
    def reset(self, prompt) -> None:
        """Loads the prompt ids; the next step runs position 0."""
        prompt = [int(t) for t in prompt]
        if not 1 <= len(prompt) <= self.max_tokens:
            raise ValueError("prompt length must be in [1, max_tokens]")
        if len(prompt) != self.n_prompt:  # n_prompt is part of the captured launches
            self.n_prompt = len(prompt)
            self._descs = None
            self._graphs = {}
        t = np.zeros(self.max_tokens, dtype=np.int32)
        t[: len(prompt)] = prompt
        self.tokens.copy_(self.torch.from_numpy(t))
        self.pos.zero_()

    def step(self, n: int = 1) -> None:
        """n eager steps on the current stream."""
        for _ in range(n):
            self.launch_step()

    def _graph(self, k: int):
        g = self._graphs.get(k)
        if g is None:
            torch = self.torch
            if self._descs is None:
                self._build()
            saved_pos = self.pos.clone()
            saved_tok = self.tokens.clone()
            self.launch_step()  # one eager step: per-kernel attributes and pointer kinds are cached
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

    def _persistent(self):
        if self.tp > 1:
            raise ValueError("the persistent engine runs one GPU; use engine='graph' with tensor parallelism")
        if self._handle is None:
            s = self.shape
            L = native.lib()
            layers = (native.DecodeLayer * s.n_layers)()
            kv_layer = s.n_kv_heads * s.head_dim * self.ctx * 2  # bytes of one layer's cache
            for i, W in enumerate(self.layers):
                layers[i] = native.DecodeLayer(
                    W["wqkv"][0].data_ptr(), W["wqkv"][1].data_ptr(), W["wo"][0].data_ptr(), W["wo"][1].data_ptr(),
                    W["wgu"][0].data_ptr(), W["wgu"][1].data_ptr(), W["wdown"][0].data_ptr(), W["wdown"][1].data_ptr(),
                    W["attn_norm"].data_ptr(), W["ffn_norm"].data_ptr(),
                    self.k_cache.data_ptr() + i * kv_layer, self.v_cache.data_ptr() + i * kv_layer)
            m = native.DecodeModel()
            m.fmt, m.n_layers, m.dim, m.n_heads, m.n_kv_heads = self.fmt, s.n_layers, s.dim, s.n_heads, s.n_kv_heads
            m.head_dim, m.ffn, m.vocab, m.ctx, m.max_tokens = s.head_dim, s.ffn, s.vocab, self.ctx, self.max_tokens
            m.eps, m.sqrt_head_dim = s.eps, self.sqrt_hd
            m.layers = layers
            m.lm_head, m.lm_scales = self.lm_head[0].data_ptr(), self.lm_head[1].data_ptr()
            for name in ("final_norm", "embed"):
                setattr(m, name, getattr(self, name).data_ptr())
            m.rope_cs = self.rope.data_ptr()
            for name, t in (("x", self.x), ("qkv", self.qkv), ("img_attn", self.img_attn), ("h", self.h),
                            ("img_h", self.img_h), ("counters", self.counters), ("logits", self.logits),
                            ("best", self.best), ("tokens", self.tokens), ("pos", self.pos)):
                setattr(m, name, t.data_ptr())
            h = ctypes.c_void_p()
            native.check(L.asm_decode_create(ctypes.byref(m), ctypes.byref(h)))
            self._handle = h
        return self._handle

    def run(self, n: int, chunk: int = 16, engine: str = "graph") -> None:
        """n decode steps.  engine "graph" (default): CUDA graphs of `chunk`
        steps (and of one step) of the per-operation launches, the same kernels
        as the eager `step`; "persistent": one cooperative launch for all n
        steps.  Each engine is deterministic; the two add a row's block
        products in different fp32 orders, so their logits agree to fp32
        rounding, not bit for bit."""
        if n <= 0:
            return
        if engine == "persistent":
            h = self._persistent()
            st = ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)
            native.check(native.lib().asm_decode_run_async(h, n, self.n_prompt, st))
            return
        if engine != "graph":
            raise ValueError(f"unknown engine {engine!r}")
        while n >= chunk:
            self._graph(chunk).replay()
            n -= chunk
        for _ in range(n):
            self._graph(1).replay()

    def generate(self, prompt, n_new: int, chunk: int = 16, engine: str = "graph") -> list[int]:
        """Greedy decode: the prompt's positions, then n_new generated tokens."""
        if len(prompt) + n_new > self.max_tokens:
            raise ValueError("prompt + n_new exceeds max_tokens")
        self.reset(prompt)
        self.run(len(prompt) - 1 + n_new, chunk, engine)
        self.torch.cuda.synchronize()
        return self.tokens[len(prompt): len(prompt) + n_new].cpu().tolist()

    def position(self) -> int:
        return int(self.pos.item())

    # ------------------------------------------------------------------ export
    def host_weights(self):
        """Host copies in the reference ABI layout (qs + fp32 scales per matrix,
        gate/up de-interleaved) for a CPU re-computation of the step (tp = 1)."""
        if self.tp != 1:
            raise ValueError("host_weights needs the whole model (tp = 1)")
        s = self.shape
        qdim = s.n_heads * s.head_dim

        def host(w):
            return w[0].cpu().numpy(), w[1].float().cpu().numpy()

        out = {"embed": self.embed.cpu().numpy(), "final_norm": self.final_norm.cpu().numpy(),
               "lm_head": host(self.lm_head), "rope": self.rope.cpu().numpy(), "layers": []}
        for L in self.layers:
            q, sc = host(L["wqkv"])
            gq, gs = host(L["wgu"])
            kvr = s.n_kv_heads * s.head_dim
            out["layers"].append({
                "wq": (q[:qdim], sc[:qdim]), "wk": (q[qdim:qdim + kvr], sc[qdim:qdim + kvr]),
                "wv": (q[qdim + kvr:], sc[qdim + kvr:]),
                "wo": host(L["wo"]), "w_gate": (gq[0::2], gs[0::2]), "w_up": (gq[1::2], gs[1::2]),
                "w_down": host(L["wdown"]),
                "attn_norm": L["attn_norm"].cpu().numpy(), "ffn_norm": L["ffn_norm"].cpu().numpy(),
            })
        return out

    # ------------------------------------------------------------------ GGUF
    @classmethod
    def from_gguf(cls, path, ctx: int = 512, max_tokens: int | None = None, device=None):
        """A Llama model from a GGUF file (llama.* metadata, Q4_0 or Q8_0 linear
        weights, F32 norms; the embedding may be F32, F16, Q4_0 or Q8_0).  Each
        linear weight is uploaded once and split on the device."""
        import torch

        from . import gguf as G

        gg = G.GGUFFile(path)
        md = gg.metadata
        arch = md.get("general.architecture", "llama")
        dim = int(md[f"{arch}.embedding_length"])
        n_heads = int(md[f"{arch}.attention.head_count"])
        shape = LlamaShape(n_layers=int(md[f"{arch}.block_count"]), dim=dim, n_heads=n_heads,
                           n_kv_heads=int(md.get(f"{arch}.attention.head_count_kv", n_heads)),
                           head_dim=dim // n_heads, ffn=int(md[f"{arch}.feed_forward_length"]),
                           vocab=gg.tensors["token_embd.weight"].rows,
                           eps=_f32_short(md.get(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5)),
                           theta=float(md.get(f"{arch}.rope.freq_base", 10000.0)))
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        types = {gg.tensors[n].type for n in gg.tensors if n.endswith(".weight") and "norm" not in n
                 and n != "token_embd.weight"}
        if types - {G.GGML_Q4_0, G.GGML_Q8_0} or len(types) != 1:
            raise ValueError(f"{path}: linear weights must all be Q4_0 or all Q8_0 (types {sorted(types)})")
        fmt = FMT_Q4_0 if types == {G.GGML_Q4_0} else FMT_Q8_0

        def up(name):
            return G.upload(gg, name, dev)

        def vec(name):
            return torch.from_numpy(gg.array(name).reshape(-1).copy()).to(dev)

        layers = []
        for i in range(shape.n_layers):
            q, k, v = up(f"blk.{i}.attn_q.weight"), up(f"blk.{i}.attn_k.weight"), up(f"blk.{i}.attn_v.weight")
            g, u = up(f"blk.{i}.ffn_gate.weight"), up(f"blk.{i}.ffn_up.weight")
            layers.append({
                "wqkv": (torch.cat([q[0], k[0], v[0]]).contiguous(), torch.cat([q[1], k[1], v[1]]).contiguous()),
                "wo": up(f"blk.{i}.attn_output.weight"),
                "wgu": (torch.stack([g[0], u[0]], 1).reshape(2 * shape.ffn, *g[0].shape[1:]).contiguous(),
                        torch.stack([g[1], u[1]], 1).reshape(2 * shape.ffn, g[1].shape[1]).contiguous()),
                "wdown": up(f"blk.{i}.ffn_down.weight"),
                "attn_norm": vec(f"blk.{i}.attn_norm.weight"), "ffn_norm": vec(f"blk.{i}.ffn_norm.weight"),
            })
        et = gg.tensors["token_embd.weight"]
        if et.type in (G.GGML_F32, G.GGML_F16):
            embed = torch.from_numpy(gg.array("token_embd.weight")).to(dev)
        else:  # dequantize the table once on the device: (q - 8 | q) * d
            eq, ed = up("token_embd.weight")
            vals = eq.float() if et.type == G.GGML_Q8_0 else torch.cat([(eq & 0x0F), (eq >> 4)], -1).float() - 8.0
            embed = (vals * ed.float().unsqueeze(-1)).reshape(et.rows, et.cols).contiguous()
        W = {"layers": layers, "final_norm": vec("output_norm.weight"), "lm_head": up("output.weight"),
             "embed": embed}
        return cls(shape, ctx=ctx, max_tokens=max_tokens, fmt=fmt, device=dev, weights=W)

    def to_gguf(self, path) -> None:
        """Writes this model (tp = 1) as a GGUF file that from_gguf reads back."""
        from . import gguf as G

        if self.tp != 1:
            raise ValueError("to_gguf needs the whole model (tp = 1)")
        s = self.shape
        gt = G.GGML_Q4_0 if self.fmt == FMT_Q4_0 else G.GGML_Q8_0
        qd, kvd = s.n_heads * s.head_dim, s.n_kv_heads * s.head_dim
        tensors = []

        def lin(name, qs, sc):
            qs, sc = qs.cpu().numpy(), sc.float().cpu().numpy()
            tensors.append((name, (qs.shape[1] * 32, qs.shape[0]), gt, G.blocks_from_planes(qs, sc)))

        def f32(name, t):
            a = t.float().cpu().numpy()
            tensors.append((name, tuple(reversed(a.shape)), G.GGML_F32, a.tobytes()))

        f32("token_embd.weight", self.embed)
        for i, L in enumerate(self.layers):
            q, sc = L["wqkv"]
            lin(f"blk.{i}.attn_q.weight", q[:qd], sc[:qd])
            lin(f"blk.{i}.attn_k.weight", q[qd:qd + kvd], sc[qd:qd + kvd])
            lin(f"blk.{i}.attn_v.weight", q[qd + kvd:], sc[qd + kvd:])
            lin(f"blk.{i}.attn_output.weight", *L["wo"])
            gq, gs = L["wgu"]
            lin(f"blk.{i}.ffn_gate.weight", gq[0::2], gs[0::2])
            lin(f"blk.{i}.ffn_up.weight", gq[1::2], gs[1::2])
            lin(f"blk.{i}.ffn_down.weight", *L["wdown"])
            f32(f"blk.{i}.attn_norm.weight", L["attn_norm"])
            f32(f"blk.{i}.ffn_norm.weight", L["ffn_norm"])
        f32("output_norm.weight", self.final_norm)
        lin("output.weight", *self.lm_head)
        md = {"general.architecture": "llama", "llama.embedding_length": s.dim, "llama.block_count": s.n_layers,
              "llama.feed_forward_length": s.ffn, "llama.attention.head_count": s.n_heads,
              "llama.attention.head_count_kv": s.n_kv_heads, "llama.attention.layer_norm_rms_epsilon": float(s.eps),
              "llama.rope.freq_base": float(s.theta), "llama.context_length": self.ctx}
        G.write_gguf(path, md, tensors)

    def close(self):
        if self._handle is not None:
            native.lib().asm_decode_destroy(self._handle)
            self._handle = None
        self._graphs = {}
        if self._xchg_own is not None:
            self.torch.cuda.synchronize()
            for p in self._xchg_peers:
                native.lib().asm_ipc_close(p)
            native.lib().asm_ipc_free(self._xchg_own)
            self._xchg_peers, self._xchg_own = [], None
        for L in self.layers:
            for k in ("wqkv", "wo", "wgu", "wdown"):
                ops.unmark_static(*L[k])
        ops.unmark_static(*self.lm_head)
        self._graphs = {}


__all__ = ["LlamaShape", "LLAMA_7B", "LLAMA2_70B", "LlamaDecoder", "Shard", "shard_plan", "rope_table",
           "FMT_Q4_0", "FMT_Q8_0"]
