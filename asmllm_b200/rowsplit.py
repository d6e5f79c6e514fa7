"""Row-split (sharded) matvec over a tensor-parallel group, one process per GPU.

The reference parallelises a matvec by splitting its output rows among the
threads of its pool: ``asm_threadpool_dispatch_q4`` hands worker t a
contiguous row range and every worker writes its rows into the one shared y
(src/runtime/threadpool.c:408-486; ``asm_matmul_q4_mt`` at :390-486).  Across
GPUs the same split is: rank r holds rows ``[r*M, (r+1)*M)`` of a
``(tp*M) x K`` matrix, computes them, and the full y is all-gathered.  The
gather rides on the matvec kernel (``asm_matvec_rowsplit_async``): each
finished row goes into this rank's ``y_full`` and, as a (sequence, value)
word, into every other rank's gather buffer by NVLink peer stores;
``asm_rowsplit_wait_async`` completes a step (one bounded wait per word).

Host logic here (shard ranges, the exchange of IPC handles) is plain Python
over ``torch.distributed`` and is tested with gloo ranks on the CPU.
"""
from __future__ import annotations

import ctypes

from . import native
from .ops import MV_INDEPENDENT, MV_PACKED, _check_dev, _ptr, _stream_handle, _torch


def shard_range(m_total: int, tp: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of rank `rank` when m_total rows are split evenly over
    tp ranks (the C ABI's equal shards: m_total must be a multiple of tp)."""
    if tp < 1 or not 0 <= rank < tp:
        raise ValueError(f"rank {rank} of tp {tp}")
    if m_total % tp:
        raise ValueError(f"{m_total} rows do not split evenly over {tp} ranks")
    m = m_total // tp
    return rank * m, (rank + 1) * m


def exchange_handles(own: bytes, group=None) -> list[bytes]:
    """Every rank's handle in rank order (all_gather_object over `group`)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = [None] * world
    dist.all_gather_object(out, own, group=group)
    return out


def gather_buffer_bytes(m: int, tp: int) -> int:
    """Bytes of one matvec's gather buffer: 2 parities x tp source ranks x m rows of 64-bit words."""
    return 2 * tp * m * 8


class RowSplitGroup:
    """Gather buffers and step counter of `n` row-split matvecs per step.

    ``rows[j]`` = rows per rank of matvec j.  With tp = 1 the matvecs are
    plain (no buffers, no wait)."""

    def __init__(self, rows: list[int], tp: int, rank: int, group=None, device=None):
        torch = _torch()
        if not 1 <= len(rows) <= 8:
            raise ValueError("1 to 8 matvecs per step")
        self.rows, self.tp, self.rank = list(rows), tp, rank
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.seq = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._own, self._peers = [], []
        self._bufs = []  # per matvec: [tp] device addresses (own buffer at index rank)
        L = native.lib()
        for m in self.rows:
            addrs = [0] * tp
            if tp > 1:
                ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
                native.check(L.asm_ipc_alloc(gather_buffer_bytes(m, tp), ctypes.byref(ptr), handle))
                self._own.append(ptr)
                for r, hr in enumerate(exchange_handles(handle.raw, group)):
                    if r == rank:
                        addrs[r] = ptr.value
                        continue
                    peer = ctypes.c_void_p()
                    native.check(L.asm_ipc_open(hr, ctypes.byref(peer)))
                    self._peers.append(peer)
                    addrs[r] = peer.value
            self._bufs.append((ctypes.c_void_p * 8)(*addrs, *([0] * (8 - tp))))
        if tp > 1:
            import torch.distributed as dist

            dist.barrier(group=group)
        self._wait = native.RowsplitWait()
        self._wait.n, self._wait.tp, self._wait.rank = len(self.rows), tp, rank
        for j, m in enumerate(self.rows):
            self._wait.own[j] = self._bufs[j][rank] or None
            self._wait.M[j] = m
        self._wait.seq, self._wait.done = self.seq.data_ptr(), self.done.data_ptr()

    def matvec(self, j: int, fmt: int, w, x, y_full, scales=None, *, independent=False, stream=None):
        """Rows of matvec j on this rank into y_full[rank*M:(rank+1)*M] and to every peer.
        w: packed rows (uint8 [M, row bytes]) when scales is None, else the quant plane
        with fp16 scales [M, K/32]."""
        torch = _torch()
        m = self.rows[j]
        _check_dev(x, (torch.float32,), "x")
        _check_dev(y_full, (torch.float32,), "y_full")
        if y_full.numel() != self.tp * m:
            raise ValueError(f"y_full holds {y_full.numel()} values, not tp * M = {self.tp * m}")
        flags = (MV_INDEPENDENT if independent else 0) | (MV_PACKED if scales is None else 0)
        self._wait.y_full[j] = y_full.data_ptr()
        native.check(native.lib().asm_matvec_rowsplit_async(
            fmt, _ptr(w), None if scales is None else _ptr(scales), _ptr(x), _ptr(y_full), m, x.shape[-1],
            self.tp, self.rank, self._bufs[j], _ptr(self.seq), flags, _stream_handle(stream)))

    def wait(self, stream=None):
        """Completes the step: every matvec's full y_full on this rank (the y_full
        tensors are the ones given to the step's matvec calls)."""
        native.check(native.lib().asm_rowsplit_wait_async(ctypes.byref(self._wait), _stream_handle(stream)))

    def close(self):
        L = native.lib()
        for p in self._peers:
            L.asm_ipc_close(p)
        for p in self._own:
            L.asm_ipc_free(p)
        self._peers, self._own = [], []
