"""Multi-GPU partitioning of the row log-sum-exp path (one process per GPU).

Two layouts (the reference itself is single-GPU; both are additions):

* Batch rows (FuseLSE fwd/bwd, IntLSE, sparse over batch columns): rows are
  independent, so each rank owns a contiguous block of rows and runs the
  single-GPU kernels on it.  No collective is on the data path; results stay
  on their rank unless the caller gathers them.

* Vocab shards (LLM logits split along N across ranks): each rank reduces its
  columns to per-row partial states (m, s) = (max, sum exp(x - m)), the ranks
  exchange the 8-byte states of every row, and each rank combines the G states
  of a row locally:  lse = M + log(sum_g s_g exp(m_g - M)).  Two exchanges:
  VocabShardExchange (the product path) has the partial kernel store the pairs
  straight into every rank's buffer over NVLink, then a combine kernel
  publishes this rank's delivery (a system-scope release of the call's epoch
  into every rank's flag word) and waits for all ranks; vocab_sharded_logsumexp
  does the same with ext.lse_partial, an NCCL all-gather and ext.lse_combine
  (the baseline, and the path for groups without peer memory).
  Every rank ends with the full (B,) result.  The association differs from a
  single-GPU pass, so results agree to rounding, not bit for bit.
  The backward needs no exchange: with the combined lse on every rank, each
  rank's shard gradient is g * exp(x_shard - lse), the single-GPU backward
  kernel on its own columns (VocabShardedLogSumExp).

The local compute functions are injectable so the exchange logic can be
exercised on CPU ranks over gloo.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def split_range(n: int, parts: int, index: int) -> tuple[int, int]:
    """Contiguous [lo, hi) block `index` of `parts` over n items; the first
    n % parts blocks get one extra item."""
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError(f"bad split: parts={parts} index={index}")
    base, extra = divmod(n, parts)
    lo = index * base + min(index, extra)
    return lo, lo + base + (1 if index < extra else 0)


def local_rows(n_rows: int, group=None) -> tuple[int, int]:
    """This rank's row block under batch-row sharding."""
    return split_range(n_rows, dist.get_world_size(group), dist.get_rank(group))


def local_columns(n_cols: int, group=None) -> tuple[int, int]:
    """This rank's column block under vocab sharding."""
    return split_range(n_cols, dist.get_world_size(group), dist.get_rank(group))


def gather_partials(ms: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather (B, 2) partial states into (G, B, 2), rank-major."""
    G = dist.get_world_size(group)
    out = torch.empty((G, *ms.shape), dtype=ms.dtype, device=ms.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, ms.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), ms.contiguous(), group=group)
    return out


def vocab_sharded_logsumexp(x_shard: torch.Tensor, group=None,
                            partial_fn: Optional[Callable] = None,
                            combine_fn: Optional[Callable] = None) -> torch.Tensor:
    """log-sum-exp over rows whose columns are split across the ranks of `group`.

    x_shard: this rank's (B, N_g) columns (fp32 or fp16, contiguous).  Every
    rank must pass the same B.  Returns the (B,) fp32 result on every rank.
    """
    if partial_fn is None or combine_fn is None:
        from . import ext
        partial_fn = partial_fn or ext.lse_partial
        combine_fn = combine_fn or ext.lse_combine
    ms = partial_fn(x_shard)
    if ms.dim() != 2 or ms.size(1) != 2:
        raise RuntimeError("partial state must be (B, 2)")
    return combine_fn(gather_partials(ms, group))


class VocabShardedLogSumExp(torch.autograd.Function):
    """Autograd over a vocab-sharded log-sum-exp.

    forward(x_shard, exchange, backward_fn): lse = exchange(x_shard) — a
    VocabShardExchange, or any callable such as
    `lambda x: vocab_sharded_logsumexp(x, group)` — the full (B,) result on
    every rank.  backward: d lse / d x_shard = exp(x_shard - lse), so this
    rank's gradient is backward_fn(g, x_shard, lse) on its own columns
    (ext.onepass_lse_float_backward by default: fp32 shards).  g must be the
    full gradient of the loss with respect to lse on every rank (a loss
    computed identically on every rank from the replicated lse), not a
    per-rank part of it.
    """

    @staticmethod
    def forward(ctx, x_shard, exchange, backward_fn=None):
        lse = exchange(x_shard)
        ctx.save_for_backward(x_shard, lse)
        ctx.backward_fn = backward_fn
        return lse

    @staticmethod
    def backward(ctx, grad_output):
        x_shard, lse = ctx.saved_tensors
        fn = ctx.backward_fn
        if fn is None:
            from . import ext
            fn = ext.onepass_lse_float_backward
        return fn(grad_output.contiguous(), x_shard, lse), None, None


def vocab_sharded_logsumexp_grad(x_shard: torch.Tensor, exchange: Callable,
                                 backward_fn: Optional[Callable] = None) -> torch.Tensor:
    """Vocab-sharded log-sum-exp whose result carries a gradient to x_shard."""
    return VocabShardedLogSumExp.apply(x_shard, exchange, backward_fn)


class _RawDeviceBytes:
    """A raw device allocation exposed to torch (no ownership) through the CUDA
    array interface, so torch ops can zero it or read its header words."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


class VocabShardExchange:
    """Vocab-sharded log-sum-exp with the (max, sumexp) exchange done by this
    library's own kernels over NVLink peer memory (fl_lse_vocab_exchange): the
    partial kernel stores each row's pair into every rank's exchange buffer;
    a combine kernel publishes this rank's delivery with a system-scope
    release of the call's epoch, waits (bounded) for all ranks and finishes
    the rows.  No NCCL call on the data path.

    Each rank's exchange buffer is its own cudaMalloc allocation
    (fl_ipc_buffer_alloc), shared with the other ranks by CUDA IPC handles
    (exchanged once over the process group) and mapped there with plain peer
    mappings (fl_ipc_buffer_open): unicast peer mappings only, no NVLS group.
    Made once per (group, rows); close() (or garbage collection) unmaps the
    peers' buffers and frees this rank's after a barrier.  Every rank must
    call with the same B, in the same sequence.
    """

    def __init__(self, rows: int, group=None, device=None):
        import ctypes

        from . import _lib
        self.group = group if group is not None else dist.group.WORLD
        self.G = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.rows = rows
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        dev = self.device.index
        nbytes = ctypes.c_int64()
        _lib.call("fl_vocab_exchange_bytes", self.G, rows, ctypes.byref(nbytes))
        self.nbytes = nbytes.value
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        _lib.call("fl_ipc_buffer_alloc", dev, self.nbytes, ctypes.byref(ptr), handle)
        self._own = ptr.value
        self._opened = []
        handles = [None] * self.G
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        addrs = []
        for q, h in enumerate(handles):
            if q == self.rank:
                addrs.append(self._own)
                continue
            peer = ctypes.c_void_p()
            _lib.call("fl_ipc_buffer_open", dev, (ctypes.c_ubyte * 64).from_buffer_copy(h),
                      ctypes.byref(peer))
            self._opened.append(peer.value)
            addrs.append(peer.value)
        self.buf = torch.as_tensor(_RawDeviceBytes(self._own, self.nbytes), device=self.device)
        self._ptrs = torch.tensor(addrs, dtype=torch.int64, device=self.device)
        self.peer_array = self._ptrs.data_ptr()
        dist.barrier(self.group)  # every rank's buffer is mapped before anyone writes

    @classmethod
    def single_rank(cls, rows: int, device="cuda"):
        """G = 1 exchange on one GPU, without a process group (tests, 1-GPU runs)."""
        import ctypes

        from . import _lib
        self = cls.__new__(cls)
        self.group, self.G, self.rank, self.rows = None, 1, 0, rows
        self._own, self._opened = None, []
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        nbytes = ctypes.c_int64()
        _lib.call("fl_vocab_exchange_bytes", 1, rows, ctypes.byref(nbytes))
        self.nbytes = nbytes.value
        self.buf = torch.zeros(nbytes.value, dtype=torch.uint8, device=self.device)
        self._ptrs = torch.tensor([self.buf.data_ptr()], dtype=torch.int64, device=self.device)
        self.peer_array = self._ptrs.data_ptr()
        return self

    def close(self, barrier: bool = True) -> None:
        """Unmaps the peers' buffers and frees this rank's.  With barrier=True
        (every rank calls close) no rank frees its buffer while another still
        has it mapped."""
        from . import _lib
        if not getattr(self, "_own", None):
            return
        torch.cuda.synchronize(self.device)
        dev = self.device.index
        for p in self._opened:
            _lib.call("fl_ipc_buffer_close", dev, p)
        self._opened = []
        if barrier and self.group is not None:
            dist.barrier(self.group)
        self.buf = None
        _lib.call("fl_ipc_buffer_free", dev, self._own)
        self._own = None

    def __del__(self):
        try:
            self.close(barrier=False)
        except Exception:
            pass

    def __call__(self, x_shard: torch.Tensor) -> torch.Tensor:
        import ctypes

        from . import _lib
        if getattr(self, "buf", None) is None:
            raise RuntimeError("this exchange was closed")
        if x_shard.dim() != 2 or x_shard.size(0) != self.rows:
            raise RuntimeError(f"expected a ({self.rows}, N) shard, got {tuple(x_shard.shape)}")
        if not (x_shard.is_cuda and x_shard.device == self.device and x_shard.is_contiguous()):
            raise RuntimeError(f"shard must be contiguous on {self.device}")
        if x_shard.dtype not in (torch.float32, torch.float16):
            raise RuntimeError("shard must be fp32 or fp16")
        out = torch.empty(self.rows, dtype=torch.float32, device=self.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        _lib.call("fl_lse_vocab_exchange", ctypes.c_void_p(x_shard.data_ptr()),
                  0 if x_shard.dtype == torch.float32 else 1, self.rows, x_shard.size(1),
                  ctypes.c_void_p(self.peer_array), ctypes.c_void_p(self.buf.data_ptr()),
                  self.rank, self.G, _lib.ptr(out), stream)
        return out

    def error(self) -> bool:
        """True once a combine gave up waiting for a peer (sticky)."""
        if getattr(self, "buf", None) is None:
            raise RuntimeError("this exchange was closed")
        return bool(self.buf[4:8].view(torch.int32).item())


def batch_sharded_logsumexp(x_local: torch.Tensor, robust: bool = True,
                            gather: bool = False, group=None,
                            lse_fn: Optional[Callable] = None) -> torch.Tensor:
    """Row log-sum-exp of this rank's rows; with gather=True, the (B_total,)
    result on every rank (rows may differ in count across ranks)."""
    if lse_fn is None:
        from . import ext
        lse_fn = ext.onepass_lse_float_robust if robust else ext.onepass_lse_float
    out = lse_fn(x_local)
    if not gather:
        return out
    G = dist.get_world_size(group)
    counts = torch.tensor([out.numel()], dtype=torch.int64, device=out.device)
    all_counts = [torch.zeros_like(counts) for _ in range(G)]
    dist.all_gather(all_counts, counts, group=group)
    n = [int(c.item()) for c in all_counts]
    width = max(n) if n else 0
    padded = torch.zeros(width, dtype=out.dtype, device=out.device)
    padded[: out.numel()] = out
    pieces = [torch.empty_like(padded) for _ in range(G)]
    dist.all_gather(pieces, padded, group=group)
    return torch.cat([p[:k] for p, k in zip(pieces, n)])
