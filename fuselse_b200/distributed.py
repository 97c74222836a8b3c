"""Multi-GPU partitioning of the row log-sum-exp path (one process per GPU).

Two layouts (the reference itself is single-GPU; both are additions):

* Batch rows (FuseLSE fwd/bwd, IntLSE, sparse over batch columns): rows are
  independent, so each rank owns a contiguous block of rows and runs the
  single-GPU kernels on it.  No collective is on the data path; results stay
  on their rank unless the caller gathers them.

* Vocab shards (LLM logits split along N across ranks): each rank reduces its
  columns to per-row partial states (m, s) = (max, sum exp(x - m)) with
  ext.lse_partial, the ranks exchange the 8-byte states of every row with one
  all-gather (NCCL over NVLink), and each rank combines the G states of a row
  locally (ext.lse_combine):  lse = M + log(sum_g s_g exp(m_g - M)).
  Every rank ends with the full (B,) result.  The association differs from a
  single-GPU pass, so results agree to rounding, not bit for bit.

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
