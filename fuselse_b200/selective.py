"""Fused selective log-softmax: per-token log-probabilities of chosen tokens.

`selective_log_softmax(logits, index)` returns, for logits (..., V) and integer
targets (...), `logits[..., index] - logsumexp(logits, -1)` — the value that
`trl.trainer.utils.selective_log_softmax` (trl 1.0.0) computes for the RLHF
experiment of the reference (experiment_rlhf_logsumexp/run_rlhf.py:145-157,
where torch.logsumexp is routed to onepass_lse_float by rlhf_timing.py:23-37).
trl makes two passes over the logits — a gather of the target logit and one
log-sum-exp call per sequence — and for 16-bit inputs a full log_softmax per
sequence; here one kernel pass per row produces the target's log-probability
and the row's LSE together, and the backward is one fused pass
`g * (onehot(index) - softmax(x))`.

Inputs that are not CUDA fp32/fp16 are delegated to a torch restatement of
trl's published algorithm (API behaviour, as the reference autograd wrapper
delegates to torch.logsumexp); fp16 logits that require grad are delegated
too (the fused backward is fp32).
"""
from __future__ import annotations

import torch

from . import ext


def torch_selective_log_softmax(logits: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """trl's algorithm restated with torch ops: for fp32/fp64 the gathered logit
    minus a log-sum-exp taken one sequence (leading index) at a time; for other
    dtypes a log_softmax per sequence, then the gather, in the input dtype."""
    if logits.dtype in (torch.float32, torch.float64):
        picked = torch.gather(logits, -1, index.unsqueeze(-1)).squeeze(-1)
        lse = torch.stack([torch.logsumexp(seq, dim=-1) for seq in logits])
        return picked - lse
    out = []
    for seq, seq_index in zip(logits, index):
        logp = torch.log_softmax(seq, dim=-1)
        out.append(torch.gather(logp, -1, seq_index.unsqueeze(-1)).squeeze(-1))
    return torch.stack(out)


class SelectiveLogSoftmax(torch.autograd.Function):
    """(R, V) fp32 rows and (R,) int64 targets -> (R,) log-probabilities."""

    @staticmethod
    def forward(ctx, rows, targets, robust, err_flag):
        logp, lse = ext.selective_logsoftmax_rows(rows, targets, robust=robust, err_flag=err_flag)
        ctx.save_for_backward(rows, lse, targets)
        return logp

    @staticmethod
    def backward(ctx, grad_output):
        rows, lse, targets = ctx.saved_tensors
        grad = ext.selective_logsoftmax_backward(grad_output.contiguous(), rows, lse, targets)
        return grad, None, None, None


class SelectiveLogSoftmaxStrided(torch.autograd.Function):
    """fp32 logits (..., V) whose rows are read in place (e.g. logits[:, :-1, :])."""

    @staticmethod
    def forward(ctx, logits, targets, robust, err_flag):
        logp, lse = ext.selective_logsoftmax_strided(logits, targets, robust=robust, err_flag=err_flag)
        ctx.save_for_backward(logits, lse, targets)
        return logp

    @staticmethod
    def backward(ctx, grad_output):
        logits, lse, targets = ctx.saved_tensors
        grad = ext.selective_logsoftmax_backward_strided(grad_output, logits, lse, targets)
        return grad, None, None, None


def selective_log_softmax(logits: torch.Tensor, index: torch.Tensor, robust: bool = True,
                          check_index: bool = False) -> torch.Tensor:
    """Log-probabilities of `index` under softmax(logits, -1), shape index.shape.

    fp32 logits give fp32 results (autograd-capable); fp16 logits give fp16
    results, computed in fp32.  A target outside [0, V) yields NaN; with
    `check_index=True` it raises RuntimeError instead (one device sync)."""
    supported = (logits.is_cuda and logits.dtype in (torch.float32, torch.float16)
                 and logits.dim() >= 1 and tuple(index.shape) == tuple(logits.shape[:-1])
                 and logits.shape[-1] >= 1 and index.device == logits.device
                 and not (logits.dtype == torch.float16 and torch.is_grad_enabled()
                          and logits.requires_grad))
    if not supported:
        return torch_selective_log_softmax(logits, index)
    V = logits.shape[-1]
    targets = index.reshape(-1).to(torch.int64).contiguous()
    err = torch.zeros(1, dtype=torch.int32, device=logits.device) if check_index else None
    grad = torch.is_grad_enabled() and logits.requires_grad
    if (logits.dtype == torch.float32 and not logits.is_contiguous()
            and ext.row_layout(logits) is not None):
        # strided rows (a slice such as logits[:, :-1, :]): read in place, no copy
        if grad:
            logp = SelectiveLogSoftmaxStrided.apply(logits, targets, robust, err)
        else:
            logp, _ = ext.selective_logsoftmax_strided(logits, targets, robust=robust, err_flag=err)
        if check_index and int(err.item()):
            raise RuntimeError(f"selective_log_softmax: index out of range for {V} classes")
        return logp.reshape(index.shape)
    rows = logits.reshape(-1, V).contiguous()
    if logits.dtype == torch.float32 and grad:
        logp = SelectiveLogSoftmax.apply(rows, targets, robust, err)
    else:
        logp, _ = ext.selective_logsoftmax_rows(rows, targets, robust=robust, err_flag=err)
    if check_index and int(err.item()):
        raise RuntimeError(f"selective_log_softmax: index out of range for {V} classes")
    return logp.reshape(index.shape).to(logits.dtype)
