"""Torch-facing entry points under the reference extension's method names.

This module stands in for the `ext` object that the reference builds with
`torch.utils.cpp_extension.load(...)` from each of its .cu files, so
`make_fuselse_logsumexp(fuselse_b200.ext, robust)` and the experiment
monkeypatches work unchanged.  Validation mirrors the reference TORCH_CHECKs
(same conditions, RuntimeError), outputs are allocated with torch on the
input's device, and kernels run on that device's current stream.

Reference bindings replaced (file:line):
  onepass_lse_float, onepass_lse_float_robust, onepass_lse_float_backward
      fuselse/gpu/fused_fp32_kernel.cu:154-261
  batched_logsumexp_fp16            fuselse/gpu/fused_fp16_kernel.cu:112-137
  batched_logsumexp, batched_logsumexp_nolut
                                    intlse/gpu/lse_kernel.cu:186-209
  batched_logsumexp_q10_6           intlse/gpu/lse_kernel_q10_6.cu:144-170
  sparse_forward_float              experiment_pyjuice/sparse_float_kernel.cu:110-172
  sparse_forward_q16                experiment_pyjuice/sparse_q16_kernel.cu:139-207
Additions without a reference counterpart: batched_logsumexp_q16_i32,
lse_partial, lse_combine, sparse_log_weights, sparse_parent_index,
sparse_backward_float, selective_logsoftmax_* (fused target gather + LSE),
row_layout / *_strided (rows read in place) and logsumexp_dim* (dim != -1).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import call, ptr


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


# --------------------------------------------------------------------------
# FuseLSE fp32 (fused_fp32_kernel.cu)
# --------------------------------------------------------------------------
def _check_f32_2d(x: torch.Tensor) -> None:
    _check(x.is_cuda, "x must be CUDA")
    _check(x.dtype == torch.float32, "x must be float32")
    _check(x.dim() == 2, "x must be 2D (B, N)")
    _check(x.is_contiguous(), "x must be contiguous")


def _lse_f32(x: torch.Tensor, robust: bool) -> torch.Tensor:
    _check_f32_2d(x)
    B, N = x.shape
    out = torch.empty((B,), dtype=torch.float32, device=x.device)
    if B == 0:
        return out
    call("fl_lse_f32_fwd", ptr(x), ptr(out), B, N, int(robust), _stream(x))
    return out


def onepass_lse_float(x: torch.Tensor) -> torch.Tensor:
    """(B, N) fp32 -> (B,) fp32 log-sum-exp; finite inputs assumed."""
    return _lse_f32(x, robust=False)


def onepass_lse_float_robust(x: torch.Tensor) -> torch.Tensor:
    """(B, N) fp32 -> (B,) fp32 log-sum-exp with IEEE NaN/Inf rules."""
    return _lse_f32(x, robust=True)


def onepass_lse_float_backward(grad_output: torch.Tensor, x: torch.Tensor,
                               lse_output: torch.Tensor) -> torch.Tensor:
    """grad_input = grad_output[:, None] * exp(x - lse_output[:, None])."""
    _check(grad_output.is_cuda, "grad_output must be CUDA")
    _check(x.is_cuda, "x must be CUDA")
    _check(lse_output.is_cuda, "lse_output must be CUDA")
    _check(x.dtype == torch.float32, "x must be float32")
    _check(grad_output.dtype == torch.float32, "grad_output must be float32")
    _check(lse_output.dtype == torch.float32, "lse_output must be float32")
    _check(x.dim() == 2, "x must be 2D (B, N)")
    _check(grad_output.dim() == 1, "grad_output must be 1D (B)")
    _check(lse_output.dim() == 1, "lse_output must be 1D (B)")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(grad_output.is_contiguous(), "grad_output must be contiguous")
    _check(lse_output.is_contiguous(), "lse_output must be contiguous")
    _check(grad_output.size(0) == x.size(0), "grad_output batch dimension must match x")
    _check(lse_output.size(0) == x.size(0), "lse_output batch dimension must match x")
    _check(grad_output.device == x.device and lse_output.device == x.device,
           "grad_output, x and lse_output must be on the same device")
    B, N = x.shape
    grad_input = torch.empty_like(x)
    if B * N == 0:
        return grad_input
    call("fl_lse_f32_bwd", ptr(grad_output), ptr(x), ptr(lse_output), ptr(grad_input), B, N,
         _stream(x))
    return grad_input


# --------------------------------------------------------------------------
# FuseLSE16 (fused_fp16_kernel.cu)
# --------------------------------------------------------------------------
def batched_logsumexp_fp16(input: torch.Tensor) -> torch.Tensor:
    """(B, N) fp16 -> (B,) fp32 log-sum-exp, fp32 arithmetic."""
    _check(input.dim() == 2, "Expected 2-D tensor (B, N)")
    _check(input.is_cuda and input.dtype == torch.float16, "Input must be CUDA fp16")
    _check(input.is_contiguous(), "Input must be contiguous")
    B, N = input.shape
    out = torch.empty((B,), dtype=torch.float32, device=input.device)
    if B == 0:
        return out
    call("fl_lse_f16_fwd", ptr(input, ctypes.c_uint16), ptr(out), B, N, _stream(input))
    return out


# --------------------------------------------------------------------------
# Selective log-softmax (fused gather + LSE; no reference kernel)
# --------------------------------------------------------------------------
def selective_logsoftmax_rows(x: torch.Tensor, index: torch.Tensor, robust: bool = True,
                              err_flag: torch.Tensor | None = None):
    """(B, N) fp32/fp16 logits and (B,) int64 targets -> (logp, lse), both (B,) fp32,
    logp[b] = x[b, index[b]] - lse[b], in one pass over each row.

    An index outside [0, N) gives logp = NaN and, with `err_flag` (a zeroed int32
    CUDA tensor of one element), sets it to 1; nothing is raised asynchronously.
    fp16 rows use the FuseLSE16 rules (robust is ignored)."""
    _check(x.dim() == 2, "x must be 2D (B, N)")
    _check(x.is_cuda and x.dtype in (torch.float32, torch.float16), "x must be CUDA fp32 or fp16")
    _check(x.is_contiguous(), "x must be contiguous")
    _check(index.is_cuda and index.dtype == torch.int64, "index must be CUDA int64")
    _check(index.dim() == 1 and index.size(0) == x.size(0), "index must be 1D (B) matching x")
    _check(index.is_contiguous(), "index must be contiguous")
    _check(index.device == x.device, "x and index must be on the same device")
    if err_flag is not None:
        _check(err_flag.is_cuda and err_flag.dtype == torch.int32 and err_flag.numel() >= 1,
               "err_flag must be a CUDA int32 tensor")
        _check(err_flag.device == x.device, "err_flag must be on x's device")
    B, N = x.shape
    _check(B == 0 or N > 0, "x has no columns to select from")
    logp = torch.empty((B,), dtype=torch.float32, device=x.device)
    lse = torch.empty((B,), dtype=torch.float32, device=x.device)
    if B == 0:
        return logp, lse
    err = ptr(err_flag, ctypes.c_int) if err_flag is not None else None
    if x.dtype == torch.float32:
        call("fl_selective_logsoftmax_f32", ptr(x), ptr(index, ctypes.c_int64), ptr(logp), ptr(lse),
             B, N, int(robust), err, _stream(x))
    else:
        call("fl_selective_logsoftmax_f16", ptr(x, ctypes.c_uint16), ptr(index, ctypes.c_int64),
             ptr(logp), ptr(lse), B, N, err, _stream(x))
    return logp, lse


def selective_logsoftmax_backward(grad_output: torch.Tensor, x: torch.Tensor, lse: torch.Tensor,
                                  index: torch.Tensor) -> torch.Tensor:
    """grad_input[b, j] = grad_output[b] * ([j == index[b]] - exp(x[b, j] - lse[b])), fp32."""
    _check(x.is_cuda and x.dtype == torch.float32 and x.dim() == 2 and x.is_contiguous(),
           "x must be a contiguous 2D CUDA float32 tensor")
    for t, name in ((grad_output, "grad_output"), (lse, "lse")):
        _check(t.is_cuda and t.dtype == torch.float32 and t.dim() == 1 and t.is_contiguous(),
               f"{name} must be a contiguous 1D CUDA float32 tensor")
        _check(t.size(0) == x.size(0), f"{name} batch dimension must match x")
        _check(t.device == x.device, f"{name} must be on x's device")
    _check(index.is_cuda and index.dtype == torch.int64 and index.dim() == 1 and index.is_contiguous()
           and index.size(0) == x.size(0) and index.device == x.device,
           "index must be a contiguous 1D CUDA int64 tensor matching x")
    B, N = x.shape
    grad_input = torch.empty_like(x)
    if B * N == 0:
        return grad_input
    call("fl_selective_logsoftmax_bwd", ptr(grad_output), ptr(x), ptr(lse),
         ptr(index, ctypes.c_int64), ptr(grad_input), B, N, _stream(x))
    return grad_input


# --------------------------------------------------------------------------
# In-place layouts: strided rows and dim != -1 (no contiguous copy)
# --------------------------------------------------------------------------
def row_layout(x: torch.Tensor):
    """(B, N, rows_per_group, group_stride, row_stride) when the rows of x
    (its last dim, unit stride) can be addressed where they lie: the leading
    dims, after merging the ones that nest densely, form at most two levels.
    None otherwise (the caller copies)."""
    if x.dim() == 0:
        return None
    N = x.size(-1)
    if N > 1 and x.stride(-1) != 1:
        return None
    B = 1
    levels: list[list[int]] = []  # [size, stride], outer to inner
    for size, stride in zip(x.shape[:-1], x.stride()[:-1]):
        B *= size
        if size == 1:
            continue
        if levels and levels[-1][1] == stride * size:
            levels[-1] = [levels[-1][0] * size, stride]
        else:
            levels.append([size, stride])
    if not levels:
        return (B, N, -1, 0, N)
    if len(levels) == 1:
        return (B, N, levels[0][0], 0, levels[0][1])
    if len(levels) == 2:
        return (B, N, levels[1][0], levels[0][1], levels[1][1])
    return None


def _strided_rows(x: torch.Tensor):
    _check(x.is_cuda and x.dtype == torch.float32, "x must be CUDA float32")
    lay = row_layout(x)
    _check(lay is not None, "x rows cannot be addressed in place (more than two leading stride levels)")
    return lay


def onepass_lse_float_strided(x: torch.Tensor, robust: bool = True) -> torch.Tensor:
    """Log-sum-exp over the last dim of a strided fp32 tensor (..., N) read in
    place, e.g. logits[:, :-1, :]; result shape x.shape[:-1]."""
    B, N, rpg, gs, rs = _strided_rows(x)
    out = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    if B == 0:
        return out
    call("fl_lse_f32_fwd_strided", ptr(x), ptr(out), B, N, rpg, gs, rs, int(robust), _stream(x))
    return out


def onepass_lse_float_backward_strided(grad_output: torch.Tensor, x: torch.Tensor,
                                       lse: torch.Tensor) -> torch.Tensor:
    """Dense grad_input of x's shape = grad_output[..., None] * exp(x - lse[..., None]), x read in place."""
    B, N, rpg, gs, rs = _strided_rows(x)
    g = grad_output.reshape(-1).contiguous()
    lse = lse.reshape(-1).contiguous()
    _check(g.numel() == B and lse.numel() == B, "grad_output / lse must have x.shape[:-1]")
    _check(g.dtype == torch.float32 and lse.dtype == torch.float32 and g.device == x.device
           and lse.device == x.device, "grad_output and lse must be CUDA float32 on x's device")
    grad_input = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    if B * N == 0:
        return grad_input
    call("fl_lse_f32_bwd_strided", ptr(g), ptr(x), ptr(lse), ptr(grad_input), B, N, rpg, gs, rs,
         _stream(x))
    return grad_input


def _dim_view(x: torch.Tensor, dim: int):
    _check(x.is_cuda and x.dtype == torch.float32, "x must be CUDA float32")
    _check(x.is_contiguous(), "x must be contiguous")
    d = dim if dim >= 0 else dim + x.dim()
    _check(0 <= d < x.dim(), f"dim {dim} out of range for {x.dim()}-D input")
    outer = 1
    for s in x.shape[:d]:
        outer *= s
    inner = 1
    for s in x.shape[d + 1:]:
        inner *= s
    return d, outer, x.size(d), inner


def logsumexp_dim(x: torch.Tensor, dim: int, robust: bool = True) -> torch.Tensor:
    """Log-sum-exp of a contiguous fp32 tensor over any dim, read in place."""
    d, outer, N, inner = _dim_view(x, dim)
    out = torch.empty(x.shape[:d] + x.shape[d + 1:], dtype=torch.float32, device=x.device)
    if outer * inner == 0:
        return out
    call("fl_lse_f32_fwd_dim", ptr(x), ptr(out), outer, N, inner, int(robust), _stream(x))
    return out


def logsumexp_dim_backward(grad_output: torch.Tensor, x: torch.Tensor, lse: torch.Tensor,
                           dim: int) -> torch.Tensor:
    """grad_input = grad_output * exp(x - lse), broadcast over `dim`."""
    d, outer, N, inner = _dim_view(x, dim)
    g = grad_output.contiguous()
    lse = lse.contiguous()
    _check(g.numel() == outer * inner and lse.numel() == outer * inner,
           "grad_output / lse must have x's shape without dim")
    _check(g.dtype == torch.float32 and lse.dtype == torch.float32 and g.device == x.device
           and lse.device == x.device, "grad_output and lse must be CUDA float32 on x's device")
    grad_input = torch.empty_like(x)
    if x.numel() == 0:
        return grad_input
    call("fl_lse_f32_bwd_dim", ptr(g), ptr(x), ptr(lse), ptr(grad_input), outer, N, inner,
         _stream(x))
    return grad_input


def selective_logsoftmax_strided(x: torch.Tensor, index: torch.Tensor, robust: bool = True,
                                 err_flag: torch.Tensor | None = None):
    """selective_logsoftmax_rows for fp32 logits (..., N) whose rows are read in
    place (e.g. logits[:, :-1, :]); index has x.shape[:-1]; returns (logp, lse)
    flattened to (B,)."""
    B, N, rpg, gs, rs = _strided_rows(x)
    t = index.reshape(-1).to(torch.int64).contiguous()
    _check(t.is_cuda and t.numel() == B and t.device == x.device, "index must have x.shape[:-1] on x's device")
    _check(B == 0 or N > 0, "x has no columns to select from")
    if err_flag is not None:
        _check(err_flag.is_cuda and err_flag.dtype == torch.int32 and err_flag.device == x.device,
               "err_flag must be a CUDA int32 tensor on x's device")
    logp = torch.empty((B,), dtype=torch.float32, device=x.device)
    lse = torch.empty((B,), dtype=torch.float32, device=x.device)
    if B == 0:
        return logp, lse
    err = ptr(err_flag, ctypes.c_int) if err_flag is not None else None
    call("fl_selective_logsoftmax_f32_strided", ptr(x), ptr(t, ctypes.c_int64), ptr(logp), ptr(lse),
         B, N, rpg, gs, rs, int(robust), err, _stream(x))
    return logp, lse


def selective_logsoftmax_backward_strided(grad_output: torch.Tensor, x: torch.Tensor,
                                          lse: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """Dense grad_input of x's shape for the strided selective log-softmax."""
    B, N, rpg, gs, rs = _strided_rows(x)
    g = grad_output.reshape(-1).contiguous()
    lse = lse.reshape(-1).contiguous()
    t = index.reshape(-1).to(torch.int64).contiguous()
    _check(g.numel() == B and lse.numel() == B and t.numel() == B,
           "grad_output, lse and index must have x.shape[:-1]")
    _check(g.dtype == torch.float32 and lse.dtype == torch.float32 and g.device == x.device
           and lse.device == x.device and t.device == x.device,
           "grad_output and lse must be CUDA float32 on x's device")
    grad_input = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    if B * N == 0:
        return grad_input
    call("fl_selective_logsoftmax_bwd_strided", ptr(g), ptr(x), ptr(lse), ptr(t, ctypes.c_int64),
         ptr(grad_input), B, N, rpg, gs, rs, _stream(x))
    return grad_input


# --------------------------------------------------------------------------
# IntLSE (lse_kernel.cu, lse_kernel_q10_6.cu)
# --------------------------------------------------------------------------
def _check_intlse_f32(input: torch.Tensor) -> None:
    _check(input.dim() == 2, "Expected 2-D tensor (B, N)")
    _check(input.is_cuda and input.dtype == torch.float32,
           "Expected input.is_cuda() && input.dtype() == torch::kFloat32 to be true, but got false.")
    _check(input.is_contiguous(), "Input must be contiguous")


def _intlse_f32(input: torch.Tensor, use_lut: bool) -> torch.Tensor:
    _check_intlse_f32(input)
    B, N = input.shape
    out = torch.empty((B,), dtype=torch.float32, device=input.device)
    if B == 0:
        return out
    call("fl_intlse_q16_f32", ptr(input), ptr(out), B, N, int(use_lut), _stream(input))
    return out


def batched_logsumexp(input: torch.Tensor) -> torch.Tensor:
    """IntLSE Q16.16: (B, N) fp32 base-e -> (B,) fp32 base-e, bit-identical to the reference."""
    return _intlse_f32(input, use_lut=True)


def batched_logsumexp_nolut(input: torch.Tensor) -> torch.Tensor:
    """IntLSE Q16.16 without the correction table (ablation)."""
    return _intlse_f32(input, use_lut=False)


def batched_logsumexp_q16_i32(input: torch.Tensor, use_lut: bool = True) -> torch.Tensor:
    """IntLSE Q16.16 from int32 fixed-point input (base 2) -> (B,) fp32 base-e."""
    _check(input.dim() == 2, "Expected 2-D tensor (B, N)")
    _check(input.is_cuda, "Input must be CUDA")
    _check(input.dtype == torch.int32, "Input must be int32 (Q16.16 base-2 fixed-point)")
    _check(input.is_contiguous(), "Input must be contiguous")
    B, N = input.shape
    out = torch.empty((B,), dtype=torch.float32, device=input.device)
    if B == 0:
        return out
    call("fl_intlse_q16_i32", ptr(input, ctypes.c_int32), ptr(out), B, N, int(use_lut),
         _stream(input))
    return out


def batched_logsumexp_q10_6(input: torch.Tensor) -> torch.Tensor:
    """IntLSE Q10.6: (B, N) int16 base-2 -> (B,) fp32 base-e, bit-identical to the reference."""
    _check(input.dim() == 2, "Expected 2-D tensor (B, N)")
    _check(input.is_cuda, "Input must be CUDA")
    _check(input.dtype == torch.int16, "Input must be int16 (Q10.6 base-2 fixed-point)")
    _check(input.is_contiguous(), "Input must be contiguous")
    B, N = input.shape
    out = torch.empty((B,), dtype=torch.float32, device=input.device)
    if B == 0:
        return out
    call("fl_intlse_q10_6_i16", ptr(input, ctypes.c_int16), ptr(out), B, N, _stream(input))
    return out


# --------------------------------------------------------------------------
# Vocab-shard partial states
# --------------------------------------------------------------------------
def lse_partial(x: torch.Tensor) -> torch.Tensor:
    """(B, N) fp32/fp16 -> (B, 2) fp32 rows of (max, sum exp(x - max))."""
    _check(x.dim() == 2, "Expected 2-D tensor (B, N)")
    _check(x.is_cuda and x.dtype in (torch.float32, torch.float16), "Input must be CUDA fp32 or fp16")
    _check(x.is_contiguous(), "Input must be contiguous")
    B, N = x.shape
    ms = torch.empty((B, 2), dtype=torch.float32, device=x.device)
    if B == 0:
        return ms
    if x.dtype == torch.float32:
        call("fl_lse_f32_partial", ptr(x), ptr(ms), B, N, _stream(x))
    else:
        call("fl_lse_f16_partial", ptr(x, ctypes.c_uint16), ptr(ms), B, N, _stream(x))
    return ms


def lse_combine(ms: torch.Tensor) -> torch.Tensor:
    """(G, B, 2) shard partials -> (B,) fp32 log-sum-exp over all shards."""
    _check(ms.dim() == 3 and ms.size(2) == 2, "Expected (G, B, 2) partial states")
    _check(ms.is_cuda and ms.dtype == torch.float32, "Partials must be CUDA fp32")
    _check(ms.is_contiguous(), "Partials must be contiguous")
    G, B, _ = ms.shape
    out = torch.empty((B,), dtype=torch.float32, device=ms.device)
    if B == 0:
        return out
    call("fl_lse_combine", ptr(ms), ptr(out), G, B, _stream(ms))
    return out


# --------------------------------------------------------------------------
# Sparse PC sum layer (sparse_float_kernel.cu / sparse_q16_kernel.cu)
# --------------------------------------------------------------------------
def _sparse(fn: str, node_mars, element_mars, params, nids, cids, pids, block_size: int,
            err_flag=None) -> None:
    _check(node_mars.is_cuda, "node_mars must be CUDA")
    _check(element_mars.is_cuda, "element_mars must be CUDA")
    _check(params.is_cuda, "params must be CUDA")
    for name, t, dt in (("node_mars", node_mars, torch.float32),
                        ("element_mars", element_mars, torch.float32),
                        ("params", params, torch.float32),
                        ("nids", nids, torch.int64), ("cids", cids, torch.int64),
                        ("pids", pids, torch.int64)):
        _check(t.dtype == dt, f"{name} must be {dt}")
        _check(t.is_contiguous(), f"{name} must be contiguous")
        _check(t.device == node_mars.device, f"{name} must be on {node_mars.device}")
    _check(node_mars.dim() == 2 and element_mars.dim() == 2, "node_mars / element_mars must be 2-D")
    _check(cids.dim() == 2 and pids.shape == cids.shape and nids.dim() == 1 and
           nids.size(0) == cids.size(0), "nids (K,), cids and pids (K, E) expected")
    batch = node_mars.size(1)
    _check(element_mars.size(1) == batch, "element_mars and node_mars batch sizes differ")
    num_nblocks, num_edges = cids.shape
    ef = ptr(err_flag, ctypes.c_int) if err_flag is not None else None
    call(fn, ptr(node_mars), ptr(element_mars), ptr(params), ptr(nids, ctypes.c_int64),
         ptr(cids, ctypes.c_int64), ptr(pids, ctypes.c_int64), node_mars.size(0),
         element_mars.size(0), params.numel(), num_nblocks, num_edges, batch, int(block_size),
         ef, _stream(node_mars))


def sparse_forward_float(node_mars, element_mars, params, nids, cids, pids, block_size) -> None:
    """In place: node_mars[nids[k]+p, b] = LSE_e(log params[pids[k,e]+p] + element_mars[cids[k,e], b])."""
    _sparse("fl_sparse_f32", node_mars, element_mars, params, nids, cids, pids, block_size)


def sparse_forward_q16(node_mars, element_mars, params, nids, cids, pids, block_size) -> None:
    """Q16.16 version of sparse_forward_float, bit-identical to the reference kernel."""
    _sparse("fl_sparse_q16", node_mars, element_mars, params, nids, cids, pids, block_size)


def sparse_parent_index(nids: torch.Tensor, cids: torch.Tensor, pids: torch.Tensor,
                        block_size: int, num_elements: int):
    """Child -> parent-unit index of a layer structure, built once:
    (child_ptr, unit_node, unit_param).  The parent units of child c — one per
    edge (k, e) with cids[k, e] = c and per p < block_size — are
    [child_ptr[c], child_ptr[c+1]) of unit_node (node row nids[k] + p) and
    unit_param (pids[k, e] + p), in edge order (a stable sort, so the backward
    sums each child's parents in a fixed order).  Edges whose child is out of
    range are left out."""
    _check(cids.is_cuda and cids.dtype == torch.int64 and cids.dim() == 2, "cids must be CUDA int64 (K, E)")
    _check(pids.shape == cids.shape and nids.dim() == 1 and nids.size(0) == cids.size(0),
           "nids (K,), cids and pids (K, E) expected")
    E = cids.size(1)
    flat = cids.reshape(-1)
    valid = (flat >= 0) & (flat < num_elements)
    keys = torch.where(valid, flat, torch.full_like(flat, num_elements))
    order = torch.argsort(keys, stable=True)
    counts = torch.bincount(keys, minlength=num_elements + 1)[:num_elements] * block_size
    child_ptr = torch.zeros(num_elements + 1, dtype=torch.int64, device=cids.device)
    torch.cumsum(counts, 0, out=child_ptr[1:])
    ar = torch.arange(block_size, device=cids.device, dtype=torch.int64)
    unit_node = (nids[order // max(E, 1)][:, None] + ar[None, :]).reshape(-1).contiguous()
    unit_param = (pids.reshape(-1)[order][:, None] + ar[None, :]).reshape(-1).contiguous()
    return child_ptr, unit_node, unit_param


def sparse_bwd_workspace_bytes(num_nodes: int, batch: int, num_units: int) -> int:
    """Bytes of the workspace sparse_backward_float(..., fold=True) uses for
    node_mars of (num_nodes, batch) and num_units parent units (the length of
    sparse_parent_index's unit arrays, cids.numel() * block_size)."""
    nbytes = ctypes.c_int64()
    call("fl_sparse_f32_bwd_workspace", int(num_nodes), int(batch), int(num_units),
         ctypes.byref(nbytes))
    return nbytes.value


def sparse_backward_float(node_mars, node_grads, element_mars, params, nids, cids, pids,
                          block_size: int, element_grads=None, param_grads=None, parents=None,
                          err_flag=None, fold: bool = True, workspace=None):
    """Gradient of sparse_forward_float, added into element_grads (like
    element_mars) and param_grads (like params); either may be None to skip it.
    node_grads is d loss / d node_mars (only the layer's rows are read);
    `parents` is sparse_parent_index(nids, cids, pids, block_size,
    element_mars.size(0)), built here if None.  fold=True (the default) first
    folds G and node_mars into one row per node so the element gradients gather
    half the bytes, and takes the parameter gradients from the same pass; its
    scratch is `workspace` (a CUDA uint8 tensor of at least
    sparse_bwd_workspace_bytes(*node_mars.shape, num_units)), allocated here if None.
    Returns (element_grads, param_grads)."""
    for name, t, dt in (("node_mars", node_mars, torch.float32), ("node_grads", node_grads, torch.float32),
                        ("element_mars", element_mars, torch.float32), ("params", params, torch.float32),
                        ("nids", nids, torch.int64), ("cids", cids, torch.int64),
                        ("pids", pids, torch.int64)):
        _check(t.is_cuda and t.dtype == dt and t.is_contiguous(), f"{name} must be contiguous CUDA {dt}")
        _check(t.device == node_mars.device, f"{name} must be on {node_mars.device}")
    _check(node_grads.shape == node_mars.shape, "node_grads must match node_mars")
    _check(cids.dim() == 2 and pids.shape == cids.shape and nids.dim() == 1 and
           nids.size(0) == cids.size(0), "nids (K,), cids and pids (K, E) expected")
    batch = node_mars.size(1)
    _check(element_mars.size(1) == batch, "element_mars and node_mars batch sizes differ")
    for name, t, like in (("element_grads", element_grads, element_mars), ("param_grads", param_grads, params)):
        if t is not None:
            _check(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.shape == like.shape
                   and t.device == node_mars.device,
                   f"{name} must be a contiguous CUDA fp32 tensor shaped like {tuple(like.shape)}")
    child_ptr = unit_node = unit_param = None
    num_units = 0
    if element_grads is not None:
        if parents is None:
            parents = sparse_parent_index(nids, cids, pids, block_size, element_mars.size(0))
        child_ptr, unit_node, unit_param = parents
        _check(child_ptr.numel() == element_mars.size(0) + 1 and unit_node.shape == unit_param.shape,
               "parents index does not match this layer")
        num_units = unit_node.numel()
    num_nblocks, num_edges = cids.shape
    ws, ws_bytes = None, 0
    if fold and element_grads is not None:
        need = sparse_bwd_workspace_bytes(node_mars.size(0), batch, num_units)
        if workspace is None:
            workspace = torch.empty(need, dtype=torch.uint8, device=node_mars.device)
        _check(workspace.is_cuda and workspace.dtype == torch.uint8 and workspace.is_contiguous()
               and workspace.numel() >= need and workspace.device == node_mars.device,
               f"workspace must be a contiguous CUDA uint8 tensor of >= {need} bytes")
        ws, ws_bytes = ctypes.c_void_p(workspace.data_ptr()), workspace.numel()
    ef = ptr(err_flag, ctypes.c_int) if err_flag is not None else None
    call("fl_sparse_f32_bwd", ptr(node_mars), ptr(node_grads), ptr(element_mars), ptr(params),
         ptr(nids, ctypes.c_int64), ptr(cids, ctypes.c_int64), ptr(pids, ctypes.c_int64),
         ptr(child_ptr, ctypes.c_int64), ptr(unit_node, ctypes.c_int64),
         ptr(unit_param, ctypes.c_int64), num_units, ptr(element_grads), ptr(param_grads),
         node_mars.size(0), element_mars.size(0), params.numel(), num_nblocks, num_edges, batch,
         int(block_size), ws, ws_bytes, ef, _stream(node_mars))
    return element_grads, param_grads


def sparse_log_weights(params: torch.Tensor) -> torch.Tensor:
    """The device-formed log-weights __logf(fmaxf(w, 1e-45f)) the sparse kernels use."""
    _check(params.is_cuda and params.dtype == torch.float32 and params.is_contiguous(),
           "params must be contiguous CUDA fp32")
    out = torch.empty_like(params)
    if params.numel():
        call("fl_sparse_log_weights", ptr(params), ptr(out), params.numel(), _stream(params))
    return out


def version() -> int:
    return _lib.lib().fl_version()
