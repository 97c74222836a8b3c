"""Probabilistic-circuit sum layers: the pyjuice hook and an autograd form.

`make_sparse_dispatcher(ext_call)` returns a replacement for pyjuice's
`SumLayer._forward_sparse` that routes the log-likelihood ("LL") propagation
through one of this library's sparse kernels, with the call shape of the
reference experiment's hook (experiment_pyjuice/run_pyjuice.py:63-77): other
propagation algorithms go to the original method, `local_ids` selects node
blocks first, and the kernel writes node_mars in place.

`sparse_sum_layer(node_mars, element_mars, params, nids, cids, pids,
block_size)` is the same layer as a differentiable function: it returns a
copy of node_mars with the layer's rows replaced, and its backward gives the
gradients of element_mars and params through fl_sparse_f32_bwd (the
reference has a forward only) and passes node_mars' gradient through on the
rows the layer does not write.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import ext


def make_sparse_dispatcher(ext_call: Optional[Callable] = None, original: Optional[Callable] = None):
    """A `_forward_sparse(self, node_mars, element_mars, params, nids, cids, pids,
    local_ids=None, partition_id=-1, propagation_alg="LL", **kwargs)` method.

    ext_call(node_mars, element_mars, params, nids, cids, pids, block_size)
    defaults to ext.sparse_forward_float; `original` is the method to fall back
    to for propagation algorithms other than "LL" (pyjuice's own)."""
    call = ext_call if ext_call is not None else ext.sparse_forward_float

    def _forward_sparse(self, node_mars, element_mars, params, nids, cids, pids,
                        local_ids=None, partition_id=-1, propagation_alg="LL", **kwargs):
        if propagation_alg != "LL":
            if original is None:
                raise NotImplementedError(f"propagation_alg={propagation_alg!r} needs the original method")
            return original(self, node_mars, element_mars, params, nids, cids, pids,
                            local_ids=local_ids, partition_id=partition_id,
                            propagation_alg=propagation_alg, **kwargs)
        if local_ids is not None:
            nids, cids, pids = nids[local_ids], cids[local_ids], pids[local_ids]
        call(node_mars, element_mars, params, nids.contiguous(), cids.contiguous(),
             pids.contiguous(), self.block_size)
        return None

    return _forward_sparse


def layer_rows(nids: torch.Tensor, block_size: int) -> torch.Tensor:
    """Node rows a layer writes: nids[k] + p for p < block_size, in (k, p) order."""
    return (nids[:, None] + torch.arange(block_size, device=nids.device)[None, :]).reshape(-1)


class SparseSumLayer(torch.autograd.Function):
    @staticmethod
    def forward(ctx, node_mars, element_mars, params, nids, cids, pids, block_size, parents):
        out = node_mars.detach().clone()
        ext.sparse_forward_float(out, element_mars.detach(), params.detach(), nids, cids, pids, block_size)
        ctx.save_for_backward(out, element_mars, params, nids, cids, pids)
        ctx.block_size = block_size
        ctx.parents = parents
        return out

    @staticmethod
    def backward(ctx, grad_out):
        out, element_mars, params, nids, cids, pids = ctx.saved_tensors
        bs = ctx.block_size
        g = grad_out.contiguous()
        need_em, need_w = ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        em_grads = torch.zeros_like(element_mars) if need_em else None
        w_grads = torch.zeros_like(params) if need_w else None
        if need_em or need_w:
            ext.sparse_backward_float(out, g, element_mars.detach().contiguous(),
                                      params.detach().contiguous(), nids, cids, pids, bs,
                                      element_grads=em_grads, param_grads=w_grads,
                                      parents=ctx.parents)
        g_nodes = None
        if ctx.needs_input_grad[0]:
            g_nodes = g.clone()
            g_nodes[layer_rows(nids, bs)] = 0.0  # overwritten by the layer
        return g_nodes, em_grads, w_grads, None, None, None, None, None


def sparse_sum_layer(node_mars, element_mars, params, nids, cids, pids, block_size: int,
                     parents=None) -> torch.Tensor:
    """Differentiable sparse sum layer (fp32): node_mars with rows nids[k] + p
    replaced by LSE_e(log max(params[pids[k,e]+p], 1e-45) + element_mars[cids[k,e]]).
    `parents` = ext.sparse_parent_index(nids, cids, pids, block_size,
    element_mars.size(0)) may be passed to reuse the structure's index."""
    return SparseSumLayer.apply(node_mars, element_mars, params, nids, cids, pids, int(block_size),
                                parents)
