"""torch.logsumexp-compatible wrapper with autograd (reference: fuselse/gpu/autograd.py:6-61).

`make_fuselse_logsumexp(extension, robust=True)` takes any object exposing the
reference method names (`onepass_lse_float[_robust]`,
`onepass_lse_float_backward`) — `fuselse_b200.ext` by default — and returns
`logsumexp(input, dim=-1, keepdim=False)`.

Behaviour kept from the reference:
  * inputs that are not CUDA fp32, not reduced over the last dim, or whose last
    dim is < 2 are delegated to torch.logsumexp (API behaviour, not a CPU
    kernel of this library);
  * with grad enabled and input.requires_grad, an autograd Function saves the
    flattened input and the result and calls the fused backward;
  * otherwise 2-D contiguous inputs go straight to the forward kernel, others
    are flattened to (-1, N) first.
"""
from __future__ import annotations

import torch


def make_fuselse_logsumexp(extension=None, robust: bool = True):
    if extension is None:
        from . import ext as extension
    forward_kernel = extension.onepass_lse_float_robust if robust else extension.onepass_lse_float
    backward_kernel = extension.onepass_lse_float_backward
    reference_logsumexp = torch.logsumexp

    class FuseLSEFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, input_tensor):
            row_size = input_tensor.shape[-1]
            flat_input = input_tensor.reshape(-1, row_size).contiguous()
            output = forward_kernel(flat_input)
            ctx.save_for_backward(flat_input, output)
            ctx.input_shape = tuple(input_tensor.shape)
            return output.reshape(input_tensor.shape[:-1])

        @staticmethod
        def backward(ctx, grad_output):
            flat_input, output = ctx.saved_tensors
            flat_grad = grad_output.reshape(-1).contiguous()
            grad_input = backward_kernel(flat_grad, flat_input, output)
            return grad_input.reshape(ctx.input_shape)

    def logsumexp(input_tensor, dim=-1, keepdim=False):
        if isinstance(dim, (tuple, list)):
            if len(dim) != 1:
                return reference_logsumexp(input_tensor, dim=dim, keepdim=keepdim)
            dim = dim[0]
        normalized_dim = dim if dim >= 0 else input_tensor.dim() + dim
        supported = (
            input_tensor.is_cuda
            and input_tensor.dtype == torch.float32
            and input_tensor.dim() >= 1
            and normalized_dim == input_tensor.dim() - 1
            and input_tensor.shape[-1] >= 2
        )
        if not supported:
            return reference_logsumexp(input_tensor, dim=dim, keepdim=keepdim)
        if torch.is_grad_enabled() and input_tensor.requires_grad:
            result = FuseLSEFunction.apply(input_tensor)
        elif input_tensor.dim() == 2 and input_tensor.is_contiguous():
            result = forward_kernel(input_tensor)
        else:
            row_size = input_tensor.shape[-1]
            flat_input = input_tensor.reshape(-1, row_size).contiguous()
            result = forward_kernel(flat_input).reshape(input_tensor.shape[:-1])
        return result.unsqueeze(-1) if keepdim else result

    logsumexp.FuseLSEFunction = FuseLSEFunction
    return logsumexp
