"""torch.logsumexp-compatible wrapper with autograd (reference: fuselse/gpu/autograd.py:6-61).

`make_fuselse_logsumexp(extension, robust=True)` takes any object exposing the
reference method names (`onepass_lse_float[_robust]`,
`onepass_lse_float_backward`) — `fuselse_b200.ext` by default — and returns
`logsumexp(input, dim=-1, keepdim=False)`.

Behaviour kept from the reference:
  * inputs that are not CUDA fp32, or whose reduced dim is < 2 long, are
    delegated to torch.logsumexp (API behaviour, not a CPU kernel of this
    library);
  * with grad enabled and input.requires_grad, an autograd Function saves the
    input and the result and calls the fused backward;
  * otherwise 2-D contiguous inputs go straight to the forward kernel.

Where the reference copies (`reshape(-1, N).contiguous()`, autograd.py:19,56)
or delegates (dim != -1, :44-49), an extension that also provides the
in-place layouts (`fuselse_b200.ext` does) reads the tensor where it lies:
  * last-dim reductions of non-contiguous inputs whose rows are unit-stride
    and whose leading dims form at most two stride levels (a slice such as
    logits[:, :-1, :]) go to the strided-row kernels;
  * reductions over another dim of a contiguous input go to the
    middle-dim kernels.
Anything else is copied to a contiguous (-1, N) view as the reference does,
or delegated to torch.logsumexp.
"""
from __future__ import annotations

import torch


def make_fuselse_logsumexp(extension=None, robust: bool = True):
    if extension is None:
        from . import ext as extension
    forward_kernel = extension.onepass_lse_float_robust if robust else extension.onepass_lse_float
    backward_kernel = extension.onepass_lse_float_backward
    in_place = all(hasattr(extension, n) for n in (
        "row_layout", "onepass_lse_float_strided", "onepass_lse_float_backward_strided",
        "logsumexp_dim", "logsumexp_dim_backward"))
    reference_logsumexp = torch.logsumexp

    def dense_rows(t):
        """(..., N) as a dense (R, N) matrix — a view when the rows already are
        dense, else the copy the reference makes — and the leading shape."""
        return t.reshape(-1, t.shape[-1]).contiguous(), t.shape[:-1]

    class DenseRowsLSE(torch.autograd.Function):
        """Last-dim reduction over dense rows.  Keeps the (R, N) rows and their
        lse for the backward, which is one fused pass g * exp(x - lse)."""

        @staticmethod
        def forward(ctx, t):
            rows, lead = dense_rows(t)
            lse = forward_kernel(rows)
            ctx.save_for_backward(rows, lse)
            ctx.shape = t.shape
            return lse.view(lead)

        @staticmethod
        def backward(ctx, g):
            rows, lse = ctx.saved_tensors
            return backward_kernel(g.reshape(-1).contiguous(), rows, lse).view(ctx.shape)

    class FuseLSEStridedFunction(torch.autograd.Function):
        """Last-dim reduction of a strided input, read in place (no copy)."""

        @staticmethod
        def forward(ctx, input_tensor):
            output = extension.onepass_lse_float_strided(input_tensor, robust=robust)
            ctx.save_for_backward(input_tensor, output)
            return output

        @staticmethod
        def backward(ctx, grad_output):
            input_tensor, output = ctx.saved_tensors
            return extension.onepass_lse_float_backward_strided(grad_output, input_tensor, output)

    class FuseLSEDimFunction(torch.autograd.Function):
        """Reduction over a dim other than the last of a contiguous input."""

        @staticmethod
        def forward(ctx, input_tensor, dim):
            output = extension.logsumexp_dim(input_tensor, dim, robust=robust)
            ctx.save_for_backward(input_tensor, output)
            ctx.dim = dim
            return output

        @staticmethod
        def backward(ctx, grad_output):
            input_tensor, output = ctx.saved_tensors
            return extension.logsumexp_dim_backward(grad_output, input_tensor, output, ctx.dim), None

    def logsumexp(input_tensor, dim=-1, keepdim=False):
        if isinstance(dim, (tuple, list)):
            if len(dim) != 1:
                return reference_logsumexp(input_tensor, dim=dim, keepdim=keepdim)
            dim = dim[0]
        if not (input_tensor.is_cuda and input_tensor.dtype == torch.float32
                and input_tensor.dim() >= 1):
            return reference_logsumexp(input_tensor, dim=dim, keepdim=keepdim)
        normalized_dim = dim if dim >= 0 else input_tensor.dim() + dim
        last = input_tensor.dim() - 1
        if not 0 <= normalized_dim <= last or input_tensor.shape[normalized_dim] < 2:
            return reference_logsumexp(input_tensor, dim=dim, keepdim=keepdim)
        grad = torch.is_grad_enabled() and input_tensor.requires_grad
        if normalized_dim != last:
            if not (in_place and input_tensor.is_contiguous()):
                return reference_logsumexp(input_tensor, dim=dim, keepdim=keepdim)
            result = (FuseLSEDimFunction.apply(input_tensor, normalized_dim) if grad
                      else extension.logsumexp_dim(input_tensor, normalized_dim, robust=robust))
            return result.unsqueeze(normalized_dim) if keepdim else result
        strided = (in_place and not input_tensor.is_contiguous()
                   and extension.row_layout(input_tensor) is not None)
        if strided:
            result = (FuseLSEStridedFunction.apply(input_tensor) if grad
                      else extension.onepass_lse_float_strided(input_tensor, robust=robust))
        elif grad:
            result = DenseRowsLSE.apply(input_tensor)
        else:  # no graph: a dense 2-D input goes to the kernel as it is
            rows, lead = dense_rows(input_tensor)
            result = forward_kernel(rows).view(lead)
        return result.unsqueeze(-1) if keepdim else result

    logsumexp.autograd_function = DenseRowsLSE
    return logsumexp
