"""fuselse_b200 — row log-sum-exp kernels for NVIDIA B200 (sm_100a).

A drop-in for the FuseLSE / IntLSE reference call surface:

    import fuselse_b200
    logsumexp = fuselse_b200.make_fuselse_logsumexp(fuselse_b200.ext, robust=True)
    y = logsumexp(x, dim=-1)          # x: CUDA fp32, autograd-capable

`fuselse_b200.ext` carries the reference extension method names
(onepass_lse_float[_robust|_backward], batched_logsumexp[_nolut|_fp16|_q10_6],
sparse_forward_float, sparse_forward_q16) backed by the C ABI of
libfuselse_b200.so (include/fuselse_b200.h).  `fuselse_b200.distributed`
shards rows across GPUs and combines vocab-sharded rows over NCCL or the
library's own NVLink exchange.  `selective_log_softmax(logits, index)` is the
fused per-token log-probability (target gather + LSE in one pass).
`fuselse_b200.pc` has the pyjuice `SumLayer._forward_sparse` hook and a
differentiable sparse sum layer (its backward on the device too), and
`fuselse_b200.host` runs the forward and backward on rows held in pinned host
memory with the copies overlapped.
"""
from . import ext
from .autograd import make_fuselse_logsumexp
from .selective import selective_log_softmax

__all__ = ["ext", "make_fuselse_logsumexp", "selective_log_softmax"]
