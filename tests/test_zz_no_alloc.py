"""fl_lse_vocab_exchange_noalloc: the single-rank vocab exchange for callers
that cannot allocate device memory (a host whose GPU is driven through a
plugin or embedded runtime that owns every allocation, or code whose memory
budget is fixed before it runs).  Its exchange buffer is a static array inside
the library instead of a caller allocation.

Called through the C ABI and compared, on two calls in a row, with the
allocating entry point fl_lse_vocab_exchange (G = 1, caller buffer) on the same
input, within the tolerance of the other fp32/fp16 tests.  This file sorts
last so that a run stopping at its first failure has already run every other
test; it also passes alone in a fresh process.
"""
import ctypes

import pytest
import torch

from fuselse_b200 import _lib
from fuselse_b200.distributed import VocabShardExchange

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _noalloc(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty(x.size(0), dtype=torch.float32, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    _lib.call("fl_lse_vocab_exchange_noalloc", ctypes.c_void_p(x.data_ptr()),
              0 if x.dtype == torch.float32 else 1, x.size(0), x.size(1), _lib.ptr(out), stream)
    return out


def _rel(a, b):
    return ((a - b).abs() / b.abs().clamp_min(1.0)).max().item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_noalloc_matches_allocating_entry_two_calls(dtype):
    B, N = 8192, 16032
    g = torch.Generator(device="cuda").manual_seed(11)
    x = (torch.randn(B, N, generator=g, device="cuda") * 3).to(dtype)
    x[5] = float("-inf")
    ref = VocabShardExchange.single_rank(B, "cuda")
    for _ in range(2):
        want = ref(x)
        got = _noalloc(x)
        torch.cuda.synchronize()
        assert got[5] == float("-inf") and want[5] == float("-inf")
        fin = torch.isfinite(want)
        assert torch.isfinite(got[fin]).all()
        assert _rel(got[fin], want[fin]) <= RTOL


def test_noalloc_rejects_oversize_request():
    x = torch.zeros(300_000, 4, device="cuda")
    with pytest.raises(_lib.FuseLSEError, match="at most 262112 rows"):
        _noalloc(x)
