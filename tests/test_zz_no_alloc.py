"""fl_lse_vocab_exchange_noalloc: the single-rank vocab exchange for callers
that cannot allocate device memory (a host whose GPU is driven through a
plugin or embedded runtime that owns every allocation, or code whose memory
budget is fixed before it runs).  Its exchange buffer is a static array inside
the library instead of a caller allocation.

Called through the C ABI and compared, on two calls in a row, with the
allocating entry point fl_lse_vocab_exchange (G = 1, caller buffer) on the same
input and with the fp64 oracle, within the tolerance of the other fp32/fp16
tests; the row limit is checked at its boundary.  This file sorts last so that
a run stopping at its first failure has already run every other test; it also
passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from fuselse_b200 import _lib
from fuselse_b200.distributed import VocabShardExchange
from oracle import oracle as O

MAX_ROWS = 262112  # (4 MiB - 512 B of header and flags) / 16 B per row

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
    f64 = torch.from_numpy(O.lse_f64(x.float().cpu().numpy())).cuda()
    for _ in range(2):
        want = ref(x)
        got = _noalloc(x)
        torch.cuda.synchronize()
        assert got[5] == float("-inf") and want[5] == float("-inf")
        fin = torch.isfinite(want)
        assert torch.isfinite(got[fin]).all()
        assert _rel(got[fin], want[fin]) <= RTOL
        assert _rel(got[fin].double(), f64[fin]) <= RTOL


def test_noalloc_row_limit_boundary():
    # the largest accepted request fills the static buffer exactly
    B, N = MAX_ROWS, 7
    x = torch.randn(B, N, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda")
    want = torch.from_numpy(O.lse_f64(x.cpu().numpy())).cuda()
    for _ in range(2):
        got = _noalloc(x)
        torch.cuda.synchronize()
        assert _rel(got.double(), want) <= RTOL
    np.testing.assert_array_equal(got.cpu().numpy(),
                                  VocabShardExchange.single_rank(B, "cuda")(x).cpu().numpy())
    with pytest.raises(_lib.FuseLSEError, match=f"at most {MAX_ROWS} rows"):
        _noalloc(torch.zeros(MAX_ROWS + 1, 4, device="cuda"))


def test_noalloc_rejects_oversize_request():
    x = torch.zeros(300_000, 4, device="cuda")
    with pytest.raises(_lib.FuseLSEError, match=f"at most {MAX_ROWS} rows"):
        _noalloc(x)
