"""Failure detection of the vocab exchange, on one GPU and without a fault.

fl_lse_vocab_exchange's combine kernel waits for every rank's flag with a
bounded poll.  Here one process calls it as rank 0 of a G = 2 group whose peer
table holds two buffers of this GPU, so "rank 1" never publishes: the wait must
run out within the limit (lowered to 50 ms for the test), the rows come out
NaN, the sticky error word is set, and the context stays usable — the next
well-formed exchange on a zero-filled buffer gives the fp64 result.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from fuselse_b200 import _lib
from fuselse_b200.distributed import VocabShardExchange
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HEADER = 256  # header bytes; the flags (one u32 per rank) follow


def _set_limit(ns: int) -> int:
    prev = ctypes.c_int64()
    _lib.call("fl_vocab_exchange_set_wait_limit", ns, ctypes.byref(prev))
    return prev.value


def _exchange(x, peers, local, rank, G, out):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.call("fl_lse_vocab_exchange", ctypes.c_void_p(x.data_ptr()), 0, x.size(0), x.size(1),
              ctypes.c_void_p(peers.data_ptr()), ctypes.c_void_p(local.data_ptr()), rank, G,
              _lib.ptr(out), stream)


def test_exchange_wait_runs_out_and_reports():
    B, N, G = 64, 1000, 2
    nbytes = ctypes.c_int64()
    _lib.call("fl_vocab_exchange_bytes", G, B, ctypes.byref(nbytes))
    bufs = [torch.zeros(nbytes.value, dtype=torch.uint8, device="cuda") for _ in range(G)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    x = torch.randn(B, N, generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    out = torch.zeros(B, device="cuda")
    prev = _set_limit(50_000_000)
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _exchange(x, peers, bufs[0], 0, G, out)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        _set_limit(prev)
    assert elapsed < 5.0, f"the bounded wait took {elapsed:.1f} s"
    assert torch.isnan(out).all(), "rows of a call whose peer never arrived must be NaN"
    hdr = bufs[0][:16].view(torch.int32).cpu().numpy()
    assert hdr[1] == 1, "sticky error word"
    assert hdr[0] == 1, "the call still finished (epoch advanced)"
    # rank 0 published its delivery into both buffers' flag words; rank 1's stayed 0
    assert bufs[0][HEADER:HEADER + 8].view(torch.int32).tolist() == [1, 0]
    assert bufs[1][HEADER:HEADER + 8].view(torch.int32).tolist() == [1, 0]

    # the context is still usable: a well-formed exchange gives the right rows
    ex = VocabShardExchange.single_rank(B)
    for _ in range(2):
        got = ex(x).cpu().numpy()
        want = O.lse_f64(x.cpu().numpy())
        assert np.max(np.abs(got - want) / np.maximum(np.abs(want), 1.0)) <= 1e-5
    assert not ex.error()
    # and the failed buffer, zero-filled again, serves a G = 1 exchange
    bufs[0].zero_()
    one = torch.tensor([bufs[0].data_ptr()], dtype=torch.int64, device="cuda")
    out1 = torch.empty(B, device="cuda")
    _exchange(x, one, bufs[0], 0, 1, out1)
    np.testing.assert_array_equal(out1.cpu().numpy(), ex(x).cpu().numpy())
    assert bufs[0][4:8].view(torch.int32).item() == 0
