"""world_size-2 gloo tests of the multi-GPU host logic on CPU ranks.

The local reductions are injected as CPU stand-ins built on the fp64 oracle
(the product's kernels need a GPU); what is under test is the exchange:
shard boundaries, the all-gather of (max, sumexp) partials, their rank-major
layout, the combine rule, and the batch-row gather.  A failure test makes one
rank drop out before the collective and checks that the other rank's
collective ends with an error instead of hanging.
"""
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial_cpu(x: torch.Tensor) -> torch.Tensor:
    a = x.double().numpy()
    with np.errstate(invalid="ignore", over="ignore"):
        m = a.max(axis=1)
        ms = np.where(m == -np.inf, 0.0, m)
        s = np.exp(a - ms[:, None]).sum(axis=1)
    return torch.from_numpy(np.stack([m, s], axis=1).astype(np.float32))


def _combine_cpu(ms: torch.Tensor) -> torch.Tensor:
    a = ms.double().numpy()               # (G, B, 2)
    m, s = a[..., 0], a[..., 1]
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        M = m.max(axis=0)
        Ms = np.where(M == -np.inf, 0.0, M)
        tot = (s * np.exp(m - Ms[None])).sum(axis=0)
        out = Ms + np.log(tot)
    out = np.where(M == np.inf, np.inf, out)
    out = np.where(M == -np.inf, -np.inf, out)
    return torch.from_numpy(out.astype(np.float32))


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=5 if mode == "fail" else 60))
        from fuselse_b200 import distributed as D
        from oracle import oracle as O

        gen = torch.Generator().manual_seed(0)
        B, N = 33, 1003
        x = torch.randn(B, N, generator=gen) * 3
        x[5, 7] = float("inf")
        x[6] = float("-inf")
        x[7, :500] = float("-inf")
        if mode == "vocab":
            lo, hi = D.local_columns(N)
            got = D.vocab_sharded_logsumexp(x[:, lo:hi].contiguous(), partial_fn=_partial_cpu,
                                            combine_fn=_combine_cpu)
            want = O.lse_f64(x.numpy())
            np.testing.assert_allclose(got.numpy(), want, rtol=1e-6)
            q.put((rank, "ok"))
        elif mode == "vocab_grad":
            lo, hi = D.local_columns(N)
            xs = x[8:, lo:hi].contiguous().double().requires_grad_()
            exchange = lambda t: D.vocab_sharded_logsumexp(t.detach().float(), partial_fn=_partial_cpu,
                                                           combine_fn=_combine_cpu).double()
            bwd = lambda g, xv, lse: g[:, None] * torch.exp(xv - lse[:, None])
            lse = D.vocab_sharded_logsumexp_grad(xs, exchange, bwd)
            w = torch.arange(1, lse.numel() + 1, dtype=torch.float64)  # same loss on every rank
            (lse * w).sum().backward()
            full = x[8:].double()
            want = w[:, None] * torch.softmax(full, dim=1)[:, lo:hi]
            np.testing.assert_allclose(xs.grad.numpy(), want.numpy(), rtol=1e-5, atol=1e-9)
            q.put((rank, "ok"))
        elif mode == "batch":
            lo, hi = D.local_rows(B)
            lse = lambda t: torch.from_numpy(O.lse_f64(t.numpy()).astype(np.float32))
            got = D.batch_sharded_logsumexp(x[lo:hi], gather=True, lse_fn=lse)
            np.testing.assert_allclose(got.numpy(), O.lse_f64(x.numpy()), rtol=1e-6)
            q.put((rank, "ok"))
        elif mode == "fail":
            if rank == 1:
                q.put((rank, "left"))
                q.close()
                q.join_thread()  # flush before the abrupt exit
                os._exit(0)  # drops out between steps, before its collective
            try:
                D.vocab_sharded_logsumexp(x[:, :10].contiguous(), partial_fn=_partial_cpu,
                                          combine_fn=_combine_cpu)
                q.put((rank, "no error"))
            except Exception as e:  # gloo reports the missing peer
                q.put((rank, "error:" + type(e).__name__))
            q.close()
            q.join_thread()
            os._exit(0)
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "exception:" + traceback.format_exc()))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, v = q.get(timeout=120)
        res[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_vocab_shard_combine_ws2():
    res = _run("vocab")
    assert res == {0: "ok", 1: "ok"}, res


def test_vocab_shard_backward_ws2():
    res = _run("vocab_grad")
    assert res == {0: "ok", 1: "ok"}, res


def test_batch_shard_gather_ws2():
    res = _run("batch")
    assert res == {0: "ok", 1: "ok"}, res


def test_rank_dropout_surfaces_as_error_ws2():
    res = _run("fail")
    assert res[1] == "left"
    assert res[0].startswith("error:"), res
