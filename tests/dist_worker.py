"""Per-rank body of tests/test_gpu_dist.py (run under torchrun, one process per GPU).

Each rank builds the same seeded inputs, takes its shard and checks the
distributed result against the single-GPU kernels on the full input:
  * vocab shards: ext.lse_partial on the local columns + NCCL all-gather of the
    (max, sumexp) pairs + ext.lse_combine, fp16 logits of the LLM config shape
    (rows scaled down);
  * vocab shards through the library's NVLink exchange, forward and backward;
  * batch rows: robust fp32 forward on the local rows, gathered;
  * sparse layer over batch-column shards (fp32 and Q16.16), gathered, and its
    backward: element gradients gathered, parameter gradients all-reduced.
Exits non-zero on any mismatch.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
    from fuselse_b200 import distributed as D, ext, workloads as W

    G = dist.get_world_size()
    # vocab shards of fp16 logits (B, 128256)
    B, V = 256, 128256
    logits = W.fp16_logits(B, V, seed=3, device=dev)
    lo, hi = D.local_columns(V)
    got = D.vocab_sharded_logsumexp(logits[:, lo:hi].contiguous())
    want = ext.batched_logsumexp_fp16(logits)
    err = ((got - want).abs() / want.abs().clamp_min(1.0)).max().item()
    assert err <= 1e-5, f"vocab-shard combine err {err}"
    # fp32 shards, robust rules across shards (-inf row, +inf in one shard)
    x = W.fp32_rows(64, 40000, seed=4, device=dev)
    x[3] = float("-inf")
    x[5, 39999] = float("inf")
    lo, hi = D.local_columns(x.size(1))
    got = D.vocab_sharded_logsumexp(x[:, lo:hi].contiguous())
    want = ext.onepass_lse_float_robust(x)
    assert got[3] == float("-inf") and got[5] == float("inf")
    fin = torch.isfinite(want)
    err = ((got[fin] - want[fin]).abs() / want[fin].abs().clamp_min(1.0)).max().item()
    assert err <= 1e-5, f"fp32 vocab-shard err {err}"
    # the same through the library's own NVLink exchange (peer stores + flags),
    # several calls in a row (epochs, slot alternation) and from a CUDA graph
    ex = D.VocabShardExchange(B, device=dev)
    lo, hi = D.local_columns(V)
    shard = logits[:, lo:hi].contiguous()
    want16 = ext.batched_logsumexp_fp16(logits)
    for _ in range(3):
        got = ex(shard)
        err = ((got - want16).abs() / want16.abs().clamp_min(1.0)).max().item()
        assert err <= 1e-5, f"peer exchange err {err}"
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ex(shard)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            g_out = ex(shard)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g_out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        err = ((g_out - want16).abs() / want16.abs().clamp_min(1.0)).max().item()
        assert err <= 1e-5, f"peer exchange (graph replay) err {err}"
    del graph
    ex32 = D.VocabShardExchange(x.size(0), device=dev)
    lo, hi = D.local_columns(x.size(1))
    got = ex32(x[:, lo:hi].contiguous())
    assert got[3] == float("-inf") and got[5] == float("inf")
    err = ((got[fin] - want[fin]).abs() / want[fin].abs().clamp_min(1.0)).max().item()
    assert err <= 1e-5, f"fp32 peer exchange err {err}"
    assert not ex.error() and not ex32.error()
    # vocab-sharded forward + backward through autograd: each rank's shard
    # gradient equals those columns of the single-GPU backward
    xs = x[8:, lo:hi].contiguous().requires_grad_()
    ex_g = D.VocabShardExchange(xs.size(0), device=dev)
    lse = D.vocab_sharded_logsumexp_grad(xs, ex_g)
    w = torch.linspace(0.5, 2.0, lse.numel(), device=dev)  # same loss on every rank
    (lse * w).sum().backward()
    full = x[8:].contiguous()
    want_g = ext.onepass_lse_float_backward(w, full, ext.onepass_lse_float_robust(full))[:, lo:hi]
    fin_g = torch.isfinite(want_g)
    assert torch.equal(fin_g, torch.isfinite(xs.grad)), "vocab-shard backward: special values differ"
    gerr = (xs.grad[fin_g] - want_g[fin_g]).abs().max().item()
    assert gerr <= 1e-6 + 1e-5 * want_g[fin_g].abs().max().item(), f"vocab-shard backward err {gerr}"
    # the exchange buffers are CUDA IPC allocations: every rank unmaps its
    # peers' buffers, then (after a barrier inside close) frees its own
    for e in (ex, ex32, ex_g):
        e.close()
    # batch rows
    xb = W.fp32_rows(1000, 20000, seed=5, device=dev)
    r0, r1 = D.local_rows(xb.size(0))
    gathered = D.batch_sharded_logsumexp(xb[r0:r1], gather=True)
    # fewer rows per rank can change the launch shape (rows split over a
    # cluster), hence the float association: equal to rounding, not bit for bit
    want_b = ext.onepass_lse_float_robust(xb)
    err = ((gathered - want_b).abs() / want_b.abs().clamp_min(1.0)).max().item()
    assert err <= 1e-5, f"batch-shard gather err {err}"
    # IntLSE's reduction order is fixed per row, so sharded rows are bit-exact
    _, qb, _ = W.intlse_inputs(256, 40000, seed=6, device=dev)
    r0, r1 = D.local_rows(qb.size(0))
    got_q = D.batch_sharded_logsumexp(qb[r0:r1], gather=True, lse_fn=ext.batched_logsumexp_q16_i32)
    assert torch.equal(got_q, ext.batched_logsumexp_q16_i32(qb)), "IntLSE batch shards differ"
    # sparse layer sharded over batch columns: each rank holds its own
    # (P, batch/G) slice of element_mars; a column's result depends on that
    # column alone, so the gathered columns equal the 1-GPU layer bit for bit
    node, em, params, nids, cids, pids, bs = W.sparse_layer(P=20000, S=3000, E=32, batch=256,
                                                            seed=7, device=dev)
    c0, c1 = D.local_columns(em.size(1))
    for fn in (ext.sparse_forward_float, ext.sparse_forward_q16):
        full = node.clone()
        fn(full, em, params, nids, cids, pids, bs)
        mine = node[:, c0:c1].contiguous()
        fn(mine, em[:, c0:c1].contiguous(), params, nids, cids, pids, bs)
        parts = [torch.empty(node.size(0), hi - lo, device=dev)
                 for lo, hi in (D.split_range(em.size(1), G, r) for r in range(G))]
        dist.all_gather(parts, mine)
        assert torch.equal(torch.cat(parts, dim=1), full), f"{fn.__name__}: batch-column shards differ"
    # its backward over the same shards (data-parallel training): a column's
    # element gradients depend on that column alone (bit-exact), the parameter
    # gradients sum over the batch, so each rank's partial is all-reduced
    full = node.clone()
    ext.sparse_forward_float(full, em, params, nids, cids, pids, bs)
    up = torch.randn(node.shape, generator=torch.Generator(device=dev).manual_seed(8), device=dev)
    parents = ext.sparse_parent_index(nids, cids, pids, bs, em.size(0))
    gem, gw = torch.zeros_like(em), torch.zeros_like(params)
    ext.sparse_backward_float(full, up, em, params, nids, cids, pids, bs, element_grads=gem,
                              param_grads=gw, parents=parents)
    mine = full[:, c0:c1].contiguous()
    gem_r, gw_r = torch.zeros(em.size(0), c1 - c0, device=dev), torch.zeros_like(params)
    ext.sparse_backward_float(mine, up[:, c0:c1].contiguous(), em[:, c0:c1].contiguous(), params,
                              nids, cids, pids, bs, element_grads=gem_r, param_grads=gw_r,
                              parents=parents)
    parts = [torch.empty(em.size(0), hi - lo, device=dev)
             for lo, hi in (D.split_range(em.size(1), G, r) for r in range(G))]
    dist.all_gather(parts, gem_r)
    assert torch.equal(torch.cat(parts, dim=1), gem), "sparse backward: element-gradient shards differ"
    dist.all_reduce(gw_r)
    gerr = (gw_r - gw).abs().max().item()
    assert gerr <= 1e-6 + 1e-5 * gw.abs().max().item(), f"sparse backward: parameter gradients err {gerr}"
    dist.barrier()
    if dist.get_rank() == 0:
        print(f"dist ok: world {G}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
