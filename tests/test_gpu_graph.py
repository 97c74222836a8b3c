"""The hot path inside a CUDA graph: forward + backward captured through the
public entry points (C ABI launches on the capturing stream), replayed, and
compared with eager calls on the same buffers."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fwd_bwd_graph_capture_matches_eager(ext):
    B, N = 64, 128256
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(B, N, generator=g, device="cuda")
    go = torch.rand(B, generator=g, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):  # warm-up on the capture stream
            lse = ext.onepass_lse_float_robust(x)
            gx = ext.onepass_lse_float_backward(go, x, lse)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            lse_g = ext.onepass_lse_float_robust(x)
            gx_g = ext.onepass_lse_float_backward(go, x, lse_g)
    torch.cuda.current_stream().wait_stream(s)
    lse_g.zero_()
    gx_g.zero_()
    graph.replay()
    torch.cuda.synchronize()
    lse_e = ext.onepass_lse_float_robust(x)
    gx_e = ext.onepass_lse_float_backward(go, x, lse_e)
    assert torch.equal(lse_g, lse_e)
    assert torch.equal(gx_g, gx_e)
    x.add_(1.0)          # replay sees new input values in the same buffer
    graph.replay()
    torch.cuda.synchronize()
    assert torch.allclose(lse_g, ext.onepass_lse_float_robust(x), rtol=0, atol=0)
    del graph


def test_intlse_graph_capture(ext):
    q = (torch.randn(16384, 4096, device="cuda") * 65536 * 2).round().to(torch.int32)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ext.batched_logsumexp_q16_i32(q)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            out = ext.batched_logsumexp_q16_i32(q)
    torch.cuda.current_stream().wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int32), ext.batched_logsumexp_q16_i32(q).view(torch.int32))
    del graph


def test_capture_with_torch_graph_default_stream(ext):
    """torch.cuda.graph() captures on its own side stream, which this library
    has not seen before the capture starts: the first call on it must not
    query the stream in a way the capture refuses (the capture would be
    invalidated).  Forward, backward, selective log-softmax and IntLSE."""
    B, N = 96, 50000
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(B, N, generator=g, device="cuda")
    go = torch.rand(B, generator=g, device="cuda")
    t = torch.randint(0, N, (B,), generator=g, device="cuda")
    q = (x * 65536).round().to(torch.int32)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        lse_g = ext.onepass_lse_float_robust(x)
        gx_g = ext.onepass_lse_float_backward(go, x, lse_g)
        logp_g, lse2_g = ext.selective_logsoftmax_rows(x, t)
        iq_g = ext.batched_logsumexp_q16_i32(q)
    graph.replay()
    torch.cuda.synchronize()
    lse = ext.onepass_lse_float_robust(x)
    assert torch.equal(lse_g, lse)
    assert torch.equal(gx_g, ext.onepass_lse_float_backward(go, x, lse))
    logp, lse2 = ext.selective_logsoftmax_rows(x, t)
    assert torch.equal(logp_g, logp) and torch.equal(lse2_g, lse2)
    assert torch.equal(iq_g.view(torch.int32), ext.batched_logsumexp_q16_i32(q).view(torch.int32))
    del graph
