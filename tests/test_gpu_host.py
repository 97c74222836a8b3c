"""GPU parity of the host-row pipeline (fuselse_b200.host): chunked, copy-overlapped
forward + backward from pinned host memory against the device entry points on the
same values (bit-identical: the same kernels on the same rows), over several
calls in a row (the device ring is reused) and a partial last chunk."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pinned(t):
    return t.contiguous().pin_memory()


@pytest.mark.parametrize("B,N,chunk", [(300, 5003, 64), (7, 128256, 4), (1, 17, 8), (129, 1024, 32)])
def test_pipeline_matches_device_entry_points(ext, B, N, chunk):
    from fuselse_b200.host import HostRowPipeline
    pipe = HostRowPipeline(N, chunk_rows=chunk, depth=3)
    for call in range(3):
        g_ = torch.Generator().manual_seed(B + N + call)
        x = _pinned(torch.randn(B, N, generator=g_) * 3)
        g = _pinned(torch.randn(B, generator=g_))
        lse_h = _pinned(torch.empty(B))
        gx_h = _pinned(torch.empty(B, N))
        pipe.run(x, lse_h, g, gx_h)
        torch.cuda.synchronize()
        xd = x.cuda()
        lse_d = ext.onepass_lse_float_robust(xd)
        gx_d = ext.onepass_lse_float_backward(g.cuda(), xd, lse_d)
        assert torch.equal(lse_h, lse_d.cpu()), f"lse differs (call {call})"
        assert torch.equal(gx_h, gx_d.cpu()), f"grad differs (call {call})"


def test_forward_only_and_checks():
    from fuselse_b200.host import HostRowPipeline, logsumexp_fwd_bwd_host
    pipe = HostRowPipeline(100, chunk_rows=16)
    x = _pinned(torch.randn(50, 100))
    lse = _pinned(torch.empty(50))
    pipe.run(x, lse)
    torch.cuda.synchronize()
    torch.testing.assert_close(lse, torch.logsumexp(x, -1), rtol=1e-5, atol=1e-5)
    with pytest.raises(RuntimeError, match="pinned"):
        pipe.run(torch.randn(50, 100), lse)
    with pytest.raises(RuntimeError, match="go together"):
        pipe.run(x, lse, g_host=_pinned(torch.ones(50)))
    lse2, gx2 = logsumexp_fwd_bwd_host(x, _pinned(torch.ones(50)), chunk_rows=16)
    torch.testing.assert_close(gx2, torch.softmax(x, -1), rtol=1e-5, atol=1e-6)
