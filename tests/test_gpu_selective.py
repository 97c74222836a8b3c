"""GPU parity of the fused selective log-softmax (target gather + LSE, and its backward).

Checked against the fp64 oracle (oracle.selective_f64 / selective_bwd_f64) on the
same inputs, and against the caller's own algorithm (trl's selective_log_softmax,
restated with torch ops in fuselse_b200.selective.torch_selective_log_softmax)
run with torch on the GPU, for values and for gradients through autograd.

Tolerance: the log-probability inherits the LSE's error, so |logp - want| is
held to 1e-5 x max(|lse|, 1) (fp32 and fp16 input, both computed in fp32);
gradients given the same lse to 1e-6 absolute + 1e-5 relative; gradients
compared with torch's (computed from torch's lse) to a relative 1e-5 x
max(|lse|, 1), the forward's bound, since d(softmax)/softmax = -d(lse).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _randn(B, N, seed=0, scale=1.0, dev="cuda"):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(B, N, generator=g, device=dev) * scale


def _targets(B, N, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    t = torch.randint(0, max(N, 1), (B,), generator=g)
    if B >= 3 and N >= 2:
        t[0], t[1], t[2] = 0, N - 1, N // 2  # head, tail and middle columns
    return t.cuda()


def _check_logp(got_logp, got_lse, want_logp, want_lse, what):
    got_logp, got_lse = np.asarray(got_logp, np.float64), np.asarray(got_lse, np.float64)
    scale = np.maximum(np.abs(np.where(np.isfinite(want_lse), want_lse, 0.0)), 1.0)
    for got, want, name in ((got_logp, want_logp, "logp"), (got_lse, want_lse, "lse")):
        fin = np.isfinite(want)
        same = (np.isnan(got) & np.isnan(want)) | (got == want)
        assert np.all(same | fin), f"{what} {name}: special values differ"
        if fin.any():
            err = np.abs(got[fin] - want[fin]) / scale[fin]
            assert np.isfinite(got[fin]).all() and err.max() <= RTOL, \
                f"{what} {name}: max err {err.max():.3g}"


SHAPES = [(1, 1), (3, 2), (7, 3), (5, 5), (512, 256), (33, 1023), (9, 4096), (5, 4097),
          (2400, 3000), (4, 16385), (3, 65537), (64, 128256)]


@pytest.mark.parametrize("B,N", SHAPES)
def test_fwd_f32_vs_oracle(ext, B, N):
    x = _randn(B, N, seed=B * 7 + N, scale=2.0)
    t = _targets(B, N, seed=B + N)
    logp, lse = ext.selective_logsoftmax_rows(x, t)
    want_logp, want_lse = O.selective_f64(x.cpu().numpy(), t.cpu().numpy())
    _check_logp(logp.cpu().numpy(), lse.cpu().numpy(), want_logp, want_lse, f"{B}x{N}")


@pytest.mark.parametrize("phase", [1, 2, 3])
def test_fwd_f32_misaligned_rows(ext, phase):
    B, N = 6, 1001
    buf = _randn(1, B * N + 4, seed=phase).reshape(-1)
    x = buf[phase:phase + B * N].view(B, N)
    t = _targets(B, N, seed=phase)
    logp, lse = ext.selective_logsoftmax_rows(x, t)
    want_logp, want_lse = O.selective_f64(x.cpu().numpy(), t.cpu().numpy())
    _check_logp(logp.cpu().numpy(), lse.cpu().numpy(), want_logp, want_lse, f"phase {phase}")


def test_fwd_robust_rows(ext):
    from fuselse_b200 import workloads as W
    x = W.robust_rows(8, 777, seed=3)
    t = _targets(8, 777, seed=4)
    logp, lse = ext.selective_logsoftmax_rows(x, t, robust=True)
    want_logp, want_lse = O.selective_f64(x.cpu().numpy(), t.cpu().numpy())
    _check_logp(logp.cpu().numpy(), lse.cpu().numpy(), want_logp, want_lse, "robust")


@pytest.mark.parametrize("B,N", [(8192, 16032), (16, 50257), (3, 7)])
def test_fwd_f16_vs_oracle(ext, B, N):
    from fuselse_b200 import workloads as W
    x = W.fp16_logits(B, N, seed=5)
    t = _targets(B, N, seed=6)
    logp, lse = ext.selective_logsoftmax_rows(x, t)
    want_logp, want_lse = O.selective_f64(x.float().cpu().numpy(), t.cpu().numpy())
    _check_logp(logp.cpu().numpy(), lse.cpu().numpy(), want_logp, want_lse, f"f16 {B}x{N}")


def test_bad_index_gives_nan_and_flag(ext):
    B, N = 40, 5000
    x = _randn(B, N, seed=11)
    t = _targets(B, N, seed=12)
    t[5], t[17], t[30] = -1, N, 1 << 40
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    logp, lse = ext.selective_logsoftmax_rows(x, t, err_flag=err)
    assert int(err.item()) == 1
    got = logp.cpu().numpy()
    assert np.isnan(got[[5, 17, 30]]).all()
    want_logp, want_lse = O.selective_f64(x.cpu().numpy(), t.cpu().numpy())
    _check_logp(got, lse.cpu().numpy(), want_logp, want_lse, "bad index rows")
    # a clean call leaves a zeroed flag alone
    err.zero_()
    ext.selective_logsoftmax_rows(x, _targets(B, N, seed=13), err_flag=err)
    assert int(err.item()) == 0


def test_check_index_raises():
    import fuselse_b200
    x = _randn(4, 100, seed=1)
    t = torch.tensor([0, 5, 100, 2], device="cuda")
    with pytest.raises(RuntimeError, match="out of range"):
        fuselse_b200.selective_log_softmax(x, t, check_index=True)


@pytest.mark.parametrize("B,N", [(3, 2), (7, 1003), (512, 256), (2400, 3000), (64, 128256)])
def test_bwd_vs_oracle(ext, B, N):
    x = _randn(B, N, seed=B + 3 * N, scale=2.0)
    t = _targets(B, N, seed=N)
    g = _randn(1, B, seed=99).reshape(-1).contiguous()
    _, lse = ext.selective_logsoftmax_rows(x, t)
    gx = ext.selective_logsoftmax_backward(g, x, lse, t).cpu().numpy().astype(np.float64)
    want = O.selective_bwd_f64(g.cpu().numpy(), x.cpu().numpy(), lse.cpu().numpy(), t.cpu().numpy())
    np.testing.assert_allclose(gx, want, rtol=1e-5, atol=1e-6)


def test_bwd_misaligned_and_bad_index(ext):
    B, N = 5, 999
    buf = _randn(1, 2 * B * N + 8, seed=21).reshape(-1)
    x = buf[1:1 + B * N].view(B, N)
    t = _targets(B, N, seed=22)
    t[3] = N + 5  # no one-hot term for this row
    g = torch.ones(B, device="cuda")
    _, lse = ext.selective_logsoftmax_rows(x, t)
    want = O.selective_bwd_f64(g.cpu().numpy(), x.cpu().numpy(), lse.cpu().numpy(), t.cpu().numpy())
    # same-phase (vector) and differing-phase (scalar) output buffers
    for out_off in (0, 1):
        gx = ext.selective_logsoftmax_backward(g, x, lse, t) if out_off == 0 else None
        if gx is None:
            from fuselse_b200 import _lib
            import ctypes
            gbuf = torch.empty(B * N + 4, device="cuda")
            gx = gbuf[2:2 + B * N].view(B, N)
            _lib.call("fl_selective_logsoftmax_bwd", _lib.ptr(g), _lib.ptr(x), _lib.ptr(lse),
                      _lib.ptr(t, ctypes.c_int64), _lib.ptr(gx), B, N,
                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        np.testing.assert_allclose(gx.cpu().numpy(), want, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("shape", [(2, 37, 5000), (3, 17, 128256), (4, 1, 9)])
def test_autograd_vs_trl_restatement(shape):
    import fuselse_b200
    from fuselse_b200.selective import torch_selective_log_softmax
    *lead, V = shape
    x0 = _randn(int(np.prod(lead)), V, seed=V, scale=3.0).reshape(shape)
    g = torch.Generator(device="cpu").manual_seed(V)
    idx = torch.randint(0, V, tuple(lead), generator=g).cuda()
    up = _randn(1, int(np.prod(lead)), seed=5).reshape(tuple(lead))

    x1 = x0.clone().requires_grad_()
    y1 = fuselse_b200.selective_log_softmax(x1, idx)
    (y1 * up).sum().backward()

    x2 = x0.clone().requires_grad_()
    y2 = torch_selective_log_softmax(x2, idx)
    (y2 * up).sum().backward()

    assert y1.shape == y2.shape == idx.shape and y1.dtype == torch.float32
    lse = torch.logsumexp(x0, -1).abs().clamp_min(1.0)
    assert ((y1 - y2).abs() / lse).max().item() <= RTOL
    torch.testing.assert_close(x1.grad, x2.grad, rtol=RTOL * lse.max().item(), atol=1e-6)


def test_f16_result_dtype_and_value():
    import fuselse_b200
    from fuselse_b200.selective import torch_selective_log_softmax
    x = (_randn(2 * 50, 3000, seed=8, scale=3.0)).half().reshape(2, 50, 3000)
    idx = torch.randint(0, 3000, (2, 50), device="cuda")
    y = fuselse_b200.selective_log_softmax(x, idx)
    want = torch_selective_log_softmax(x, idx)  # trl's 16-bit path: log_softmax per sequence
    assert y.dtype == torch.float16 and y.shape == (2, 50)
    torch.testing.assert_close(y.float(), want.float(), rtol=2e-3, atol=2e-3)


@pytest.mark.slow
def test_full_rlhf_llama3_shape(ext):
    """(4, 1023, 128256): vs torch on the GPU, and size-independent properties:
    logp <= 0, and each gradient row sums to g * (1 - sum softmax) = 0."""
    from fuselse_b200.selective import torch_selective_log_softmax
    R, V = 4 * 1023, 128256
    x = _randn(R, V, seed=42)
    t = _targets(R, V, seed=43)
    logp, lse = ext.selective_logsoftmax_rows(x, t)
    want = torch_selective_log_softmax(x.view(4, 1023, V), t.view(4, 1023)).reshape(-1)
    assert (logp <= 0).all()
    assert ((logp - want).abs() / lse.abs().clamp_min(1)).max().item() <= RTOL
    gx = ext.selective_logsoftmax_backward(torch.ones(R, device="cuda"), x, lse, t)
    assert gx.double().sum(dim=1).abs().max().item() <= 1e-4
    del gx


@pytest.mark.parametrize("shape", [(2, 300, 32000), (1, 129, 50257)])
def test_vs_reference_rlhf_composition(shape):
    """Against the reference's own path for this caller: trl's gather minus
    the reference kernel onepass_lse_float (built from
    fuselse/gpu/fused_fp32_kernel.cu) per sequence, as run_rlhf.py:145-157
    runs it with torch.logsumexp routed to that kernel."""
    import fuselse_b200
    from tests.conftest import ref_ext_or_skip
    ref = ref_ext_or_skip("ref_fused_fp32")
    B, T, V = shape
    g = torch.Generator(device="cuda").manual_seed(V + T)
    logits = torch.randn(B, T, V, generator=g, device="cuda") * 2
    idx = torch.randint(0, V, (B, T), generator=g, device="cuda")
    want = (torch.gather(logits, -1, idx.unsqueeze(-1)).squeeze(-1)
            - torch.stack([ref.onepass_lse_float(seq) for seq in logits]))
    got = fuselse_b200.selective_log_softmax(logits, idx, robust=False)
    scale = torch.logsumexp(logits, -1).abs().clamp_min(1.0)
    assert ((got - want).abs() / scale).max().item() <= RTOL
