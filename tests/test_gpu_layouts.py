"""GPU parity of the in-place layouts: strided rows (e.g. logits[:, :-1, :]) and
reductions over a dim other than the last, forward and backward, against the
fp64 oracle and torch autograd.  Same tolerances as the row kernels: 1e-5
relative to max(|lse|, 1) for values, 1e-5 rel + 1e-6 abs for gradients given
the same lse.  Gradients compared with torch's own (which uses torch's lse)
carry the forward's error too: d(exp(x - lse)) / exp(x - lse) = -d(lse), so
their relative tolerance is the forward bound 1e-5 x max(|lse|, 1)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _randn(*shape, seed=0, scale=2.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, generator=g, device="cuda") * scale


def _close_lse(got, want, what):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    fin = np.isfinite(want)
    assert np.all((np.isnan(got) & np.isnan(want)) | (got == want) | fin), f"{what}: specials"
    if fin.any():
        err = np.abs(got[fin] - want[fin]) / np.maximum(np.abs(want[fin]), 1.0)
        assert err.max() <= RTOL, f"{what}: max err {err.max():.3g}"


def _grad_close(got, want, lse):
    rtol = RTOL * max(1.0, lse.abs().max().item())
    torch.testing.assert_close(got, want, rtol=rtol, atol=1e-6)


def _views():
    base = _randn(3, 18, 1001, seed=1)
    big = _randn(4, 9, 4096 + 3, seed=2)
    return {
        "slice_T": base[:, :-1, :],           # two stride levels, V odd: row phases vary
        "slice_T_aligned": _randn(2, 33, 4096, seed=3)[:, 1:, :],
        "every_other_row": _randn(64, 777, seed=4)[::2],
        "column_window": big[:, :, 3:],         # rows start mid-vector
        "narrow_rows": _randn(50, 300, seed=5)[:, 10:260],
    }


VIEW_NAMES = ["slice_T", "slice_T_aligned", "every_other_row", "column_window", "narrow_rows"]


@pytest.mark.parametrize("name", VIEW_NAMES)
def test_strided_forward_and_backward(ext, name):
    x = _views()[name]
    assert not x.is_contiguous() and ext.row_layout(x) is not None
    lse = ext.onepass_lse_float_strided(x)
    dense = x.contiguous().cpu().numpy()
    want = O.lse_f64(dense)
    _close_lse(lse.cpu().numpy(), want, name)
    g = _randn(*x.shape[:-1], seed=9, scale=1.0)
    gx = ext.onepass_lse_float_backward_strided(g, x, lse)
    want_gx = O.lse_bwd_f64(g.reshape(-1).cpu().numpy(), dense.reshape(-1, x.shape[-1]),
                            lse.reshape(-1).cpu().numpy())
    np.testing.assert_allclose(gx.reshape(-1, x.shape[-1]).cpu().numpy(), want_gx,
                               rtol=1e-5, atol=1e-6)


def test_row_layout_rejects_three_levels(ext):
    x = _randn(4, 5, 6, 7, seed=1)[:, ::2, ::2, :]
    assert ext.row_layout(x) is None


def test_autograd_strided_input_matches_torch():
    import fuselse_b200
    lse_fn = fuselse_b200.make_fuselse_logsumexp()
    base = _randn(2, 65, 5003, seed=11)
    x1 = base[:, :-1, :].detach().requires_grad_()  # leaf views: grads land on x1
    x1_view = x1
    y = lse_fn(x1_view, dim=-1)
    up = _randn(*y.shape, seed=12, scale=1.0)
    (y * up).sum().backward()
    x2 = base[:, :-1, :].detach().clone().requires_grad_()
    (torch.logsumexp(x2, -1) * up).sum().backward()
    _close_lse(y.detach().cpu().numpy(), torch.logsumexp(x2, -1).detach().cpu().numpy(), "autograd fwd")
    _grad_close(x1.grad, x2.grad, y.detach())


@pytest.mark.parametrize("shape,dim", [((5, 300, 7), 1), ((2000, 64), 0), ((3, 4, 50, 33), 2),
                                       ((1, 100000, 40), 1), ((6, 3, 1000), 1), ((129, 2), 0)])
def test_dim_forward_and_backward(ext, shape, dim):
    x = _randn(*shape, seed=sum(shape))
    if x.numel() > 10:
        x.view(-1)[7] = float("-inf")
    out = ext.logsumexp_dim(x, dim)
    want = O.lse_f64(np.moveaxis(x.cpu().numpy(), dim, -1))
    _close_lse(out.cpu().numpy(), want, f"{shape} dim {dim}")
    # backward against the fp64 formula given the same lse (the forward's own
    # error is covered above)
    g = _randn(*out.shape, seed=3, scale=1.0)
    gx = ext.logsumexp_dim_backward(g, x, out, dim)
    xm = np.moveaxis(x.cpu().numpy(), dim, -1)
    want_gx = O.lse_bwd_f64(g.reshape(-1).cpu().numpy(), xm.reshape(-1, xm.shape[-1]),
                            out.reshape(-1).cpu().numpy()).reshape(xm.shape)
    np.testing.assert_allclose(np.moveaxis(gx.cpu().numpy(), dim, -1), want_gx, rtol=1e-5, atol=1e-6)


def test_dim_robust_rows(ext):
    x = _randn(4, 500, 37, seed=21)
    x[1, :, 3] = float("-inf")     # an all -inf reduction
    x[2, 17, 5] = float("inf")
    x[3, 400, 36] = float("nan")
    out = ext.logsumexp_dim(x, 1).cpu().numpy()
    want = O.lse_f64(np.moveaxis(x.cpu().numpy(), 1, -1))
    _close_lse(out, want, "robust dim")
    assert out[1, 3] == -np.inf and out[2, 5] == np.inf and np.isnan(out[3, 36])


def test_autograd_dim_matches_torch():
    import fuselse_b200
    lse_fn = fuselse_b200.make_fuselse_logsumexp()
    x1 = _randn(8, 3000, 16, seed=31).requires_grad_()
    y = lse_fn(x1, dim=1, keepdim=True)
    assert y.shape == (8, 1, 16)
    up = _randn(*y.shape, seed=32, scale=1.0)
    (y * up).sum().backward()
    x2 = x1.detach().clone().requires_grad_()
    (torch.logsumexp(x2, 1, keepdim=True) * up).sum().backward()
    _grad_close(x1.grad, x2.grad, y.detach())


def test_selective_on_sliced_logits_matches_trl_restatement():
    import fuselse_b200
    from fuselse_b200.selective import torch_selective_log_softmax
    full = _randn(3, 41, 7001, seed=41)
    ids = torch.randint(0, 7001, (3, 41), device="cuda")
    x1 = full.detach().requires_grad_()
    logits = x1[:, :-1, :]            # the RLHF slice: strided rows, no copy
    idx = ids[:, 1:]
    y1 = fuselse_b200.selective_log_softmax(logits, idx)
    up = _randn(*y1.shape, seed=42, scale=1.0)
    (y1 * up).sum().backward()
    x2 = full.detach().clone().requires_grad_()
    y2 = torch_selective_log_softmax(x2[:, :-1, :], idx)
    (y2 * up).sum().backward()
    lse = torch.logsumexp(full[:, :-1, :], -1).abs().clamp_min(1.0)
    assert ((y1 - y2).abs() / lse).max().item() <= RTOL
    _grad_close(x1.grad, x2.grad, lse)
