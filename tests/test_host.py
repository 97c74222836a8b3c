"""CPU tests of the host layer: validation and error behaviour of the
reference-named entry points, the torch.logsumexp delegation rules of
make_fuselse_logsumexp, the partitioning helpers, and the selective
log-softmax oracle against the caller's algorithm (torch, CPU)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

import fuselse_b200
from fuselse_b200 import distributed as D
from fuselse_b200 import ext


def test_ext_exposes_reference_names():
    for name in ("onepass_lse_float", "onepass_lse_float_robust", "onepass_lse_float_backward",
                 "batched_logsumexp_fp16", "batched_logsumexp", "batched_logsumexp_nolut",
                 "batched_logsumexp_q10_6", "sparse_forward_float", "sparse_forward_q16"):
        assert callable(getattr(ext, name))


@pytest.mark.parametrize("fn,x,msg", [
    (ext.onepass_lse_float, torch.zeros(2, 3), "x must be CUDA"),
    (ext.onepass_lse_float_robust, torch.zeros(2, 3), "x must be CUDA"),
    (ext.batched_logsumexp_fp16, torch.zeros(2, 3), "Input must be CUDA fp16"),
    (ext.batched_logsumexp_fp16, torch.zeros(3), "Expected 2-D tensor (B, N)"),
    (ext.batched_logsumexp, torch.zeros(2, 3), "Expected input.is_cuda()"),
    (ext.batched_logsumexp_q10_6, torch.zeros(2, 3, dtype=torch.int16), "Input must be CUDA"),
    (ext.batched_logsumexp_q16_i32, torch.zeros(2, 3, dtype=torch.int32), "Input must be CUDA"),
])
def test_validation_matches_reference_checks(fn, x, msg):
    with pytest.raises(RuntimeError, match=msg.replace("(", r"\(").replace(")", r"\)")):
        fn(x)


def test_backward_validation():
    with pytest.raises(RuntimeError, match="grad_output must be CUDA"):
        ext.onepass_lse_float_backward(torch.zeros(2), torch.zeros(2, 3), torch.zeros(2))


def test_sparse_validation():
    z = torch.zeros(2, 2)
    with pytest.raises(RuntimeError, match="node_mars must be CUDA"):
        ext.sparse_forward_q16(z, z, torch.zeros(4), torch.zeros(1, dtype=torch.long),
                               torch.zeros(1, 2, dtype=torch.long), torch.zeros(1, 2, dtype=torch.long), 1)


def test_logsumexp_delegates_unsupported_inputs_to_torch():
    lse = fuselse_b200.make_fuselse_logsumexp(ext, robust=True)
    x = torch.randn(4, 7, 5, dtype=torch.float64)
    torch.testing.assert_close(lse(x, dim=-1), torch.logsumexp(x, dim=-1))       # CPU
    xf = x.float()
    torch.testing.assert_close(lse(xf, dim=1, keepdim=True), torch.logsumexp(xf, dim=1, keepdim=True))
    torch.testing.assert_close(lse(xf[..., :1], dim=-1), torch.logsumexp(xf[..., :1], dim=-1))
    g = xf.clone().requires_grad_()
    lse(g, dim=-1).sum().backward()
    torch.testing.assert_close(g.grad, torch.softmax(xf, -1))


def test_logsumexp_accepts_reference_style_extension_object():
    calls = []

    class Fake:
        @staticmethod
        def onepass_lse_float(x):
            calls.append("plain")
            return x.sum(-1)

        onepass_lse_float_robust = onepass_lse_float
        onepass_lse_float_backward = None

    lse = fuselse_b200.make_fuselse_logsumexp(Fake, robust=False)
    # CPU input is delegated, the fake is never called
    lse(torch.zeros(2, 3))
    assert calls == []


@pytest.mark.parametrize("n,parts", [(10, 3), (512, 8), (7, 8), (0, 2), (128256, 8)])
def test_split_range_partitions(n, parts):
    blocks = [D.split_range(n, parts, i) for i in range(parts)]
    assert blocks[0][0] == 0 and blocks[-1][1] == n
    for (a, b), (c, d) in zip(blocks, blocks[1:]):
        assert b == c and b >= a
    sizes = [b - a for a, b in blocks]
    assert max(sizes) - min(sizes) <= 1


def test_split_range_rejects_bad_index():
    with pytest.raises(ValueError):
        D.split_range(10, 2, 2)


# ---------------------------------------------------------------- selective log-softmax
def test_selective_oracle_matches_trl_restatement_cpu():
    from fuselse_b200.selective import torch_selective_log_softmax
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 11, 257, generator=g, dtype=torch.float64) * 4
    idx = torch.randint(0, 257, (3, 11), generator=g)
    want = torch_selective_log_softmax(x, idx).numpy()
    logp, lse = O.selective_f64(x.reshape(-1, 257).numpy(), idx.reshape(-1).numpy())
    np.testing.assert_allclose(logp.reshape(3, 11), want, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(lse, torch.logsumexp(x, -1).reshape(-1).numpy(), rtol=1e-12)


def test_selective_oracle_bad_index_is_nan():
    x = np.zeros((3, 4))
    logp, lse = O.selective_f64(x, np.array([0, 4, -1]))
    assert logp[0] == pytest.approx(-np.log(4)) and np.isnan(logp[1:]).all()


def test_selective_bwd_oracle_matches_autograd_cpu():
    from fuselse_b200.selective import torch_selective_log_softmax
    g = torch.Generator().manual_seed(1)
    x = (torch.randn(2, 5, 33, generator=g, dtype=torch.float64) * 3).requires_grad_()
    idx = torch.randint(0, 33, (2, 5), generator=g)
    up = torch.randn(2, 5, generator=g, dtype=torch.float64)
    (torch_selective_log_softmax(x, idx) * up).sum().backward()
    xf = x.detach().reshape(-1, 33).numpy()
    lse = O.lse_f64(xf)
    want = O.selective_bwd_f64(up.reshape(-1).numpy(), xf, lse, idx.reshape(-1).numpy())
    np.testing.assert_allclose(x.grad.reshape(-1, 33).numpy(), want, rtol=1e-12, atol=1e-14)


def test_selective_delegates_cpu_inputs_to_torch():
    import fuselse_b200
    from fuselse_b200.selective import torch_selective_log_softmax
    x = torch.randn(2, 6, 50)
    idx = torch.randint(0, 50, (2, 6))
    torch.testing.assert_close(fuselse_b200.selective_log_softmax(x, idx),
                               torch_selective_log_softmax(x, idx))


def test_selective_validation_without_gpu():
    from fuselse_b200 import ext
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.selective_logsoftmax_rows(torch.zeros(2, 3), torch.zeros(2, dtype=torch.int64))
    with pytest.raises(RuntimeError, match="contiguous 2D CUDA"):
        ext.selective_logsoftmax_backward(torch.zeros(2), torch.zeros(2, 3), torch.zeros(2),
                                          torch.zeros(2, dtype=torch.int64))


# ---------------------------------------------------------------- in-place row layouts
def test_row_layout_cases():
    x = torch.zeros(3, 18, 1001)
    assert ext.row_layout(x) == (54, 1001, 54, 0, 1001)                 # dense: one level
    assert ext.row_layout(x[:, :-1, :]) == (51, 1001, 17, 18 * 1001, 1001)
    assert ext.row_layout(x[::2]) == (36, 1001, 18, 2 * 18 * 1001, 1001)  # every other group
    assert ext.row_layout(x[:, ::2, :]) == (27, 1001, 27, 0, 2002)       # nests: one level
    assert ext.row_layout(x[:, :, 5:]) == (54, 996, 54, 0, 1001)
    assert ext.row_layout(torch.zeros(4, 5, 6, 7)[:, ::2, ::2, :]) is None  # three levels
    assert ext.row_layout(x.transpose(1, 2)) is None                      # last dim not unit-stride
    assert ext.row_layout(torch.zeros(1, 1, 9)) == (1, 9, -1, 0, 9)


# ---------------------------------------------------------------- sparse backward oracle
@pytest.mark.parametrize("tied", [False, True], ids=["untied", "tied"])
def test_sparse_bwd_oracle_matches_torch_autograd_cpu(tied):
    """The fp64 gradient oracle against torch autograd of the layer formula
    (run_pyjuice.py:90-119 with the 1e-45 floor), block_size 2, shared
    children and one weight below the floor; tied: several edges share a
    parameter, and one node's children are all -inf.  Such a node's
    node_mars is -inf and it passes no gradient (torch's logsumexp backward
    gives NaN there, which tied parameters would spread), so torch's graph is
    built over the live nodes only and compared with the oracle on the full
    layer."""
    rng = np.random.default_rng(0)
    P, K, E, batch, bs = 40, 6, 5, 7, 2
    em = rng.standard_normal((P, batch)) * 3 - 5
    nm0 = np.zeros((K * bs + 3, batch))
    nids = np.arange(K) * bs + 3
    cids = rng.integers(0, P - 1, size=(K, E))
    pids = np.arange(K * E).reshape(K, E) * bs
    params = rng.random(K * E * bs) + 0.05
    params[4] = 1e-50
    live = np.ones(K, bool)
    if tied:
        pids = pids % (3 * E * bs)   # nodes 3-5 reuse nodes 0-2's parameters
        cids[1] = P - 1              # node 1's children: all the -inf row
        em[P - 1] = -np.inf
        live[1] = False
    G = rng.standard_normal(nm0.shape)

    em_t = torch.tensor(em, requires_grad=True)
    w_t = torch.tensor(params, requires_grad=True)
    ar = np.arange(bs)
    n = (nids[:, None] + ar[None, :])                                   # (K, bs)
    c = np.repeat(cids[:, None, :], bs, axis=1)                         # (K, bs, E)
    q = pids[:, None, :] + ar[None, :, None]                            # (K, bs, E)
    out = torch.tensor(nm0).clone()
    nl, cl, ql = (torch.tensor(a[live].reshape(-1, *a.shape[2:])) for a in (n, c, q))
    out[nl] = torch.logsumexp(em_t[cl] + w_t[ql].clamp(min=1e-45).log().unsqueeze(-1), dim=1)
    nm = out.detach().numpy().copy()
    nm[n[~live].reshape(-1)] = -np.inf                                  # the dead node's forward value
    (out * torch.tensor(G)).sum().backward()
    gem, gw = O.sparse_bwd_f64(nm, G, em, params, nids, cids, pids, bs)
    np.testing.assert_allclose(gem, em_t.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(gw, w_t.grad.numpy(), rtol=1e-10, atol=1e-12)
    assert gw[4] == 0.0
    assert np.isfinite(gem).all() and np.isfinite(gw).all()
