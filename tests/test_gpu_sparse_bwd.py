"""GPU parity of the sparse sum-layer backward (fl_sparse_f32_bwd) and its
autograd form (fuselse_b200.pc.sparse_sum_layer).

References: the fp64 gradient oracle (oracle.sparse_bwd_f64) on the same
inputs, given the kernel's own forward output; and torch autograd through the
torch restatement of the layer (run_pyjuice.py:90-119 with the kernels'
1e-45 weight floor) on the GPU.  Tolerance: 1e-5 relative + 1e-6 x the
largest gradient magnitude (the gradients are sums of up to E * block_size
positive-weighted terms, or of the batch for parameters).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_gpu_sparse import layer, to_dev

pytestmark = pytest.mark.gpu


def _close(got, want, what):
    got = np.asarray(got, np.float64)
    scale = max(np.abs(want).max(), 1e-30)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6 * scale, err_msg=what)


# (E, batch, block_size): vector (batch % 4 == 0) and scalar column paths,
# partial column groups, block_size > 1, E not a multiple of the edge step,
# more than 32 edges and (E=64, 300 children) more than 32 parents per child
CASES = [(1, 1, 1), (5, 3, 2), (8, 64, 1), (17, 100, 3), (32, 130, 1), (33, 512, 1), (64, 1000, 2)]


@pytest.mark.parametrize("fold", [True, False], ids=["fold", "nofold"])
@pytest.mark.parametrize("E,batch,bs", CASES)
def test_sparse_bwd_vs_oracle(ext, E, batch, bs, fold):
    node, em, params, nids, cids, pids = layer(E * 77 + batch, 300, 40, E, batch, bs,
                                               zero_w=0.02, neg_inf=0.02)
    node_d, em_d, w_d, nids_d, cids_d, pids_d = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(node_d, em_d, w_d, nids_d, cids_d, pids_d, bs)
    rng = np.random.default_rng(batch)
    G = rng.standard_normal(node.shape).astype(np.float32)
    G[rng.random(node.shape) < 0.05] = 0.0  # zero upstream gradients fold to +inf rows
    G_d = torch.from_numpy(G).cuda()
    gem = torch.zeros_like(em_d)
    gw = torch.zeros_like(w_d)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ext.sparse_backward_float(node_d, G_d, em_d, w_d, nids_d, cids_d, pids_d, bs,
                              element_grads=gem, param_grads=gw, err_flag=err, fold=fold)
    assert int(err.item()) == 0
    want_em, want_w = O.sparse_bwd_f64(node_d.cpu().numpy(), G, em, params, nids, cids, pids, bs)
    _close(gem.cpu().numpy(), want_em, f"element grads E={E} batch={batch} bs={bs}")
    _close(gw.cpu().numpy(), want_w, f"param grads E={E} batch={batch} bs={bs}")


@pytest.mark.parametrize("fold", [True, False], ids=["fold", "nofold"])
def test_sparse_bwd_wide_range(ext, fold):
    """Upstream gradients of both signs over 1e-20 .. 1e3 and weights scaled
    down to 1e-30: the folded rows' exponent bias keeps every term in range."""
    node, em, params, nids, cids, pids = layer(21, 500, 64, 24, 192, 1)
    rng = np.random.default_rng(22)
    params = (params * 10.0 ** rng.uniform(-30, 0, params.shape)).astype(np.float32)
    t = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(*t, 1)
    G = (np.sign(rng.standard_normal(node.shape)) * 10.0 ** rng.uniform(-20, 3, node.shape)).astype(np.float32)
    gem = torch.zeros_like(t[1])
    gw = torch.zeros_like(t[2])
    ext.sparse_backward_float(t[0], torch.from_numpy(G).cuda(), *t[1:], 1, element_grads=gem,
                              param_grads=gw, fold=fold)
    want_em, want_w = O.sparse_bwd_f64(t[0].cpu().numpy(), G, em, params, nids, cids, pids, 1)
    _close(gem.cpu().numpy(), want_em, "element grads, wide range")
    _close(gw.cpu().numpy(), want_w, "param grads, wide range")


def test_sparse_bwd_fold_workspace(ext):
    """A caller-owned workspace (reused across calls, larger than needed)
    gives the same element gradients as one allocated per call; one that is
    too small is refused."""
    node, em, params, nids, cids, pids = layer(13, 400, 50, 16, 96, 2)
    t = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(*t, 2)
    G = torch.randn_like(t[0])
    need = ext.sparse_bwd_workspace_bytes(*t[0].shape, t[4].numel() * 2)
    ws = torch.full((need + 4096,), 0xFF, dtype=torch.uint8, device="cuda")  # NaN-filled rows
    outs = []
    for w in (None, ws, ws):
        gem = torch.zeros_like(t[1])
        ext.sparse_backward_float(t[0], G, *t[1:], 2, element_grads=gem, workspace=w)
        outs.append(gem)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    with pytest.raises(RuntimeError, match="workspace"):
        ext.sparse_backward_float(t[0], G, *t[1:], 2, element_grads=torch.zeros_like(t[1]),
                                  workspace=ws[:need - 1])


def test_sparse_bwd_accumulates_and_skips(ext):
    node, em, params, nids, cids, pids = layer(5, 200, 30, 16, 64, 1)
    t = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(*t, 1)
    G = torch.ones_like(t[0])
    gem = torch.full_like(t[1], 0.5)
    ext.sparse_backward_float(t[0], G, t[1], t[2], t[3], t[4], t[5], 1, element_grads=gem)
    want_em, want_w = O.sparse_bwd_f64(t[0].cpu().numpy(), G.cpu().numpy(), em, params, nids,
                                       cids, pids, 1)
    _close(gem.cpu().numpy() - 0.5, want_em, "accumulated element grads")
    gw = torch.zeros_like(t[2])
    ext.sparse_backward_float(t[0], G, t[1], t[2], t[3], t[4], t[5], 1, param_grads=gw)
    _close(gw.cpu().numpy(), want_w, "param grads alone")


def test_sparse_bwd_bad_indices_set_flag(ext):
    node, em, params, nids, cids, pids = layer(9, 100, 10, 8, 32, 1)
    t = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(*t, 1)
    parents = ext.sparse_parent_index(t[3], t[4], t[5], 1, 100)
    cids_bad = t[4].clone()
    cids_bad[3, 2] = 100  # == num_elements
    for ci, pr in ((cids_bad, parents), (t[4], (parents[0], parents[1] + 10 ** 6, parents[2]))):
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        gem = torch.zeros_like(t[1])
        gw = torch.zeros_like(t[2])
        ext.sparse_backward_float(t[0], torch.ones_like(t[0]), t[1], t[2], t[3], ci, t[5], 1,
                                  element_grads=gem, param_grads=gw, parents=pr, err_flag=err)
        assert int(err.item()) == 1
        assert torch.isfinite(gem).all() and torch.isfinite(gw).all()


def test_sparse_bwd_index_built_from_bad_child(ext):
    """An edge whose child is out of range, in the parent index too: the index
    leaves it out of every child's range; both paths skip it, flag it and agree,
    whatever the workspace held before."""
    node, em, params, nids, cids, pids = layer(31, 100, 12, 8, 64, 1)
    t = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(*t, 1)
    cids_bad = t[4].clone()
    cids_bad[2, 5] = 100  # == num_elements
    parents = ext.sparse_parent_index(t[3], cids_bad, t[5], 1, 100)
    G = torch.randn_like(t[0])
    outs = []
    for fold in (True, False):
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        ws = None
        if fold:  # 0x7f bytes: every float slot reads 3.4e38 unless written
            ws = torch.full((ext.sparse_bwd_workspace_bytes(*t[0].shape, parents[1].numel()),), 0x7F,
                            dtype=torch.uint8, device="cuda")
        gem, gw = torch.zeros_like(t[1]), torch.zeros_like(t[2])
        ext.sparse_backward_float(t[0], G, t[1], t[2], t[3], cids_bad, t[5], 1, element_grads=gem,
                                  param_grads=gw, parents=parents, err_flag=err, fold=fold, workspace=ws)
        assert int(err.item()) == 1
        assert torch.isfinite(gem).all() and torch.isfinite(gw).all()
        outs.append((gem, gw))
    for a, b in zip(*outs):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6 * max(b.abs().max().item(), 1e-30))


def _torch_layer(node_mars, em, params, nids, cids, pids, bs):
    """The reference experiment's torch restatement (run_pyjuice.py:90-119),
    with the kernels' 1e-45 floor, as a differentiable function."""
    K, E = cids.shape
    n = (nids[:, None] + torch.arange(bs, device=nids.device)[None, :]).reshape(-1)
    c = cids[:, None, :].expand(K, bs, E).reshape(K * bs, E)
    q = (pids[:, None, :] + torch.arange(bs, device=pids.device)[None, :, None]).reshape(K * bs, E)
    lw = params[q].clamp(min=1e-45).log().unsqueeze(-1)
    out = node_mars.clone()
    out[n] = torch.logsumexp(em[c] + lw, dim=1)
    return out


@pytest.mark.parametrize("E,batch,bs", [(8, 64, 1), (16, 100, 2), (32, 512, 1)])
def test_autograd_layer_vs_torch(E, batch, bs):
    from fuselse_b200.pc import sparse_sum_layer
    node, em, params, nids, cids, pids = layer(E + batch, 500, 60, E, batch, bs)
    node_d, em_d, w_d, nids_d, cids_d, pids_d = to_dev(node, em, params, nids, cids, pids)
    up = torch.randn(node.shape, device="cuda")
    leaves1 = [t.clone().requires_grad_() for t in (node_d, em_d, w_d)]
    out1 = sparse_sum_layer(*leaves1, nids_d, cids_d, pids_d, bs)
    (out1 * up).sum().backward()
    leaves2 = [t.clone().requires_grad_() for t in (node_d, em_d, w_d)]
    out2 = _torch_layer(*leaves2, nids_d, cids_d, pids_d, bs)
    (out2 * up).sum().backward()
    torch.testing.assert_close(out1, out2, rtol=1e-5, atol=1e-5)
    for a, b, name in zip(leaves1, leaves2, ("node_mars", "element_mars", "params")):
        scale = b.grad.abs().max().item()
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-4, atol=1e-5 * max(scale, 1e-30),
                                   msg=lambda m: f"{name}: {m}")


def test_pyjuice_style_dispatcher():
    """The hook has the reference experiment's call shape (run_pyjuice.py:63-77)."""
    from fuselse_b200.pc import make_sparse_dispatcher

    class FakeSumLayer:
        block_size = 2
        _forward_sparse = make_sparse_dispatcher()

    node, em, params, nids, cids, pids = layer(3, 100, 12, 8, 16, 2)
    t = to_dev(node, em, params, nids, cids, pids)
    local = torch.tensor([1, 4, 7], device="cuda")
    FakeSumLayer()._forward_sparse(t[0], t[1], t[2], t[3], t[4], t[5], local_ids=local)
    want = O.sparse_f64(node, em, params, nids[[1, 4, 7]], cids[[1, 4, 7]], pids[[1, 4, 7]], 2)
    np.testing.assert_allclose(t[0].cpu().numpy(), want, rtol=1e-5, atol=1e-5)
