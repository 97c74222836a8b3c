"""GPU parity of the sparse PC sum layer: fp32 within 1e-5 relative, Q16.16 bit for bit.

References: the fp64 restatement of run_pyjuice.py:90-119 (with the kernels'
1e-45 weight floor), the Q16.16 oracle replaying the reference chain order on
device-formed log-weights, and the reference kernels built from source.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.conftest import ref_ext_or_skip

pytestmark = pytest.mark.gpu


def layer(seed, P, K, E, batch, bs, zero_w=0.0, neg_inf=0.0):
    rng = np.random.default_rng(seed)
    em = (rng.standard_normal((P, batch)) * 5 - 20).astype(np.float32)
    if neg_inf:
        em[rng.random(em.shape) < neg_inf] = -np.inf
    num_nodes = K * bs + 5
    node = np.full((num_nodes, batch), 3.0, np.float32)
    nids = (np.arange(K) * bs + 5).astype(np.int64)
    cids = np.stack([rng.choice(P, size=E, replace=E > P) for _ in range(K)]).astype(np.int64)
    pids = (np.arange(K * E).reshape(K, E) * bs).astype(np.int64)
    params = rng.dirichlet(np.ones(max(E, 1)), size=K * bs).astype(np.float32).reshape(-1)
    params = np.ascontiguousarray(params[: max(K * E * bs, 1)])
    if zero_w:
        params[rng.random(params.shape) < zero_w] = 0.0
    return node, em, params, nids, cids, pids


def to_dev(*arrs):
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def logw_layout(ext, params, pids, bs):
    K, E = pids.shape
    idx = (pids[:, None, :] + np.arange(bs)[None, :, None]).reshape(K * bs, E)
    lw = ext.sparse_log_weights(torch.from_numpy(params).cuda()).cpu().numpy()
    return lw[idx] if E else np.zeros((K * bs, 0), np.float32)


CASES = [(E, batch, bs) for E in (1, 5, 8, 9, 16, 17, 32, 33, 64, 100)
         for batch, bs in ((1, 1), (3, 2), (4, 1), (64, 1), (100, 3), (130, 1))]


@pytest.mark.parametrize("E,batch,bs", CASES)
def test_sparse_q16_bitexact_vs_oracle(ext, E, batch, bs):
    node, em, params, nids, cids, pids = layer(E * 1000 + batch, 300, 40, E, batch, bs,
                                               zero_w=0.02, neg_inf=0.03)
    want = O.sparse_q16(node, em, logw_layout(ext, params, pids, bs), nids, cids, bs)
    t = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_q16(*t, bs)
    np.testing.assert_array_equal(t[0].cpu().numpy().view(np.int32), want.view(np.int32))


@pytest.mark.parametrize("E,batch,bs", CASES)
def test_sparse_f32_vs_fp64(ext, E, batch, bs):
    node, em, params, nids, cids, pids = layer(E * 1000 + batch + 1, 300, 40, E, batch, bs,
                                               neg_inf=0.03)
    want = O.sparse_f64(node, em, params, nids, cids, pids, bs)
    t = to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(*t, bs)
    got = t[0].cpu().numpy().astype(np.float64)
    fin = np.isfinite(want)
    # all-(-inf) children: the reference's -1e30 seed gives -1e30
    assert np.all(got[~fin] == np.float32(-1e30)) or np.all(got[~fin] == want[~fin])
    err = np.abs(got[fin] - want[fin]) / np.maximum(np.abs(want[fin]), 1.0)
    assert err.max() <= 1e-5, err.max()


@pytest.mark.parametrize("E,batch,bs", [(32, 64, 1), (9, 5, 2), (70, 33, 3), (17, 1, 1), (32, 130, 2)])
def test_sparse_vs_reference_kernels(ext, E, batch, bs):
    rq = ref_ext_or_skip("ref_sparse_q16")
    rf = ref_ext_or_skip("ref_sparse_float")
    node, em, params, nids, cids, pids = layer(E + batch, 500, 60, E, batch, bs, zero_w=0.02,
                                               neg_inf=0.02)
    a, b = to_dev(node, em, params, nids, cids, pids), to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_q16(*a, bs)
    rq.sparse_forward_q16(*b, bs)
    np.testing.assert_array_equal(a[0].cpu().numpy().view(np.int32), b[0].cpu().numpy().view(np.int32))
    a, b = to_dev(node, em, params, nids, cids, pids), to_dev(node, em, params, nids, cids, pids)
    ext.sparse_forward_float(*a, bs)
    rf.sparse_forward_float(*b, bs)
    x, y = a[0].cpu().numpy().astype(np.float64), b[0].cpu().numpy().astype(np.float64)
    fin = np.isfinite(y) & (y > -1e29)
    assert np.all((x > -1e29) == (y > -1e29))
    assert (np.abs(x[fin] - y[fin]) / np.maximum(np.abs(y[fin]), 1.0)).max() <= 1e-5


def test_sparse_bad_indices_flagged(ext):
    node, em, params, nids, cids, pids = layer(5, 100, 10, 8, 8, 1)
    cids[3, 2] = 10_000          # child out of range -> that node's row is NaN
    nids[4] = 10_000             # output row out of range -> write skipped
    t = to_dev(node, em, params, nids, cids, pids)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    ext._sparse("fl_sparse_f32", *t, 1, err_flag=flag)
    out = t[0].cpu().numpy()
    assert flag.item() == 1
    assert np.isnan(out[nids[3]]).all()
    assert np.isfinite(out[nids[5]]).all()


@pytest.mark.slow
def test_sparse_baseline_config_vs_reference(ext):
    """P=262144 product nodes, 65536 sum nodes x 32 children, batch 512."""
    rq = ref_ext_or_skip("ref_sparse_q16")
    rf = ref_ext_or_skip("ref_sparse_float")
    from fuselse_b200 import workloads as W
    _, em, params, nids, cids, pids, _ = W.sparse_layer()
    S, batch = cids.size(0), em.size(1)
    out_a = torch.zeros(S, batch, device="cuda")
    out_b = torch.zeros(S, batch, device="cuda")
    ext.sparse_forward_q16(out_a, em, params, nids, cids, pids, 1)
    for lo in range(0, S, 32768):  # the reference grid's y extent is capped at 65535
        hi = min(S, lo + 32768)
        rq.sparse_forward_q16(out_b, em, params, nids[lo:hi], cids[lo:hi], pids[lo:hi], 1)
    assert torch.equal(out_a.view(torch.int32), out_b.view(torch.int32))
    ext.sparse_forward_float(out_a, em, params, nids, cids, pids, 1)
    for lo in range(0, S, 32768):
        hi = min(S, lo + 32768)
        rf.sparse_forward_float(out_b, em, params, nids[lo:hi], cids[lo:hi], pids[lo:hi], 1)
    rel = ((out_a - out_b).abs() / out_b.abs().clamp_min(1.0)).max().item()
    assert rel <= 1e-5, rel
