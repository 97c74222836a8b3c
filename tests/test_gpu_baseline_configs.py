"""GPU parity at the benchmark configurations themselves (not only at smaller
shapes that take another launch shape).

* FuseLSE fp32 forward + backward at (512, 128256) — one 256-thread CTA per
  row, the shape the headline number is quoted on — plain and robust, against
  the reference kernels (fuselse/gpu/fused_fp32_kernel.cu:50-150, built from
  source into oracle/_ref) and the fp64 oracle.
* The robust-mode variant of that configuration at (512, 128256) and
  (512, 256): 1 % of entries -inf (seed 1), row 0 all -inf, row 1 one +inf and
  one NaN (fuselse_b200.workloads.robust_rows).
* FuseLSE16 over the full (8192, 128256) fp16 logits against the reference
  fp16 kernel (fused_fp16_kernel.cu:25-132) at 2e-3 and the fp64 oracle at
  1e-5, and the same logits split into 8 contiguous vocab shards of 16032
  (partial states per shard, then the combine) on one GPU.
* The vocab-sharded forward + backward (VocabShardedLogSumExp) through the
  single-rank NVLink exchange, against the fp64 value and gradient.

Tolerances: fp32 1e-5 relative (relative to max(|v|, 1) for lse values, to |v|
for gradients, as in tests/test_gpu_lse.py); fp16 input 2e-3 against the
reference fp16 kernel.
"""
import numpy as np
import pytest
import torch

from fuselse_b200 import workloads as W
from oracle import oracle as O
from tests.conftest import ref_ext_or_skip

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

RTOL32 = 1e-5
TOL16 = 2e-3
HEAD_B, HEAD_N = 512, 128256


def _close(got, want, tol, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    same_special = (np.isnan(got) & np.isnan(want)) | ((got == want) & ~np.isfinite(want))
    fin = np.isfinite(want)
    bad = ~(same_special | fin)
    assert not bad.any(), f"{what}: special values differ at rows {np.nonzero(bad)[0][:8]}"
    if fin.any():
        assert np.all(np.isfinite(got[fin])), f"{what}: non-finite where the oracle is finite"
        err = np.abs(got[fin] - want[fin]) / np.maximum(np.abs(want[fin]), 1.0)
        assert err.max() <= tol, f"{what}: max rel err {err.max():.3g} > {tol}"


def _grad_close(got, want, tol, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    nan_w = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan_w), f"{what}: NaN pattern differs"
    g, w = got[~nan_w], want[~nan_w]
    err = np.abs(g - w) / np.maximum(np.abs(w), 1e-30)
    assert err.max() <= tol, f"{what}: max rel err {err.max():.3g} > {tol}"


@pytest.fixture(scope="module")
def headline_x():
    return W.fp32_rows(HEAD_B, HEAD_N, seed=0, device="cuda")


@pytest.mark.parametrize("robust", [True, False])
def test_headline_fwd_bwd_vs_oracle(ext, headline_x, robust):
    x = headline_x
    fwd = ext.onepass_lse_float_robust if robust else ext.onepass_lse_float
    lse = fwd(x)
    g = torch.ones(HEAD_B, device="cuda")
    gx = ext.onepass_lse_float_backward(g, x, lse)
    xn = x.cpu().numpy()
    lse_n = lse.cpu().numpy()
    _close(lse_n, O.lse_f64(xn), RTOL32, "forward vs fp64")
    _grad_close(gx.cpu().numpy(), O.lse_bwd_f64(g.cpu().numpy(), xn, lse_n), RTOL32,
                "backward vs fp64")


def test_headline_fwd_bwd_vs_reference_kernel(ext, headline_x):
    ref = ref_ext_or_skip("ref_fused_fp32")
    x = headline_x
    _close(ext.onepass_lse_float_robust(x).cpu().numpy(),
           ref.onepass_lse_float_robust(x).cpu().numpy(), RTOL32, "robust forward")
    _close(ext.onepass_lse_float(x).cpu().numpy(),
           ref.onepass_lse_float(x).cpu().numpy(), RTOL32, "plain forward")
    g = torch.rand(HEAD_B, generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
    lse = ref.onepass_lse_float_robust(x)  # the same lse into both backwards
    _grad_close(ext.onepass_lse_float_backward(g, x, lse).cpu().numpy(),
                ref.onepass_lse_float_backward(g, x, lse).cpu().numpy(), RTOL32, "backward")


@pytest.mark.parametrize("N", [HEAD_N, 256])
def test_robust_config_ieee_rows(ext, N):
    x = W.robust_rows(HEAD_B, N, seed=0, device="cuda")
    lse = ext.onepass_lse_float_robust(x)
    got = lse.cpu().numpy()
    assert got[0] == -np.inf, "all -inf row"
    assert np.isnan(got[1]), "+inf with NaN row"
    xn = x.cpu().numpy()
    _close(got, O.lse_f64(xn), RTOL32, f"robust rows N={N}")
    g = torch.ones(HEAD_B, device="cuda")
    gx = ext.onepass_lse_float_backward(g, x, lse).cpu().numpy()
    want = O.lse_bwd_f64(g.cpu().numpy(), xn, got)
    # the -inf entries of finite rows get exactly zero gradient
    fin_rows = np.isfinite(got)
    assert np.all(gx[fin_rows][np.isneginf(xn[fin_rows])] == 0.0)
    _grad_close(gx, want, RTOL32, f"robust backward N={N}")
    ref = ref_ext_or_skip("ref_fused_fp32")
    r = ref.onepass_lse_float_robust(x).cpu().numpy()
    assert r[0] == -np.inf and np.isnan(r[1])
    _close(got, r, RTOL32, f"robust vs reference N={N}")
    rgx = ref.onepass_lse_float_backward(g, x, lse).cpu().numpy()
    _grad_close(gx[2:], rgx[2:], RTOL32, f"robust backward vs reference N={N}")


@pytest.fixture(scope="module")
def llm_logits():
    return W.fp16_logits(8192, 128256, seed=0, device="cuda")


@pytest.fixture(scope="module")
def llm_lse_f64(llm_logits):
    rows = 1024
    return np.concatenate([O.lse_f64(llm_logits[i:i + rows].float().cpu().numpy())
                           for i in range(0, llm_logits.size(0), rows)])


def test_f16_full_config_vs_reference_and_oracle(ext, llm_logits, llm_lse_f64):
    xh = llm_logits
    got = ext.batched_logsumexp_fp16(xh).cpu().numpy()
    _close(got, llm_lse_f64, RTOL32, "fp16 (8192, 128256) vs fp64")
    ref = ref_ext_or_skip("ref_fused_fp16")
    _close(got, ref.batched_logsumexp_fp16(xh).cpu().numpy(), TOL16, "fp16 vs reference kernel")


def test_f16_full_config_eight_vocab_shards(ext, llm_logits, llm_lse_f64):
    xh = llm_logits
    parts = [ext.lse_partial(W.vocab_shard(xh, 8, i)) for i in range(8)]
    assert all(p.shape == (8192, 2) for p in parts)
    got = ext.lse_combine(torch.stack(parts)).cpu().numpy()
    _close(got, llm_lse_f64, RTOL32, "8 shards of 16032 + combine vs fp64")


def test_vocab_sharded_fwd_bwd_single_rank():
    from fuselse_b200.distributed import VocabShardExchange, vocab_sharded_logsumexp_grad
    B, N = 2048, 16032
    gen = torch.Generator(device="cuda").manual_seed(21)
    x = (torch.randn(B, N, generator=gen, device="cuda") * 3.0)
    x[7] = float("-inf")
    x[9, :4000] = float("-inf")
    ex = VocabShardExchange.single_rank(B)
    xs = x.clone().requires_grad_()
    lse = vocab_sharded_logsumexp_grad(xs, ex)
    w = torch.rand(B, generator=gen, device="cuda")
    (lse * w).sum().backward()
    xn = x.cpu().numpy()
    lse_n = lse.detach().cpu().numpy()
    _close(lse_n, O.lse_f64(xn), RTOL32, "vocab-sharded forward")
    assert lse_n[7] == -np.inf
    want = O.lse_bwd_f64(w.cpu().numpy(), xn, lse_n)
    got = xs.grad.cpu().numpy()
    rows = np.isfinite(lse_n)
    _grad_close(got[rows], want[rows], RTOL32, "vocab-sharded backward")
    assert not ex.error()
