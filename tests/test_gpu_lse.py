"""GPU parity of the FuseLSE path (fp32 fwd/bwd, fp16 fwd, shard partials).

Checked against (a) the fp64 oracle on the same inputs and (b) the reference
kernels themselves (built from the reference sources into oracle/_ref), when
present.  Tolerances (north star): fp32 within 1e-5 relative of the reference
fp32 path; fp16 input within 2e-3.  Relative error is measured against
max(|value|, 1) so rows whose log-sum-exp is near zero are held to 1e-5 absolute.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.conftest import ref_ext_or_skip

pytestmark = pytest.mark.gpu

RTOL32 = 1e-5
TOL16 = 2e-3


def _close(got, want, tol, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    same_special = (np.isnan(got) & np.isnan(want)) | ((got == want) & ~np.isfinite(want))
    fin = np.isfinite(want)
    assert np.all(same_special | fin), f"{what}: special values differ {got[~(same_special | fin)]} vs {want[~(same_special | fin)]}"
    if fin.any():
        err = np.abs(got[fin] - want[fin]) / np.maximum(np.abs(want[fin]), 1.0)
        assert np.all(np.isfinite(got[fin])), what
        assert err.max() <= tol, f"{what}: max rel err {err.max():.3g} > {tol}"


def _randn(B, N, seed=0, scale=1.0, dev="cuda"):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(B, N, generator=g, device=dev) * scale


SHAPES = [(1, 1), (3, 2), (7, 3), (5, 5), (512, 256), (33, 1023), (9, 4096), (5, 4097),
          (4, 16385), (3, 65537), (2, 300001), (64, 128256)]


@pytest.mark.parametrize("B,N", SHAPES)
@pytest.mark.parametrize("robust", [True, False])
def test_fwd_f32_vs_oracle(ext, B, N, robust):
    x = _randn(B, N, seed=B * 131 + N)
    fn = ext.onepass_lse_float_robust if robust else ext.onepass_lse_float
    _close(fn(x).cpu().numpy(), O.lse_f64(x.cpu().numpy()), RTOL32, f"{B}x{N}")


@pytest.mark.parametrize("B,N", [(512, 256), (64, 128256), (33, 1023), (3, 65537)])
def test_fwd_f32_vs_reference_kernel(ext, B, N):
    ref = ref_ext_or_skip("ref_fused_fp32")
    x = _randn(B, N, seed=7, scale=3.0)
    _close(ext.onepass_lse_float_robust(x).cpu().numpy(),
           ref.onepass_lse_float_robust(x).cpu().numpy(), RTOL32, "robust")
    _close(ext.onepass_lse_float(x).cpu().numpy(), ref.onepass_lse_float(x).cpu().numpy(),
           RTOL32, "plain")


@pytest.mark.parametrize("phase", [1, 2, 3])
@pytest.mark.parametrize("N", [5, 1023, 4099, 70001])
def test_fwd_f32_misaligned_rows(ext, phase, N):
    B = 6
    buf = _randn(1, B * N + 8, seed=phase + N).view(-1)
    x = buf[phase:phase + B * N].view(B, N)
    assert x.is_contiguous()
    _close(ext.onepass_lse_float_robust(x).cpu().numpy(), O.lse_f64(x.cpu().numpy()), RTOL32)


def test_fwd_robust_ieee_cases(ext):
    B, N = 6, 50000
    x = _randn(B, N, seed=3)
    mask = torch.rand(B, N, generator=torch.Generator(device="cuda").manual_seed(1), device="cuda") < 0.01
    x[mask] = float("-inf")
    x[0] = float("-inf")                 # all -inf -> -inf
    x[1, 10] = float("inf")              # +inf and NaN -> NaN
    x[1, 20] = float("nan")
    x[2, 30000] = float("inf")           # +inf -> +inf
    x[3, 49999] = float("nan")           # NaN at the tail -> NaN
    got = ext.onepass_lse_float_robust(x).cpu().numpy()
    want = O.lse_f64(x.cpu().numpy())
    assert got[0] == -np.inf and np.isnan(got[1]) and got[2] == np.inf and np.isnan(got[3])
    _close(got, want, RTOL32)
    ref = ref_ext_or_skip("ref_fused_fp32")
    r = ref.onepass_lse_float_robust(x).cpu().numpy()
    assert r[0] == -np.inf and np.isnan(r[1]) and r[2] == np.inf and np.isnan(r[3])
    _close(got[4:], r[4:], RTOL32)


def test_fwd_empty_rows(ext):
    x = torch.empty(4, 0, device="cuda")
    assert torch.all(ext.onepass_lse_float_robust(x) == float("-inf"))
    assert torch.all(ext.onepass_lse_float(x) == -1e30)
    assert ext.onepass_lse_float(torch.empty(0, 7, device="cuda")).shape == (0,)


@pytest.mark.parametrize("B,N", [(3, 2), (5, 5), (512, 256), (7, 4097), (64, 128256), (2, 300001)])
def test_bwd_f32_vs_oracle(ext, B, N):
    x = _randn(B, N, seed=N)
    g = _randn(B, 1, seed=1).view(B)
    lse = ext.onepass_lse_float_robust(x)
    gx = ext.onepass_lse_float_backward(g, x, lse).cpu().numpy()
    want = O.lse_bwd_f64(g.cpu().numpy(), x.cpu().numpy(), lse.cpu().numpy())
    err = np.abs(gx - want) / np.maximum(np.abs(want), 1e-30)
    assert err.max() <= RTOL32, err.max()


def test_bwd_vs_reference_kernel(ext):
    ref = ref_ext_or_skip("ref_fused_fp32")
    B, N = 64, 128256
    x = _randn(B, N, seed=11)
    g = torch.ones(B, device="cuda")
    lse = ref.onepass_lse_float_robust(x)
    a = ext.onepass_lse_float_backward(g, x, lse)
    b = ref.onepass_lse_float_backward(g, x, lse)
    rel = ((a - b).abs() / b.abs().clamp_min(1e-30)).max().item()
    assert rel <= RTOL32, rel


@pytest.mark.parametrize("phase", [1, 3])
def test_bwd_misaligned_and_mixed_phase(ext, phase):
    B, N = 4, 10007
    buf = _randn(1, B * N + 8, seed=5).view(-1)
    x = buf[phase:phase + B * N].view(B, N)
    g = torch.rand(B, device="cuda")
    lse = ext.onepass_lse_float_robust(x)
    want = O.lse_bwd_f64(g.cpu().numpy(), x.cpu().numpy(), lse.cpu().numpy())
    gx = ext.onepass_lse_float_backward(g, x, lse)      # gx 16-B aligned, x not: scalar path
    np.testing.assert_allclose(gx.cpu().numpy(), want, rtol=RTOL32, atol=0)


def test_autograd_matches_torch(ext):
    import fuselse_b200
    lse = fuselse_b200.make_fuselse_logsumexp(ext, robust=True)
    x = _randn(4 * 3, 5001, seed=2).view(4, 3, 5001).requires_grad_()
    y = lse(x, dim=-1)
    x2 = x.detach().double().requires_grad_()
    y2 = torch.logsumexp(x2, dim=-1)
    torch.testing.assert_close(y.double(), y2, rtol=RTOL32, atol=RTOL32)
    w = torch.rand_like(y)
    (y * w).sum().backward()
    (y2 * w.double()).sum().backward()
    torch.testing.assert_close(x.grad.double(), x2.grad, rtol=RTOL32, atol=1e-9)
    k = lse(x.detach(), dim=-1, keepdim=True)
    assert k.shape == (4, 3, 1)
    # non-contiguous input goes through the flatten path
    xt = x.detach().transpose(0, 1)
    torch.testing.assert_close(lse(xt, dim=-1).double(), torch.logsumexp(xt.double(), -1),
                               rtol=RTOL32, atol=RTOL32)


# ----------------------------------------------------------------------- fp16
@pytest.mark.parametrize("B,N", [(3, 2), (5, 9), (512, 256), (16, 16032), (7, 40001), (8, 128256)])
def test_fwd_f16_vs_oracle(ext, B, N):
    x = (_randn(B, N, seed=N, scale=3.0)).half()
    got = ext.batched_logsumexp_fp16(x).cpu().numpy()
    want = O.lse_f64(x.float().cpu().numpy())
    _close(got, want, RTOL32, "fp16 vs fp64 oracle")


def test_fwd_f16_llm_config_vs_reference(ext):
    ref = ref_ext_or_skip("ref_fused_fp16")
    B, N = 1024, 16032          # one vocab shard of the (8192, 128256) config
    x = _randn(B, N, seed=5, scale=3.0)
    col = torch.randint(0, N, (B,), generator=torch.Generator(device="cuda").manual_seed(6), device="cuda")
    x[torch.arange(B, device="cuda"), col] += 15.0
    xh = x.half()
    _close(ext.batched_logsumexp_fp16(xh).cpu().numpy(),
           ref.batched_logsumexp_fp16(xh).cpu().numpy(), TOL16, "fp16 vs reference")


@pytest.mark.parametrize("phase", [1, 5, 7])
def test_fwd_f16_misaligned(ext, phase):
    B, N = 5, 3001
    buf = _randn(1, B * N + 16, seed=phase).view(-1).half()
    x = buf[phase:phase + B * N].view(B, N)
    _close(ext.batched_logsumexp_fp16(x).cpu().numpy(), O.lse_f64(x.float().cpu().numpy()), RTOL32)


# ------------------------------------------------------------- shard partials
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("G", [1, 2, 3, 8])
def test_partial_combine_equals_full_row(ext, dtype, G):
    B, N = 64, 16032 * 2 + 5
    x = _randn(B, N, seed=G, scale=3.0).to(dtype)
    x[3] = float("-inf")
    x[4, :100] = float("-inf")
    cols = np.linspace(0, N, G + 1).astype(int)
    parts = [ext.lse_partial(x[:, a:b].contiguous()) for a, b in zip(cols, cols[1:])]
    got = ext.lse_combine(torch.stack(parts)).cpu().numpy()
    _close(got, O.lse_f64(x.float().cpu().numpy()), RTOL32, f"G={G}")


# ------------------------------------------------ peer-memory exchange, G = 1
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("B,N", [(1, 5), (7, 16032), (8192, 16032), (13, 100003)])
def test_vocab_exchange_single_rank(ext, dtype, B, N):
    from fuselse_b200.distributed import VocabShardExchange
    ex = VocabShardExchange.single_rank(B)
    x = _randn(B, N, seed=B + N, scale=3.0).to(dtype)
    if B > 3:
        x[2] = float("-inf")
    want = O.lse_f64(x.float().cpu().numpy())
    for _ in range(3):  # epochs advance, slots alternate
        _close(ex(x).cpu().numpy(), want, RTOL32, f"exchange {B}x{N}")
    assert not ex.error()
    assert ex.buf[:4].view(torch.int32).item() == 3  # epoch counter


def test_vocab_exchange_rejects_bad_shapes(ext):
    from fuselse_b200.distributed import VocabShardExchange
    ex = VocabShardExchange.single_rank(4)
    with pytest.raises(RuntimeError):
        ex(torch.zeros(5, 10, device="cuda"))
    with pytest.raises(RuntimeError):
        ex(torch.zeros(4, 10, device="cuda", dtype=torch.float64))


@pytest.mark.parametrize("scale", [1e6, 1e12, 1e25, 1e37])
def test_fwd_bwd_large_magnitudes(ext, scale):
    """Logits far beyond any realistic range: the sum keeps the max's own term
    at exactly 1, so the result is the max plus log of a count of ties (the
    reference's pair max + log(1 + exp(min - max)) gives the same), never
    +-inf from an overflowing rescale."""
    B, N = 37, 5003
    x = _randn(B, N, seed=int(np.log10(scale)), scale=scale)
    x[3, 17] = x[3].max() + 0  # a duplicated max in one row
    x[3, 4000] = x[3, 17]
    lse = ext.onepass_lse_float_robust(x)
    want = O.lse_f64(x.cpu().numpy())
    _close(lse.cpu().numpy(), want, RTOL32, f"scale {scale:g}")
    assert np.isfinite(lse.cpu().numpy()).all()
    g = torch.ones(B, device="cuda")
    gx = ext.onepass_lse_float_backward(g, x, lse).cpu().numpy().astype(np.float64)
    want_gx = O.lse_bwd_f64(g.cpu().numpy(), x.cpu().numpy(), lse.cpu().numpy())
    np.testing.assert_allclose(gx, want_gx, rtol=1e-5, atol=1e-6)
    ref = None
    try:
        ref = ref_ext_or_skip("ref_fused_fp32")
    except pytest.skip.Exception:
        pass
    if ref is not None and scale <= 1e25:
        _close(lse.cpu().numpy(), ref.onepass_lse_float_robust(x).cpu().numpy(), RTOL32, "vs reference")


def test_state_does_not_drift_over_many_merges(ext):
    """Many folds of rows whose max stays put (the first element is the max):
    the result matches fp64 to a few ulp of the row's lse, not to a bound that
    grows with the number of folds."""
    B, N = 8, 1 << 20
    x = _randn(B, N, seed=5, scale=0.01)
    x[:, 0] = 40.0
    lse = ext.onepass_lse_float_robust(x).cpu().numpy().astype(np.float64)
    want = O.lse_f64(x.cpu().numpy())
    assert np.abs(lse - want).max() <= 8 * np.spacing(np.float32(40.0 + np.log(N)))


def test_vocab_exchange_single_rank_close(ext):
    from fuselse_b200.distributed import VocabShardExchange
    ex = VocabShardExchange.single_rank(8)
    x = _randn(8, 100, seed=1)
    _close(ex(x).cpu().numpy(), O.lse_f64(x.cpu().numpy()), RTOL32)
    ex.close()  # a single-rank exchange owns a torch buffer: nothing to unmap
    assert not ex.error()
