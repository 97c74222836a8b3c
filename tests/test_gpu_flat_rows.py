"""GPU parity of the balanced row schedule (fold_rows_flat in csrc/rows.cuh).

fp16 rows of 4 KB .. 64 KB (16-byte aligned) whose one-warp-per-row grid would
end in a short last wave (at most half of the 4736 resident warps on B200),
and the exchange's rows longer than one warp takes (fp32 and fp16), are folded
by one CTA per SM whose warps split the CTA's rows into equal vector ranges; a
row's pieces are merged in shared memory.  These shapes exercise that path,
and its neighbours that keep one warp per row (fp32 rows among them), through
every entry (fp32 forward, fp16 forward, the shard partial + combine, the
single-rank vocab exchange) against the fp64 oracle:

* one row per CTA (B <= SM count: every row split over all 32 warps);
* B just below / above the SM count and multiples of it;
* row counts that give one and two rows per warp, and many rows per CTA;
* rows whose length is not a multiple of the warp's vector group;
* the IEEE rows of the robust mode (row 0 all -inf, row 1 +inf and NaN);
* an 8-byte-aligned operand, which keeps one warp per row;
* repeat calls give identical bits (the schedule is static).

Tolerances as in tests/test_gpu_lse.py: 1e-5 relative to max(|lse|, 1).
"""
import numpy as np
import pytest
import torch

from fuselse_b200 import distributed as D
from fuselse_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    same_special = (np.isnan(got) & np.isnan(want)) | ((got == want) & ~np.isfinite(want))
    fin = np.isfinite(want)
    bad = ~(same_special | fin)
    assert not bad.any(), f"{what}: special values differ at rows {np.nonzero(bad)[0][:8]}"
    if fin.any():
        assert np.all(np.isfinite(got[fin])), f"{what}: non-finite where the oracle is finite"
        err = np.abs(got[fin] - want[fin]) / np.maximum(np.abs(want[fin]), 1.0)
        assert err.max() <= RTOL, f"{what}: max rel err {err.max():.3g} > {RTOL}"


def _rows(B, N, dtype, seed):
    x = W.fp32_rows(B, N, seed=seed, device="cuda") * 3.0
    return x.to(dtype)


F32_SHAPES = [(1, 1024), (147, 1024), (149, 1024), (300, 1024), (2368, 2048), (3000, 4096),
              (5000, 3000), (4000, 1028), (9473, 1536), (16384, 4096), (40000, 1024)]
F16_SHAPES = [(1, 2048), (149, 2048), (2368, 16032), (8192, 16032), (9473, 4104), (4000, 32768)]


@pytest.mark.parametrize("B,N", F32_SHAPES)
def test_f32_forward_and_partial(ext, B, N):
    x = _rows(B, N, torch.float32, seed=B + N)
    want = O.lse_f64(x.cpu().numpy())
    _close(ext.onepass_lse_float_robust(x).cpu().numpy(), want, f"robust {B}x{N}")
    _close(ext.onepass_lse_float(x).cpu().numpy(), want, f"plain {B}x{N}")
    ms = ext.lse_partial(x)
    _close(ext.lse_combine(ms.unsqueeze(0)).cpu().numpy(), want, f"partial {B}x{N}")


@pytest.mark.parametrize("B,N", F16_SHAPES)
def test_f16_forward_and_partial(ext, B, N):
    x = _rows(B, N, torch.float16, seed=B + N)
    want = O.lse_f64(x.float().cpu().numpy())
    _close(ext.batched_logsumexp_fp16(x).cpu().numpy(), want, f"fp16 {B}x{N}")
    ms = ext.lse_partial(x)
    _close(ext.lse_combine(ms.unsqueeze(0)).cpu().numpy(), want, f"fp16 partial {B}x{N}")


@pytest.mark.parametrize("B,N,dtype", [(100, 128256, torch.float16), (149, 2048, torch.float16),
                                       (8192, 16032, torch.float16), (3000, 4096, torch.float32),
                                       (147, 1024, torch.float32), (200, 32064, torch.float32),
                                       (1, 65536, torch.float32)])
def test_single_rank_exchange(B, N, dtype):
    x = _rows(B, N, dtype, seed=3)
    want = O.lse_f64(x.float().cpu().numpy())
    ex = D.VocabShardExchange.single_rank(B, "cuda")
    a = ex(x)
    b = ex(x)
    _close(a.cpu().numpy(), want, f"exchange {B}x{N}")
    assert torch.equal(a, b), "repeat calls differ"


def test_robust_rows_on_flat_shapes(ext):
    # fp16 shard partials (flat: 2368 rows of 4 KB) and the fp32 exchange over
    # rows longer than one warp takes (flat: 200 rows of 128 KB)
    x = W.robust_rows(2368, 2048, seed=2, device="cuda").half()
    want = O.lse_f64(x.float().cpu().numpy())
    assert np.isneginf(want[0]) and np.isnan(want[1])
    ms = ext.lse_partial(x)
    _close(ext.lse_combine(ms.unsqueeze(0)).cpu().numpy(), want, "fp16 robust rows, partial")
    y = W.robust_rows(200, 32064, seed=2, device="cuda")
    want = O.lse_f64(y.cpu().numpy())
    ex = D.VocabShardExchange.single_rank(200, "cuda")
    _close(ex(y).cpu().numpy(), want, "fp32 robust rows, exchange")


def test_misaligned_operand_keeps_warp_rows(ext):
    B, N = 2368, 16032
    buf = _rows(1, B * N + 4, torch.float16, seed=9).view(-1)
    x = buf[4:4 + B * N].view(B, N)  # 8-byte aligned
    assert x.data_ptr() % 16 == 8
    want = O.lse_f64(x.float().cpu().numpy())
    _close(ext.batched_logsumexp_fp16(x).cpu().numpy(), want, "misaligned fp16")
    ms = ext.lse_partial(x)
    _close(ext.lse_combine(ms.unsqueeze(0)).cpu().numpy(), want, "misaligned partial")


def test_repeat_calls_identical(ext):
    x = _rows(8192, 16032, torch.float16, seed=4)
    a = ext.lse_partial(x)
    b = ext.lse_partial(x)
    assert torch.equal(a, b)
    y = _rows(16384, 4096, torch.float32, seed=4)
    assert torch.equal(ext.onepass_lse_float_robust(y), ext.onepass_lse_float_robust(y))
