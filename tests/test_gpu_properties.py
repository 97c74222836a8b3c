"""Size-independent properties of the float paths at the headline size,
(512, 128256) fp32, where an fp64 oracle of every case would be slow:

* softmax rows sum to one: the backward with g = 1 gives exp(x - lse), whose
  row sums are 1 up to the rounding of 128256 terms;
* shift invariance: lse(x + c) = lse(x) + c for an exactly representable c;
* duplication: a row concatenated with itself has lse + ln 2;
* vocab sharding: the partial states of any column split, combined, give the
  full row's lse.

Tolerances: lse values within 1e-5 relative to max(|lse|, 1), as in the other
fp32 tests; row sums of the gradient within 1e-4 (each of 128256 terms carries
a relative error of ~1e-6)."""
import math

import pytest
import torch

from fuselse_b200 import workloads as W

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

B, N = 512, 128256
RTOL = 1e-5


def _rel(a, b):
    return ((a.double() - b.double()).abs() / b.double().abs().clamp_min(1.0)).max().item()


@pytest.fixture(scope="module")
def x():
    return W.fp32_rows(B, N, seed=5, device="cuda") * 2.0


def test_gradient_rows_sum_to_one(ext, x):
    lse = ext.onepass_lse_float_robust(x)
    gx = ext.onepass_lse_float_backward(torch.ones(B, device="cuda"), x, lse)
    sums = gx.double().sum(dim=1)
    assert (sums - 1.0).abs().max().item() <= 1e-4
    assert (gx >= 0).all()


@pytest.mark.parametrize("c", [3.0, -17.5, 1024.0])
def test_shift_invariance(ext, x, c):
    a = ext.onepass_lse_float_robust(x)
    b = ext.onepass_lse_float_robust(x + c)
    assert _rel(b - c, a) <= 2 * RTOL


def test_duplicated_row_adds_ln2(ext, x):
    rows = x[:64]
    a = ext.onepass_lse_float_robust(rows)
    b = ext.onepass_lse_float_robust(torch.cat([rows, rows], dim=1))
    assert _rel(b - math.log(2.0), a) <= 2 * RTOL


@pytest.mark.parametrize("shards", [2, 7, 16])
def test_any_vocab_split_combines_to_the_row(ext, x, shards):
    full = ext.onepass_lse_float_robust(x)
    parts = [ext.lse_partial(W.vocab_shard(x, shards, i)) for i in range(shards)]
    got = ext.lse_combine(torch.stack(parts))
    assert _rel(got, full) <= 2 * RTOL
