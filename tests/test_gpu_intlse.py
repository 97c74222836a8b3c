"""GPU parity of IntLSE (Q16.16 from fp32 / int32, Q10.6 from int16): bit for bit.

Every output is compared as raw bits against (a) the oracle's reference-order
restatement on the same buffer (row address phases included) and (b) the
reference kernels themselves, built from the reference sources, on the very
same device buffer.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.conftest import ref_ext_or_skip

pytestmark = pytest.mark.gpu

CONV = np.float32(1.44269504089) * np.float32(65536.0)


def _bits(t):
    return t.detach().cpu().numpy().view(np.int32)


def _phased(x: torch.Tensor, phase: int) -> torch.Tensor:
    """Same values, first element `phase` elements past an aligned boundary."""
    flat = x.reshape(-1)
    buf = torch.empty(flat.numel() + 16, dtype=x.dtype, device=x.device)
    v = buf[phase:phase + flat.numel()]
    v.copy_(flat)
    return v.view(x.shape)


def _q16_from_f32(x: np.ndarray) -> np.ndarray:
    """Host image of __float2int_rn(x * CONV): fp32 multiply, half-even, saturate, NaN -> 0."""
    with np.errstate(invalid="ignore", over="ignore"):
        p = (x.astype(np.float32) * CONV).astype(np.float32)
        r = np.rint(p.astype(np.float64))
        r = np.where(np.isnan(r), 0.0, r)
        r = np.clip(r, -2.0**31, 2.0**31 - 1)
    return r.astype(np.int64).astype(np.int32)


def _x(B, N, seed, scale=2.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(B, N, generator=g, device="cuda") * scale


NS = [1, 2, 3, 4, 5, 7, 8, 255, 256, 257, 1023, 1024, 1025, 4096, 4099, 65537]


@pytest.mark.parametrize("N", NS)
@pytest.mark.parametrize("phase", [0, 1, 2, 3])
@pytest.mark.parametrize("lut", [True, False])
def test_q16_f32_vs_oracle(ext, N, phase, lut):
    x = _phased(_x(3, N, seed=N + phase, scale=[2.0, 30.0][N % 2]), phase)
    fn = ext.batched_logsumexp if lut else ext.batched_logsumexp_nolut
    want, _ = O.intlse_rows(x.cpu().numpy(), O.Q16_F32, lut, base_phase=(phase * 4) % 16)
    np.testing.assert_array_equal(_bits(fn(x)), want.view(np.int32))


@pytest.mark.parametrize("N", NS)
@pytest.mark.parametrize("phase", [0, 1, 2, 3])
def test_q16_i32_vs_oracle(ext, N, phase):
    q = torch.from_numpy(_q16_from_f32(_x(3, N, seed=7 * N).cpu().numpy())).cuda()
    q = _phased(q, phase)
    want, _ = O.intlse_rows(q.cpu().numpy(), O.Q16_I32, True, base_phase=(phase * 4) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q16_i32(q)), want.view(np.int32))


@pytest.mark.parametrize("N", NS)
@pytest.mark.parametrize("phase", [0, 1, 2, 3])
def test_q10_6_vs_oracle(ext, N, phase):
    g = torch.Generator(device="cuda").manual_seed(N * 3 + phase)
    if N % 2:
        q = torch.randint(-32768, 32768, (3, N), generator=g, device="cuda", dtype=torch.int32)
    else:
        q = (torch.randn(3, N, generator=g, device="cuda") * 128).round().clamp(-32768, 32767)
    q = _phased(q.to(torch.int16), phase)
    want, _ = O.intlse_rows(q.cpu().numpy(), O.Q10_6_I16, True, base_phase=(phase * 2) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q10_6(q)), want.view(np.int32))


def test_q16_special_values(ext):
    x = _x(4, 1000, seed=1)
    x[0, :5] = torch.tensor([float("nan"), float("inf"), float("-inf"), 1e30, -1e30])
    x[1] = float("-inf")
    x[2] = float("inf")
    x[3, 999] = 3e9
    want, _ = O.intlse_rows(x.cpu().numpy(), O.Q16_F32, True)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp(x)), want.view(np.int32))
    ref = ref_ext_or_skip("ref_lse_q16")
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp(x)), _bits(ref.batched_logsumexp(x)))


def test_int32_extremes(ext):
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randint(-2**31, 2**31 - 1, (5, 3000), generator=g, device="cuda", dtype=torch.int64)
    q = q.to(torch.int32)
    q[0, :4] = torch.tensor([2**31 - 1, -2**31, 2**31 - 1, -2**31], dtype=torch.int32)
    want, _ = O.intlse_rows(q.cpu().numpy(), O.Q16_I32, True)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q16_i32(q)), want.view(np.int32))


@pytest.mark.parametrize("phase", [0, 1, 2, 3])
@pytest.mark.parametrize("N", [1, 3, 256, 1025, 4099, 65537])
def test_vs_reference_kernels_same_buffer(ext, phase, N):
    q16 = ref_ext_or_skip("ref_lse_q16")
    q106 = ref_ext_or_skip("ref_lse_q10_6")
    x = _phased(_x(5, N, seed=N, scale=3.0), phase)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp(x)), _bits(q16.batched_logsumexp(x)))
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_nolut(x)),
                                  _bits(q16.batched_logsumexp_nolut(x)))
    qi = _phased((x * 64).round().clamp(-32768, 32767).to(torch.int16), phase)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q10_6(qi)),
                                  _bits(q106.batched_logsumexp_q10_6(qi)))


def test_int32_entry_reproduces_float_entry(ext):
    """q = rint_sat(x * CONV) through the int32 entry == the fp32 entry on x."""
    for B, N in [(7, 4096), (3, 100003)]:
        x = _x(B, N, seed=N)
        q = torch.from_numpy(_q16_from_f32(x.cpu().numpy())).cuda()
        np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q16_i32(q)),
                                      _bits(ext.batched_logsumexp(x)))


@pytest.mark.slow
@pytest.mark.parametrize("B,N", [(16384, 4096), (64, 1048576)])
def test_baseline_configs_vs_reference(ext, B, N):
    """x ~ N(0, 2^2); Q16.16 int32 = round(x*65536), Q10.6 int16 =
    clamp(round(x*64)); every row bit-identical to the reference kernels and to the
    oracle on a sample of rows."""
    q16 = ref_ext_or_skip("ref_lse_q16")
    q106 = ref_ext_or_skip("ref_lse_q10_6")
    x = _x(B, N, seed=0, scale=2.0)
    qi32 = (x * 65536).round().to(torch.int32)
    qi16 = (x * 64).round().clamp(-32768, 32767).to(torch.int16)
    # the reference has no int32 kernel: its float kernel on xf with rint(xf*CONV) == qi32
    xf = (qi32.double() / float(CONV)).float()
    q_back = torch.from_numpy(_q16_from_f32(xf.cpu().numpy())).cuda()
    got = _bits(ext.batched_logsumexp_q16_i32(q_back))
    np.testing.assert_array_equal(got, _bits(q16.batched_logsumexp(xf)))
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q10_6(qi16)),
                                  _bits(q106.batched_logsumexp_q10_6(qi16)))
    rows = [0, 1, B // 2, B - 1]
    want, _ = O.intlse_rows(qi32[rows].cpu().numpy(), O.Q16_I32, True)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q16_i32(qi32[rows].contiguous())),
                                  want.view(np.int32))


@pytest.mark.parametrize("B,N", [(5000, 1), (3000, 5), (4000, 256), (1000, 1023), (2000, 1024), (700, 1025)])
@pytest.mark.parametrize("phase", [0, 3])
def test_many_short_rows_all_kinds(ext, B, N, phase):
    """Enough short rows that the one-CTA-per-row launch keeps only its
    resident CTAs and loops each over rows (rows of <= 4 KB): bit for bit."""
    x = _phased(_x(B, N, seed=B + N + phase, scale=3.0), phase)
    want, _ = O.intlse_rows(x.cpu().numpy(), O.Q16_F32, True, base_phase=(phase * 4) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp(x)), want.view(np.int32))
    qi = _phased(torch.from_numpy(_q16_from_f32(x.cpu().numpy())).cuda(), phase)
    want, _ = O.intlse_rows(qi.cpu().numpy(), O.Q16_I32, True, base_phase=(phase * 4) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q16_i32(qi)), want.view(np.int32))
    qs = _phased(torch.clamp(torch.round(x * 64), -32768, 32767).to(torch.int16), phase)
    want, _ = O.intlse_rows(qs.cpu().numpy(), O.Q10_6_I16, True, base_phase=(phase * 2) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q10_6(qs)), want.view(np.int32))


@pytest.mark.parametrize("N", [2048, 3072, 4096, 5120, 7168, 8192])
@pytest.mark.parametrize("phase", [0, 1])
def test_whole_round_rows_all_kinds(ext, N, phase):
    """Rows of 1024*K elements, plentiful: aligned (phase 0) they take the
    whole-rounds kernel (all of a chain's vectors loaded at once, no per-round
    predicates), misaligned (phase 1) the general one — bit for bit either way,
    with and without the correction table."""
    B = 600
    x = _phased(_x(B, N, seed=N + phase, scale=3.0), phase)
    want, _ = O.intlse_rows(x.cpu().numpy(), O.Q16_F32, True, base_phase=(phase * 4) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp(x)), want.view(np.int32))
    want, _ = O.intlse_rows(x.cpu().numpy(), O.Q16_F32, False, base_phase=(phase * 4) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_nolut(x)), want.view(np.int32))
    qi = _phased(torch.from_numpy(_q16_from_f32(x.cpu().numpy())).cuda(), phase)
    want, _ = O.intlse_rows(qi.cpu().numpy(), O.Q16_I32, True, base_phase=(phase * 4) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q16_i32(qi)), want.view(np.int32))
    qs = _phased(torch.clamp(torch.round(x * 64), -32768, 32767).to(torch.int16), phase)
    want, _ = O.intlse_rows(qs.cpu().numpy(), O.Q10_6_I16, True, base_phase=(phase * 2) % 16)
    np.testing.assert_array_equal(_bits(ext.batched_logsumexp_q10_6(qs)), want.view(np.int32))
