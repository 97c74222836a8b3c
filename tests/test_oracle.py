"""CPU tests of the oracle: pins against the reference's own code and golden vectors.

The oracle is trusted only after these pass:
  * its pair function, correction table and float->Q16.16 conversion, run in
    the AVX2 library's reduction order, reproduce the reference AVX2 IntLSE
    library (intlse/cpu/lse_kernel_simd.c, compiled from source into
    oracle/_ref) bit for bit;
  * its GPU-order restatement reproduces the golden outputs of the reference
    GPU kernels (tests/golden/*.npz, generated on a B200 by
    tests/golden/make_golden.py from the reference .cu files built from source);
  * its fp64 float path agrees with torch.logsumexp (float64) and the
    reference FuseLSE-CPU extension.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def _need_ref(name):
    if not O.ref_available(name):
        pytest.skip(f"reference build {name} absent")


@pytest.mark.parametrize("N", [2, 3, 5, 31, 63, 64, 65, 127, 129, 1000, 4096, 5000])
@pytest.mark.parametrize("scale", [0.5, 3.0, 40.0])
def test_pair_pinned_to_reference_avx2(N, scale):
    _need_ref("simd")
    rng = np.random.default_rng(N * 7 + int(scale))
    x = (rng.standard_normal((6, N)) * scale).astype(np.float32)
    got = O.simd_q16_rows(x)
    ref = O.ref_simd_rows(x)
    np.testing.assert_array_equal(got.view(np.int32), ref.view(np.int32))


def test_pair_pinned_llm_row():
    _need_ref("simd")
    rng = np.random.default_rng(0)
    x = rng.standard_normal((32, 128256)).astype(np.float32)  # BASELINE CPU config
    np.testing.assert_array_equal(O.simd_q16_rows(x).view(np.int32),
                                  O.ref_simd_rows(x).view(np.int32))


def test_pair_known_answers():
    # sub = 0: M = 2^16, table index 64 & 63 = 0 -> a + 65536
    assert O.pair_q16(1000, 1000) == 1000 + 65536
    assert O.pair_q16(O.Q_NEG_INF, O.Q_NEG_INF) == O.Q_NEG_INF + 65536
    assert O.pair_q10_6(O.Q_NEG_INF, O.Q_NEG_INF) == O.Q_NEG_INF + 64
    # far below: shift >= 17 -> M = 0, table 0 -> identity
    assert O.pair_q16(5 << 16, (5 - 40) << 16) == 5 << 16
    assert O.pair_q16(5 << 16, O.Q_NEG_INF) == 5 << 16
    # one unit below (sub = -65536): shift 1, M = 2^15, index 32 -> table 5399
    assert O.pair_q16(0, -65536) == 32768 + 5399
    assert O.pair_q16(0, -65536, use_lut=False) == 32768
    # symmetric
    rng = np.random.default_rng(1)
    for a, b in rng.integers(-2**31, 2**31, size=(200, 2)):
        assert O.pair_q16(int(a), int(b)) == O.pair_q16(int(b), int(a))
        assert O.pair_q10_6(int(a), int(b)) == O.pair_q10_6(int(b), int(a))


def test_conversion_rounding():
    c = np.float32(1.44269504089) * np.float32(65536.0)
    # half-even ties: x*CONV lands exactly on k + 0.5 only for special x; test the rounding rule itself
    assert O.lib().orc_f2i_rn(2.5) == 2 and O.lib().orc_f2i_rn(3.5) == 4
    assert O.lib().orc_f2i_rn(-2.5) == -2
    assert O.lib().orc_f2i_rn(float("nan")) == 0
    assert O.lib().orc_f2i_rn(float("inf")) == 2**31 - 1
    assert O.lib().orc_f2i_rn(float("-inf")) == -2**31
    x = np.float32(0.3)
    assert O.f32_to_q16(np.array([x]))[0] == int(np.rint(np.float32(x * c)))


def test_int32_entry_matches_float_entry_in_oracle():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((5, 777)) * 2).astype(np.float32)
    q = O.f32_to_q16(x)
    for phase in (0, 4, 8, 12):
        a, acc_a = O.intlse_rows(x, O.Q16_F32, True, phase)
        b, acc_b = O.intlse_rows(q, O.Q16_I32, True, phase)
        np.testing.assert_array_equal(acc_a, acc_b)


def test_fp64_lse_rules():
    x = np.array([[0.0, 1.0, 2.0],
                  [-np.inf, -np.inf, -np.inf],
                  [0.0, np.inf, 1.0],
                  [np.nan, np.inf, 0.0],
                  [-np.inf, 3.0, -np.inf]])
    r = O.lse_f64(x)
    assert abs(r[0] - np.log(np.exp(0) + np.exp(1) + np.exp(2))) < 1e-12
    assert r[1] == -np.inf and r[2] == np.inf and np.isnan(r[3]) and r[4] == 3.0
    t = torch.tensor(x[[0, 1, 2, 4]], dtype=torch.float64)
    np.testing.assert_allclose(r[[0, 1, 2, 4]], torch.logsumexp(t, -1).numpy())


def test_fuselse_cpu_port_matches_reference_extension():
    _need_ref("ref_fused_cpu")
    m = O.ref_ext("ref_fused_cpu")
    x = torch.randn(16, 3001, generator=torch.Generator().manual_seed(0))
    ref = m.cpu_lse_float(x).numpy()
    port = O.fuselse_cpu_port(x.numpy(), threads=2)
    np.testing.assert_allclose(port, ref, rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(port, O.lse_f64(x.numpy()), rtol=1e-5)


def _golden_files():
    return sorted(GOLDEN.glob("*.npz"))


def test_golden_fixtures_present():
    meta = GOLDEN / "MANIFEST.json"
    if not meta.exists():
        pytest.skip("golden fixtures not generated yet (tests/golden/make_golden.py on a B200)")
    names = json.loads(meta.read_text())["files"]
    for n in names:
        assert (GOLDEN / n).exists(), n


@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.stem)
def test_oracle_matches_reference_gpu_golden(path):
    """The GPU-order restatement reproduces the reference kernels' own outputs."""
    from tests.golden.golden_cases import check_case
    check_case(path)
