"""Golden cases for the reference GPU kernels (TEST INFRASTRUCTURE).

Each case is a small seeded input; make_golden.py runs the reference kernels
(built from the reference .cu sources into oracle/_ref) on a B200 and stores
inputs and outputs in tests/golden/<family>.npz.  check_case() replays the
inputs through the CPU oracle and compares:
  * IntLSE Q16.16 / Q10.6 and sparse Q16.16: bit for bit;
  * FuseLSE fp32 / fp16 (SFU __expf/__logf in the reference): the fp64
    oracle within 1e-5 relative (fp32) and 2e-3 (fp16).
"""
from __future__ import annotations

import numpy as np

INTLSE_NS = [1, 2, 3, 4, 5, 7, 8, 9, 31, 32, 33, 255, 256, 257, 1023, 1024, 1025, 2051, 5000]
PHASES = [0, 1, 2, 3]  # element offset of the first row into a 16-byte aligned buffer


def intlse_inputs(seed: int, N: int, kind: str):
    rng = np.random.default_rng(seed)
    B = 3
    if kind == "q16":
        x = (rng.standard_normal((B, N)) * np.array([[1.0], [30.0], [200.0]])).astype(np.float32)
        if N >= 6:
            x[2, :5] = [np.nan, np.inf, -np.inf, 1e30, -1e30]
        return x
    if kind == "q10_6":
        x = rng.integers(-32768, 32768, size=(B, N)).astype(np.int16)
        x[0] = np.clip(np.rint(rng.standard_normal(N) * 128), -32768, 32767).astype(np.int16)
        return x
    raise ValueError(kind)


def sparse_inputs(seed: int, E: int, batch: int, block_size: int):
    rng = np.random.default_rng(seed)
    P, K = 50, 6
    em = (rng.standard_normal((P, batch)) * 5 - 20).astype(np.float32)
    em[rng.random((P, batch)) < 0.05] = -np.inf
    num_nodes = K * block_size + 3
    node_mars = np.full((num_nodes, batch), 7.0, np.float32)
    nids = (np.arange(K) * block_size + 3).astype(np.int64)
    cids = np.stack([rng.choice(P, size=E, replace=E > P) for _ in range(K)]).astype(np.int64)
    pids = (np.arange(K * E).reshape(K, E) * block_size).astype(np.int64)
    params = rng.dirichlet(np.ones(E), size=K * block_size).astype(np.float32).reshape(-1)
    params = np.ascontiguousarray(params[: K * E * block_size])
    params[rng.random(params.shape) < 0.03] = 0.0
    return node_mars, em, params, nids, cids, pids


SPARSE_CASES = [(E, batch, bs) for E in (1, 3, 8, 9, 16, 17, 32, 33, 70)
                for batch, bs in ((1, 1), (5, 2), (8, 1), (33, 3))]

FLOAT_NS = [2, 3, 255, 256, 1000, 4097]


def float_inputs(seed: int, N: int):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((4, N)) * np.array([[1.0], [5.0], [30.0], [0.1]])).astype(np.float32)


def check_case(path) -> None:
    from oracle import oracle as O

    d = np.load(path, allow_pickle=False)
    fam = path.stem
    if fam in ("intlse_q16", "intlse_q16_nolut", "intlse_q10_6"):
        kind = O.Q10_6_I16 if fam == "intlse_q10_6" else O.Q16_F32
        lut = fam != "intlse_q16_nolut"
        esize = 2 if kind == O.Q10_6_I16 else 4
        for key in [k for k in d.files if k.startswith("x_")]:
            tag = key[2:]
            x = d[key]
            phase = int(d["phase_" + tag])
            out_ref = d["out_" + tag]
            got, _ = O.intlse_rows(x, kind, lut, base_phase=(phase * esize) % 16)
            np.testing.assert_array_equal(got.view(np.int32), out_ref.view(np.int32),
                                          err_msg=f"{fam} {tag}")
    elif fam == "sparse_q16":
        for key in [k for k in d.files if k.startswith("em_")]:
            tag = key[3:]
            out = O.sparse_q16(d["node_" + tag], d["em_" + tag], d["logw_" + tag],
                               d["nids_" + tag], d["cids_" + tag], int(d["bs_" + tag]))
            np.testing.assert_array_equal(out.view(np.int32), d["out_" + tag].view(np.int32),
                                          err_msg=f"{fam} {tag}")
    elif fam in ("fused_fp32", "fused_fp16"):
        tol = 1e-5 if fam == "fused_fp32" else 2e-3
        for key in [k for k in d.files if k.startswith("x_")]:
            tag = key[2:]
            x = d[key].astype(np.float32)
            ref = d["out_" + tag].astype(np.float64)
            want = O.lse_f64(x)
            np.testing.assert_allclose(ref, want, rtol=tol, atol=tol, err_msg=f"{fam} {tag}")
    else:
        raise AssertionError(f"unknown golden family {fam}")
