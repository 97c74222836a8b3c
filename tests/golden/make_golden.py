"""Generate tests/golden/*.npz from the reference GPU kernels (run on a B200).

    python tests/golden/make_golden.py [--out DIR]

Needs the reference extensions built from the reference sources into
oracle/_ref (python -m oracle.build, in the container that has the sources);
on the GPU box only those prebuilt files are used.  The sparse cases also call
fuselse_b200.ext.sparse_log_weights to record the device-formed log-weights the
oracle replays (the reference forms the same expression inside its kernel;
the bit-exact comparison of outputs checks that claim too).
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402
from tests.golden import golden_cases as G  # noqa: E402

OUT = Path(__file__).resolve().parent


def _phased(x: np.ndarray, phase: int, dev) -> torch.Tensor:
    """x on the device, its first element `phase` elements past a 256-B boundary."""
    flat = torch.from_numpy(np.ascontiguousarray(x).reshape(-1))
    buf = torch.empty(flat.numel() + 16, dtype=flat.dtype, device=dev)
    view = buf[phase: phase + flat.numel()]
    view.copy_(flat.to(dev))
    return view.view(x.shape)


def intlse_family(dev):
    q16 = O.ref_ext("ref_lse_q16")
    q106 = O.ref_ext("ref_lse_q10_6")
    fams = {"intlse_q16": {}, "intlse_q16_nolut": {}, "intlse_q10_6": {}}
    for i, N in enumerate(G.INTLSE_NS):
        for phase in G.PHASES:
            tag = f"N{N}_p{phase}"
            x = G.intlse_inputs(1000 + i, N, "q16")
            t = _phased(x, phase, dev)
            for fam, fn in (("intlse_q16", q16.batched_logsumexp),
                            ("intlse_q16_nolut", q16.batched_logsumexp_nolut)):
                fams[fam]["x_" + tag] = x
                fams[fam]["phase_" + tag] = np.int64(phase)
                fams[fam]["out_" + tag] = fn(t).cpu().numpy()
            xi = G.intlse_inputs(2000 + i, N, "q10_6")
            ti = _phased(xi, phase, dev)
            fams["intlse_q10_6"]["x_" + tag] = xi
            fams["intlse_q10_6"]["phase_" + tag] = np.int64(phase)
            fams["intlse_q10_6"]["out_" + tag] = q106.batched_logsumexp_q10_6(ti).cpu().numpy()
    return fams


def sparse_family(dev):
    import fuselse_b200

    ref = O.ref_ext("ref_sparse_q16")
    fam = {}
    for i, (E, batch, bs) in enumerate(G.SPARSE_CASES):
        tag = f"E{E}_b{batch}_bs{bs}"
        node, em, params, nids, cids, pids = G.sparse_inputs(3000 + i, E, batch, bs)
        T = lambda a: torch.from_numpy(a).to(dev)
        node_t = T(node)
        ref.sparse_forward_q16(node_t, T(em), T(params), T(nids), T(cids), T(pids), bs)
        K = cids.shape[0]
        # per-output-node log-weights in the layout the oracle takes: (K*bs, E)
        idx = (pids[:, None, :] + np.arange(bs)[None, :, None]).reshape(K * bs, E)
        logw_all = fuselse_b200.ext.sparse_log_weights(T(params)).cpu().numpy()
        fam.update({f"node_{tag}": node, f"em_{tag}": em, f"logw_{tag}": logw_all[idx],
                    f"nids_{tag}": nids, f"cids_{tag}": cids, f"bs_{tag}": np.int64(bs),
                    f"out_{tag}": node_t.cpu().numpy()})
    return {"sparse_q16": fam}


def float_family(dev):
    f32 = O.ref_ext("ref_fused_fp32")
    f16 = O.ref_ext("ref_fused_fp16")
    a, b = {}, {}
    for i, N in enumerate(G.FLOAT_NS):
        x = G.float_inputs(4000 + i, N)
        tag = f"N{N}"
        a["x_" + tag] = x
        a["out_" + tag] = f32.onepass_lse_float_robust(torch.from_numpy(x).to(dev)).cpu().numpy()
        xh = x.astype(np.float16)
        b["x_" + tag] = xh
        b["out_" + tag] = f16.batched_logsumexp_fp16(torch.from_numpy(xh).to(dev)).cpu().numpy()
    return {"fused_fp32": a, "fused_fp16": b}


def main():
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(OUT), help="directory for the .npz files")
    out_dir = Path(ap.parse_args().out)
    out_dir.mkdir(parents=True, exist_ok=True)
    dev = torch.device("cuda:0")
    fams = {}
    fams.update(intlse_family(dev))
    fams.update(sparse_family(dev))
    fams.update(float_family(dev))
    files = []
    for name, arrays in fams.items():
        np.savez_compressed(out_dir / f"{name}.npz", **arrays)
        files.append(f"{name}.npz")
    (out_dir / "MANIFEST.json").write_text(json.dumps(
        {"files": files, "device": torch.cuda.get_device_name(0),
         "generator": "tests/golden/make_golden.py"}, indent=1))
    print("wrote", files)


if __name__ == "__main__":
    main()
