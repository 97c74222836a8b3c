"""Speed against the reference's own CUDA kernels on the same B200 and inputs.

The reference kernels (fuselse/gpu/fused_fp32_kernel.cu, fused_fp16_kernel.cu,
intlse/gpu/lse_kernel.cu, lse_kernel_q10_6.cu, experiment_pyjuice/
sparse_float_kernel.cu, sparse_q16_kernel.cu) are built from source into
oracle/_ref by `python -m oracle.build`; each side is captured in its own CUDA
graph and replayed back to back (inputs larger than L2 except the (512,256)
latency cases), timed with CUDA events.

The table is printed (`-s`) and, when FUSELSE_B200_SPEED_OUT names a file,
written there as JSON.  Assertions only guard against regressions on the
bandwidth-sized cases: this library must not be slower than the reference.
"""
import json
import os

import pytest
import torch

from tests.conftest import ref_ext_or_skip

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _graph_us(fn, iters=20):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record()
    for _ in range(iters):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters * 1e3


_rows = []


def _record(case, ours, ref, nbytes, guard):
    _rows.append({"case": case, "ours_us": round(ours, 2), "ref_us": round(ref, 2),
                  "speedup": round(ref / ours, 3), "ours_GBs": round(nbytes / ours / 1e3, 1)})
    print(f"{case:48s} ours {ours:8.1f} us  ref {ref:8.1f} us  x{ref / ours:5.2f}")
    if guard:
        assert ours <= ref * 1.02, f"{case}: {ours:.1f} us vs reference {ref:.1f} us"


@pytest.fixture(scope="module", autouse=True)
def _report():
    yield
    out = os.environ.get("FUSELSE_B200_SPEED_OUT")
    if out and _rows:
        with open(out, "w") as f:
            json.dump(_rows, f, indent=1)


@pytest.mark.parametrize("B,N", [(512, 128256), (512, 256), (64, 128256)])
def test_fuselse_f32(ext, dev, B, N):
    from fuselse_b200 import workloads as W
    ref = ref_ext_or_skip("ref_fused_fp32")
    x = W.fp32_rows(B, N, 0, dev)
    big = B * N * 4 > 128 << 20
    _record(f"FuseLSE fp32 fwd ({B},{N})", _graph_us(lambda: ext.onepass_lse_float_robust(x)),
            _graph_us(lambda: ref.onepass_lse_float_robust(x)), B * N * 4 + B * 4, big)
    lse = ext.onepass_lse_float_robust(x)
    g = torch.ones(B, device=dev)
    _record(f"FuseLSE fp32 bwd ({B},{N})", _graph_us(lambda: ext.onepass_lse_float_backward(g, x, lse)),
            _graph_us(lambda: ref.onepass_lse_float_backward(g, x, lse)), 2 * B * N * 4 + 2 * B * 4, big)


def test_fuselse_f16(ext, dev):
    from fuselse_b200 import workloads as W
    ref = ref_ext_or_skip("ref_fused_fp16")
    x = W.fp16_logits(8192, 16032, 0, dev)
    _record("FuseLSE16 fwd (8192,16032)", _graph_us(lambda: ext.batched_logsumexp_fp16(x)),
            _graph_us(lambda: ref.batched_logsumexp_fp16(x)), x.numel() * 2 + 8192 * 4, True)


@pytest.mark.parametrize("B,N", [(16384, 4096), (64, 1048576), (512, 128256)])
def test_intlse(ext, dev, B, N):
    from fuselse_b200 import workloads as W
    q16 = ref_ext_or_skip("ref_lse_q16")
    q106 = ref_ext_or_skip("ref_lse_q10_6")
    x, qi, qs = W.intlse_inputs(B, N, 0, dev)
    _record(f"IntLSE Q16.16 fp32-in ({B},{N})", _graph_us(lambda: ext.batched_logsumexp(x)),
            _graph_us(lambda: q16.batched_logsumexp(x)), B * N * 4 + B * 4, True)
    # the reference has no int32-input entry: its fp32-input kernel is the comparison
    _record(f"IntLSE Q16.16 int32-in ({B},{N}) [ref fp32-in]",
            _graph_us(lambda: ext.batched_logsumexp_q16_i32(qi)),
            _graph_us(lambda: q16.batched_logsumexp(x)), B * N * 4 + B * 4, True)
    _record(f"IntLSE Q10.6 ({B},{N})", _graph_us(lambda: ext.batched_logsumexp_q10_6(qs)),
            _graph_us(lambda: q106.batched_logsumexp_q10_6(qs)), B * N * 2 + B * 4, True)


def test_sparse(ext, dev):
    from fuselse_b200 import workloads as W
    spf = ref_ext_or_skip("ref_sparse_float")
    spq = ref_ext_or_skip("ref_sparse_q16")
    node, em, params, nids, cids, pids, bs = W.sparse_layer(device=dev)
    S = cids.size(0)
    P, batch = em.shape
    nbytes = P * batch * 4 + S * batch * 4 + S * cids.size(1) * 20 + S * 8

    def ref_call(fn):
        # the reference launch puts nodes on gridDim.y (<= 65535): node-range slices
        for lo in range(0, S, 32768):
            fn(node, em, params, nids[lo:lo + 32768], cids[lo:lo + 32768], pids[lo:lo + 32768], bs)

    _record(f"sparse fp32 (P{P},S{S},E{cids.size(1)},b{batch})",
            _graph_us(lambda: ext.sparse_forward_float(node, em, params, nids, cids, pids, bs), 5),
            _graph_us(lambda: ref_call(spf.sparse_forward_float), 5), nbytes, True)
    _record(f"sparse Q16.16 (P{P},S{S},E{cids.size(1)},b{batch})",
            _graph_us(lambda: ext.sparse_forward_q16(node, em, params, nids, cids, pids, bs), 5),
            _graph_us(lambda: ref_call(spq.sparse_forward_q16), 5), nbytes, True)


@pytest.mark.parametrize("V,B", [(32000, 8), (50257, 8), (128256, 4), (256128, 2)])
def test_selective_rlhf_configs(dev, V, B):
    """The RLHF experiment's selective_log_softmax (run_rlhf.py:145-157, VOCAB_CONFIGS
    :66-71, T-1 = 1023 positions) with torch.logsumexp routed to the reference's
    onepass_lse_float one sequence at a time, against the fused kernel."""
    import fuselse_b200
    ref = ref_ext_or_skip("ref_fused_fp32")
    T = 1023
    g = torch.Generator(device=dev).manual_seed(V)
    logits = torch.randn(B, T, V, generator=g, device=dev)
    idx = torch.randint(0, V, (B, T), generator=g, device=dev)

    def ref_path():
        picked = torch.gather(logits, -1, idx.unsqueeze(-1)).squeeze(-1)
        return picked - torch.stack([ref.onepass_lse_float(seq) for seq in logits])

    with torch.no_grad():
        _record(f"selective log-softmax ({B},{T},{V})",
                _graph_us(lambda: fuselse_b200.selective_log_softmax(logits, idx, robust=False)),
                _graph_us(ref_path), B * T * V * 4 + B * T * 16, True)
