"""Benchmark of the row log-sum-exp hot path on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--eager] [--flush-l2] [--no-e2e] [--no-cpu-baseline]

One JSON line on rank 0.  Default workload (the headline, BASELINE metric):
FuseLSE fp32 forward + backward over (B, N) = (512, 128256), x ~ N(0, 1),
upstream gradient ones(B), robust mode.  One step = forward kernel + backward
kernel over one batch already resident in HBM.  With N GPUs (torchrun, one
process per GPU) every rank runs its own 512 rows (batch-row sharding, weak
scaling, no collective on the data path); `value` = algorithmic bytes of all
ranks / max-over-ranks device time.

Algorithmic bytes per step and GPU (the roofline numerator):
  forward  B*N*4 + B*4                = 262,670,336 B
  backward 2*B*N*4 + 2*B*4            = 525,340,672 B  (read x, g, lse; write gx)
Timing: W untimed warm-up steps, then two timed passes of K steps each, steps
back to back, with inputs larger than L2 (x and gx are 262 MB each, L2 126 MB;
each kernel pays the write-back of the previous kernel's dirty lines, as in a
training loop) and two input batches alternating step by step, so no step
finds its input left in L2 by the step before (`--same-input`: one batch);
`--flush-l2` instead evicts L2 between steps outside the events.
  * step pass (`value`, `ms_per_step`): each step — forward then backward — is
    one CUDA graph captured through the public entry points, replayed K times
    between two CUDA events on the launching stream (as a training loop that
    captures its step runs it);
  * per-kernel pass (`kernels`, `roofline`): each kernel replayed from its own
    graph with CUDA events between the kernels (`ms_per_step_kernel_pass` is
    their sum; `--kernel-graphs` reports it as the step, `--eager` launches
    directly).  `kernels.fwd.alone` times the forward again on its own (a
    graph per call, inputs alternating): inside the step it also carries the
    write-back of the backward's last dirty gradient lines.
Barrier and synchronize around each timed region; max over ranks.

`e2e` (default workload): the same metric through the public host-buffer API
(fuselse_b200.host.HostRowPipeline): every step x and g are copied in from
pinned host memory and lse and the gradient copied back, in ~16 MB chunks
whose uploads, kernels and downloads overlap on three streams; h2d/d2h bytes
are those copies.

Other workloads (`--workload`): fwd_f32 (forward alone); sls_f32 (fused
selective log-softmax forward + backward over RLHF-shaped logits
(4, 1023, 128256)); f16_vocab / f16_vocab_nccl (fp16 vocab shard of
(8192, 128256), exchanged over NVLink by the library or by NCCL); intlse_q16 /
intlse_q10_6 [_long] (IntLSE at (16384, 4096) / (64, 1048576)); sparse_f32 /
sparse_q16 (the PC sum layer) and sparse_fwdbwd_f32 (its forward + backward).

`--impl reference` times the reference's own CPU implementation of the path
(FuseLSE-CPU, fuselse/cpu/fused_fp32_cpu.cpp, built from source into
oracle/_ref; the reference has no CPU backward, so the backward is the C
port of grad*exp(x - lse)) on all host threads, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "LSE fwd+bwd HBM GB/s (% of B200 peak) at (512,128256) fp32; rows/s 1-8 GPU"
B_ROWS, N_COLS = 512, 128256
# the headline step, named identically by both arms (ours and --impl reference)
HEADLINE_WORKLOAD = ("FuseLSE fp32 forward+backward (B,N)=(512,128256) per device, x~N(0,1), "
                     "grad ones, robust")
FALLBACK_HBM_GBS = 6650.0


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "source": "fallback"}


def profiled_traffic(kernel: str):
    """Per-launch DRAM bytes from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(kernel)


# --------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        exe = shutil.which("nvidia-smi")
        if exe:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                [exe, f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        max_mhz = max(r[1] for r in rows)
        loaded = [r for r in rows if r[0] > 0.5 * max_mhz] or rows
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names[1:], r[2][1:]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max_mhz,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ workloads
class Workload:
    """A hot-path step on this rank's synthetic inputs."""
    name = ""
    config: dict = {}
    dtype = "f32"
    launches_per_step = 0

    def kernels(self):  # [(label, callable, algorithmic bytes)]
        raise NotImplementedError

    def rows(self):
        return 0


class FwdBwdF32(Workload):
    """Steps alternate between two input batches (x0, x1), so a step never
    finds its input left in L2 by the step before; within a step the backward
    reads the same x as the forward, as a training step does."""
    name = "fwdbwd_f32"
    dtype = "f32"

    def __init__(self, dev, seed, B=B_ROWS, N=N_COLS, do_bwd=True, same_input=False):
        from fuselse_b200 import ext, workloads as W
        self.ext, self.B, self.N, self.do_bwd = ext, B, N, do_bwd
        self.xs = [W.fp32_rows(B, N, seed, dev)]
        if not same_input:
            self.xs.append(W.fp32_rows(B, N, seed + 1000, dev))
        self.phases = len(self.xs)
        self.x = self.xs[0]
        self.g = torch.ones(B, device=dev)
        self.lse = torch.empty(B, device=dev)
        inputs = ("one input batch every step" if same_input else
                  "two input batches alternating step by step (no input reused from L2 across steps)")
        self.config = {"workload": (HEADLINE_WORKLOAD if (do_bwd and (B, N) == (B_ROWS, N_COLS)) else
                                    f"FuseLSE fp32 {'forward+backward' if do_bwd else 'forward'} "
                                    f"(B,N)=({B},{N}) per GPU, x~N(0,1), grad ones, robust"),
                       "B": B, "N": N,
                       "l2": f"inputs larger than L2 (x 262 MB, gx 262 MB), steps back to back, {inputs}",
                       "parallelism": "batch rows, one process per GPU, no collective"}
        self.launches_per_step = 2 if do_bwd else 1

    def set_phase(self, p):
        self.x = self.xs[p % self.phases]

    def _fwd(self):
        self.lse = self.ext.onepass_lse_float_robust(self.x)

    def _bwd(self):
        self.gx = self.ext.onepass_lse_float_backward(self.g, self.x, self.lse)

    def kernels(self):
        B, N = self.B, self.N
        k = [("fwd", self._fwd, B * N * 4 + B * 4)]
        if self.do_bwd:
            k.append(("bwd", self._bwd, 2 * B * N * 4 + 2 * B * 4))
        return k

    def rows(self):
        return self.B

    # end to end through the public host-buffer API: pinned host rows in, lse and
    # gradient back in pinned host memory every step, copies overlapped with the
    # kernels chunk by chunk (fuselse_b200.host.HostRowPipeline)
    def e2e_setup(self, dev):
        from fuselse_b200.host import HostRowPipeline
        self.pipe = HostRowPipeline(self.N, device=dev, depth=3, robust=True)
        self.x_host = self.x.cpu().pin_memory()
        self.g_host = self.g.cpu().pin_memory()
        self.gx_host = torch.empty_like(self.x_host).pin_memory()
        self.lse_host = torch.empty(self.B).pin_memory()
        self.h2d = self.x_host.numel() * 4 + self.g_host.numel() * 4
        self.d2h = self.gx_host.numel() * 4 + self.lse_host.numel() * 4
        self.e2e_api = (f"fuselse_b200.host.HostRowPipeline.run ({self.pipe.rows}-row chunks, "
                        "copies overlapped)")

    def e2e_step(self, dev):
        self.pipe.run(self.x_host, self.lse_host, self.g_host, self.gx_host)


class SelectiveF32(Workload):
    """Fused selective log-softmax forward + backward over RLHF-shaped logits
    (the Llama-3 configuration of run_rlhf.py: batch 4, T-1 = 1023 positions,
    V = 128256), targets uniform over the vocabulary, upstream gradient ones."""
    name = "sls_f32"
    dtype = "f32"

    def __init__(self, dev, seed, batch=4, T=1023, V=128256):
        from fuselse_b200 import ext, workloads as W
        self.ext = ext
        self.R, self.V = batch * T, V
        self.x = W.fp32_rows(self.R, V, seed, dev)
        gen = torch.Generator(device="cpu").manual_seed(seed + 7)
        self.t = torch.randint(0, V, (self.R,), generator=gen).to(dev)
        self.g = torch.ones(self.R, device=dev)
        self.config = {"workload": f"selective log-softmax fp32 forward+backward, logits ({batch},{T},{V}) "
                                   "x~N(0,1), targets uniform, grad ones",
                       "rows": self.R, "V": V,
                       "l2": "inputs larger than L2 (logits 2.1 GB), steps back to back",
                       "parallelism": "batch rows, one process per GPU, no collective"}
        self.launches_per_step = 2

    def _fwd(self):
        self.logp, self.lse = self.ext.selective_logsoftmax_rows(self.x, self.t)

    def _bwd(self):
        self.gx = self.ext.selective_logsoftmax_backward(self.g, self.x, self.lse, self.t)

    def kernels(self):
        R, V = self.R, self.V
        return [("sls_fwd", self._fwd, R * V * 4 + R * (8 + 4 + 4)),
                ("sls_bwd", self._bwd, 2 * R * V * 4 + R * (4 + 4 + 8))]

    def rows(self):
        return self.R


class F16Vocab(Workload):
    name = "f16_vocab"
    dtype = "f16"

    def __init__(self, dev, seed, world=1, rank=0, nccl=False):
        from fuselse_b200 import distributed as D, ext, workloads as W
        self.ext = ext
        B = 8192
        # this GPU's vocab shard of the (8192, 128256) logits (8 shards of 16032
        # columns); with fewer than 8 GPUs every rank still holds one shard
        self.xs = W.fp16_logits(B, 16032, seed, dev)
        self.B, self.Ns = B, self.xs.size(1)
        self.world, self.nccl = world, nccl
        if not nccl:
            self.ex = (D.VocabShardExchange(B, device=dev) if world > 1
                       else D.VocabShardExchange.single_rank(B, dev))
        how = ("partial + NCCL all-gather + combine" if nccl else
               "partial kernel storing (max,sumexp) into every rank's buffer over NVLink "
               "+ flag-wait combine kernel")
        self.config = {"workload": f"FuseLSE16 vocab shard (8192,16032) fp16 of (8192,128256); {how}",
                       "l2": "inputs larger than L2, steps back to back"}
        self.launches_per_step = 2

    def _step(self):
        from fuselse_b200 import distributed as D
        if not self.nccl:
            self.out = self.ex(self.xs)
            return
        ms = self.ext.lse_partial(self.xs)
        if self.world > 1:
            self.out = self.ext.lse_combine(D.gather_partials(ms))
        else:
            self.out = self.ext.lse_combine(ms.unsqueeze(0))

    def kernels(self):
        return [("partial+combine", self._step, self.B * self.Ns * 2 + self.B * 8)]

    def rows(self):
        return self.B


class VocabSplit(Workload):
    """BASELINE's LLM-logit configuration split across the job: fp16 logits
    (8192, 128256) cut into `world` contiguous vocab shards, one per GPU (8 x
    16032 at 8 GPUs; the whole row on one GPU), every rank ending with the
    full (8192,) lse.  mode "nvlink": the library's exchange (fold + pair
    stores into every rank's buffer over NVLink + flag-wait combine, one
    call); mode "nccl": lse_partial, an NCCL all-gather of the (B, 2) pairs,
    lse_combine, timed separately; mode "fold": lse_partial alone (the
    shard's fold, no exchange)."""
    name = "vocab_split"
    dtype = "f16"
    B, V = 8192, 128256

    def __init__(self, dev, world, rank, mode, parts=None):
        from fuselse_b200 import distributed as D, ext, workloads as W
        self.ext, self.world, self.mode = ext, world, mode
        parts = parts or world
        full = W.fp16_logits(self.B, self.V, seed=0, device=dev)  # identical on every rank
        self.xs = W.vocab_shard(full, parts, rank % parts)
        del full
        torch.cuda.empty_cache()
        self.Ns = self.xs.size(1)
        self.ex = None
        if mode == "nvlink":
            self.ex = (D.VocabShardExchange(self.B, device=dev) if world > 1
                       else D.VocabShardExchange.single_rank(self.B, dev))
        self.launches_per_step = {"nvlink": 2, "nccl": 2, "fold": 1}[mode]

    def _exchange(self):
        self.out = self.ex(self.xs)

    def _partial(self):
        self.ms = self.ext.lse_partial(self.xs)

    def _gather(self):
        from fuselse_b200 import distributed as D
        self.allms = D.gather_partials(self.ms) if self.world > 1 else self.ms.unsqueeze(0)

    def _combine(self):
        self.out = self.ext.lse_combine(self.allms)

    def _combine1(self):
        self.out = self.ext.lse_combine(self.ms.unsqueeze(0))

    def kernels(self):
        shard = self.B * self.Ns * 2 + self.B * 4
        if self.mode == "nvlink":
            return [("exchange", self._exchange, shard)]
        if self.mode == "fold":
            return [("fold", self._partial, shard)]
        if self.world == 1:  # nothing to gather: the combine reads the one partial
            return [("partial", self._partial, shard), ("combine", self._combine1, 0)]
        return [("partial", self._partial, shard), ("all_gather", self._gather, 0),
                ("combine", self._combine, 0)]

    def close(self):
        if self.ex is not None and self.world > 1:
            self.ex.close()
        self.ex = None

    def rows(self):
        return self.B


def vocab_exchange_record(dev, world, rank, steps, warmup, dist_on):
    """The `vocab_exchange` key: BASELINE config 3 over `world` GPUs through the
    NVLink exchange and through the NCCL all-gather, with the shard's fold
    timed alone, and the whole (8192, 128256) on one GPU (t1) for reference."""
    total_bytes = VocabSplit.B * VocabSplit.V * 2 + VocabSplit.B * 4
    rec = {"config": "FuseLSE16 fp16 logits (8192,128256) x~N(0,3^2)+15 spike, split into "
                     f"{world} contiguous vocab shards of ~{-(-VocabSplit.V // world)} columns, "
                     "full lse on every rank",
           "algorithmic_bytes": total_bytes}
    out = {}
    for mode in ("fold", "nvlink", "nccl"):
        wl = VocabSplit(dev, world, rank, mode)
        _, per = run_timed(wl, steps, warmup, dev, dist_on)
        ms = run_step_graphs(wl, steps, warmup, dev, dist_on)
        wl.close()
        per = [max_over_ranks(v, dist_on, dev) for v in per]
        ms = max_over_ranks(ms, dist_on, dev)
        labels = [lab for lab, _, _ in wl.kernels()]
        out[mode] = (ms, dict(zip(labels, per)))
        del wl
        torch.cuda.empty_cache()
    fold_ms = out["fold"][0]
    nv_ms = out["nvlink"][0]
    nc_ms, nc_k = out["nccl"]
    rec["nvlink"] = {"ms": nv_ms, "GB_s": total_bytes / (nv_ms * 1e-3) / 1e9,
                     "shard_fold_us": fold_ms * 1e3,
                     "exchange_combine_us": (nv_ms - fold_ms) * 1e3,
                     "note": "one call (fold + NVLink pair stores, then flag-wait combine); "
                             "exchange_combine_us = call time - the shard's fold timed alone"}
    rec["nccl"] = {"ms": nc_ms, "GB_s": total_bytes / (nc_ms * 1e-3) / 1e9,
                   "partial_us": nc_k["partial"] * 1e3,
                   "all_gather_us": nc_k.get("all_gather", 0.0) * 1e3,
                   "combine_us": nc_k["combine"] * 1e3}
    if world > 1:
        # the same logits whole on one GPU (every rank its own copy), for the efficiency
        wl = VocabSplit(dev, 1, 0, "nvlink", parts=1)
        t1 = run_step_graphs(wl, steps, warmup, dev, dist_on)
        wl.close()
        del wl
        torch.cuda.empty_cache()
        t1 = max_over_ranks(t1, dist_on, dev)
        rec["t1_ms"] = t1
        rec["nvlink"]["efficiency_vs_1gpu"] = t1 / (world * nv_ms)
        rec["nccl"]["efficiency_vs_1gpu"] = t1 / (world * nc_ms)
    return rec


def strong_record(dev, world, rank, steps, warmup, dist_on, t1_ms):
    """The `strong` key: the headline's 512 rows split over the job's GPUs
    (64 rows each at 8 GPUs: rows split into cluster segments), forward +
    backward per step, max over ranks; t1_ms = this run's own 512-row step."""
    from fuselse_b200.distributed import split_range
    lo, hi = split_range(B_ROWS, world, rank)
    wl = FwdBwdF32(dev, seed=rank, B=hi - lo)
    ms = run_step_graphs(wl, steps, warmup, dev, dist_on)
    ms = max_over_ranks(ms, dist_on, dev)
    del wl
    torch.cuda.empty_cache()
    total = 3 * B_ROWS * N_COLS * 4 + 3 * B_ROWS * 4
    return {"config": f"FuseLSE fp32 fwd+bwd (512,128256) split over {world} GPU(s), "
                      f"{hi - lo} rows on rank {rank}",
            "ms_per_step": ms, "rows_per_s": B_ROWS / (ms * 1e-3),
            "GB_s": total / (ms * 1e-3) / 1e9, "t1_ms": t1_ms,
            "efficiency_vs_1gpu": t1_ms / (world * ms)}


class IntLSE(Workload):
    dtype = "int32"

    def __init__(self, dev, seed, kind="q16", B=16384, N=4096):
        from fuselse_b200 import ext, workloads as W
        self.ext, self.kind = ext, kind
        x, q16, q106 = W.intlse_inputs(B, N, seed, dev)
        self.q = q16 if kind == "q16" else q106
        self.name = "intlse_" + kind + ("" if (B, N) == (16384, 4096) else "_long")
        self.dtype = "int32" if kind == "q16" else "int16"
        self.B, self.N = B, N
        self.config = {"workload": f"IntLSE {kind} (B,N)=({B},{N}), x~N(0,2^2)",
                       "l2": "inputs larger than L2, steps back to back"}
        self.launches_per_step = 1

    def _step(self):
        if self.kind == "q16":
            self.out = self.ext.batched_logsumexp_q16_i32(self.q)
        else:
            self.out = self.ext.batched_logsumexp_q10_6(self.q)

    def kernels(self):
        return [(self.name, self._step, self.q.numel() * self.q.element_size() + self.B * 4)]

    def rows(self):
        return self.B


class Sparse(Workload):
    def __init__(self, dev, seed, q16=False):
        from fuselse_b200 import ext, workloads as W
        self.ext, self.q16 = ext, q16
        self.args = W.sparse_layer(seed=seed, device=dev)
        self.name = "sparse_q16" if q16 else "sparse_f32"
        self.dtype = "int32" if q16 else "f32"
        node, em, params, nids, cids, pids, _ = self.args
        P, batch = em.shape
        S, E = cids.shape
        self.bytes = P * batch * 4 + S * batch * 4 + S * E * (8 + 8 + 4) + S * 8
        self.S = S
        self.config = {"workload": f"sparse PC sum layer {'Q16.16' if q16 else 'fp32'}: P={P}, S={S}, "
                                   f"E={E}, batch={batch}", "l2": "inputs larger than L2, steps back to back"}
        self.launches_per_step = 1

    def _step(self):
        fn = self.ext.sparse_forward_q16 if self.q16 else self.ext.sparse_forward_float
        fn(*self.args)

    def kernels(self):
        return [(self.name, self._step, self.bytes)]

    def rows(self):
        return self.S


class SparseFwdBwd(Workload):
    """Sparse PC sum layer forward + backward (fp32) on the default layer:
    the forward kernel, then fl_sparse_f32_bwd (parameter gradients
    G and node_mars folded into one row per node; element and parameter
    gradients in one child-major pass over the parent index, which is built
    once, outside the timed region, like the workspace) with a fixed upstream
    gradient."""
    name = "sparse_fwdbwd_f32"
    dtype = "f32"

    def __init__(self, dev, seed):
        from fuselse_b200 import ext, workloads as W
        self.ext = ext
        self.args = W.sparse_layer(seed=seed, device=dev)
        node, em, params, nids, cids, pids, bs = self.args
        P, batch = em.shape
        S, E = cids.shape
        self.parents = ext.sparse_parent_index(nids, cids, pids, bs, P)
        g = torch.Generator(device=dev).manual_seed(seed + 3)
        self.G = torch.randn(node.shape, generator=g, device=dev)
        self.gem = torch.zeros_like(em)
        self.gw = torch.zeros_like(params)
        self.ws = torch.empty(ext.sparse_bwd_workspace_bytes(*node.shape, self.parents[1].numel()),
                              dtype=torch.uint8, device=dev)
        self.fwd_bytes = P * batch * 4 + S * batch * 4 + S * E * (8 + 8 + 4) + S * 8
        # em read, em grads read + written, node rows and their grads read,
        # param grads read + written, the edges' cids/pids, nids, and the
        # parent-unit index (child_ptr, unit node and parameter rows)
        self.bwd_bytes = (3 * P * batch * 4 + 2 * S * batch * 4 + S * E * (8 + 8 + 4 + 4 + 16)
                          + S * 8 + (P + 1) * 8)
        self.config = {"workload": f"sparse PC sum layer fp32 forward + backward: P={P}, S={S}, "
                                   f"E={E}, batch={batch}", "l2": "inputs larger than L2, steps back to back"}
        self.launches_per_step = 4

    def _fwd(self):
        self.ext.sparse_forward_float(*self.args)

    def _bwd(self):
        node, em, params, nids, cids, pids, bs = self.args
        self.ext.sparse_backward_float(node, self.G, em, params, nids, cids, pids, bs,
                                       element_grads=self.gem, param_grads=self.gw,
                                       parents=self.parents, workspace=self.ws)

    def kernels(self):
        return [("sparse_f32", self._fwd, self.fwd_bytes), ("sparse_bwd", self._bwd, self.bwd_bytes)]

    def rows(self):
        return self.args[4].size(0)


def make_workload(name, dev, seed, world, rank, same_input=False):
    if name == "fwdbwd_f32":
        return FwdBwdF32(dev, seed, same_input=same_input)
    if name == "fwd_f32":
        return FwdBwdF32(dev, seed, do_bwd=False, same_input=same_input)
    if name == "sls_f32":
        return SelectiveF32(dev, seed)
    if name == "f16_vocab":
        return F16Vocab(dev, seed, world, rank)
    if name == "f16_vocab_nccl":
        return F16Vocab(dev, seed, world, rank, nccl=True)
    if name == "intlse_q16":
        return IntLSE(dev, seed, "q16")
    if name == "intlse_q10_6":
        return IntLSE(dev, seed, "q10_6")
    if name == "intlse_q16_long":
        return IntLSE(dev, seed, "q16", B=64, N=1048576)
    if name == "intlse_q10_6_long":
        return IntLSE(dev, seed, "q10_6", B=64, N=1048576)
    if name == "sparse_f32":
        return Sparse(dev, seed, q16=False)
    if name == "sparse_q16":
        return Sparse(dev, seed, q16=True)
    if name == "sparse_fwdbwd_f32":
        return SparseFwdBwd(dev, seed)
    raise SystemExit(f"unknown workload {name}")


# ------------------------------------------------------------------ timing
class L2Flush:
    """Evicts L2 between timed steps: a 256 MiB write (> the 126 MB L2), then a
    256 MiB read of another buffer so the write's dirty lines are written back
    here, outside the timed events, instead of inside the next timed kernel."""

    def __init__(self, dev):
        n = 256 * 1024 * 1024 // 4
        self.w = torch.empty(n, dtype=torch.float32, device=dev)
        self.r = torch.ones(n, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()
        torch.sum(self.r, dim=0, out=self.sink)


def capture_graphs(fns, warmup):
    """Each callable captured into its own CUDA graph (one memory pool), after
    warm-up on the capture stream; returns the replay callables and the graphs."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graphs = []
    with torch.cuda.stream(s):
        for _ in range(warmup):
            for fn in fns:
                fn()
        pool = None
        for fn in fns:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s, pool=pool):
                fn()
            pool = g.pool()
            graphs.append(g)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    return [g.replay for g in graphs], graphs


def run_timed(wl, steps, warmup, dev, dist_on, flush_l2=False, graphs=True):
    """Steps back to back (inputs larger than L2), or with an untimed L2Flush
    between steps; every kernel launched from its own CUDA graph (host
    overhead off the device timeline) with CUDA events between them.  A
    workload with `phases` > 1 input batches cycles through them, step k
    running on batch k % phases."""
    flush = L2Flush(dev) if flush_l2 else (lambda: None)
    phases = getattr(wl, "phases", 1)
    sets, held = [], []
    for p in range(phases):
        if phases > 1:
            wl.set_phase(p)
        ks = wl.kernels()
        if graphs:
            fns, gs = capture_graphs([fn for _, fn, _ in ks], warmup)
            held += gs
            ks = [(lab, f, b) for (lab, _, b), f in zip(ks, fns)]
        sets.append(ks)
    ks = sets[0]
    for w in range(warmup):
        for _, fn, _ in sets[w % phases]:
            fn()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(ks) + 1)] for _ in range(steps)]
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    for k in range(steps):
        flush()
        evs[k][0].record()
        for i, (_, fn, _) in enumerate(sets[k % phases]):
            fn()
            evs[k][i + 1].record()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    per_kernel = [sum(evs[k][i].elapsed_time(evs[k][i + 1]) for k in range(steps)) / steps
                  for i in range(len(ks))]
    step_ms = sum(per_kernel)
    held.clear()  # graphs holding NCCL calls must go before the process group does
    return step_ms, per_kernel


def run_step_graphs(wl, steps, warmup, dev, dist_on, flush_l2=False):
    """Each step — all of its kernels, in order — replayed from ONE CUDA graph
    (one per input batch), with CUDA events at step boundaries only; returns
    the mean step time.  Per-kernel times come from run_timed."""
    flush = L2Flush(dev) if flush_l2 else (lambda: None)
    phases = getattr(wl, "phases", 1)
    steps_fns, held = [], []
    for p in range(phases):
        if phases > 1:
            wl.set_phase(p)
        ks = wl.kernels()

        def step(ks=ks):
            for _, fn, _ in ks:
                fn()

        fns, gs = capture_graphs([step], warmup)
        held += gs
        steps_fns.append(fns[0])
    for w in range(warmup):
        steps_fns[w % phases]()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    if flush_l2:
        times = []
        for k in range(steps):
            flush()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            steps_fns[k % phases]()
            b.record()
            times.append((a, b))
        torch.cuda.synchronize()
        step_ms = sum(a.elapsed_time(b) for a, b in times) / steps
    else:
        evs[0].record()
        for k in range(steps):
            steps_fns[k % phases]()
        evs[steps].record()
        torch.cuda.synchronize()
        step_ms = evs[0].elapsed_time(evs[steps]) / steps
    if dist_on:
        torch.distributed.barrier()
    held.clear()
    return step_ms


def run_e2e(wl, steps, warmup, dev, dist_on):
    wl.e2e_setup(dev)
    for _ in range(warmup):
        wl.e2e_step(dev)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s.record()
    for _ in range(steps):
        wl.e2e_step(dev)
    e.record()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    return s.elapsed_time(e) / steps


def copy_floor(wl, steps, dev, dist_on):
    """The e2e step's host-link floor: the same bytes copied alone — the step's
    input from pinned host memory to the device on one stream while a device
    buffer of the output's size goes back to pinned host memory on another,
    every rank at once (the GPUs share the host's memory and PCIe root) — no
    kernel.  Returns ms per step: the fastest of `steps` timed repetitions."""
    dst = torch.empty_like(wl.x)
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    cur = torch.cuda.current_stream()

    def once():
        up.wait_stream(cur)
        down.wait_stream(cur)
        with torch.cuda.stream(up):
            dst.copy_(wl.x_host, non_blocking=True)
        with torch.cuda.stream(down):
            wl.gx_host.copy_(wl.x, non_blocking=True)
        cur.wait_stream(up)
        cur.wait_stream(down)

    for _ in range(2):
        once()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    evs[0].record()
    for i in range(steps):
        once()
        evs[i + 1].record()
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    del dst
    # a bound: the fastest of the timed copies (one slow copy, e.g. a host page
    # fault or another tenant on the link, does not lower the floor)
    return min(evs[i].elapsed_time(evs[i + 1]) for i in range(steps))


def max_over_ranks(v, dist_on, dev):
    if not dist_on:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ CPU side
def cpu_fwdbwd_step(x_np, threads):
    """Reference FuseLSE-CPU forward (built from the reference source) + C-port backward."""
    from oracle import oracle as O
    if O.ref_available("ref_fused_cpu"):
        m = O.ref_ext("ref_fused_cpu")
        torch.set_num_threads(threads)
        lse = m.cpu_lse_float(torch.from_numpy(x_np)).numpy()
        kind = "reference"
    else:
        lse = O.fuselse_cpu_port(x_np, threads)
        kind = "port"
    g = np.ones(x_np.shape[0], np.float32)
    O.lse_bwd_port(g, x_np, lse, threads)
    return kind


def cpu_baseline(rows, budget_s=10.0):
    from oracle import oracle as O
    threads = O.host_threads()
    x = np.random.default_rng(0).standard_normal((rows, N_COLS)).astype(np.float32)
    kind = cpu_fwdbwd_step(x, threads)  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        cpu_fwdbwd_step(x, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    per = el / reps
    bytes_ = 3 * rows * N_COLS * 4 + 3 * rows * 4
    return {"value": bytes_ / per / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"fwd+bwd over ({rows},{N_COLS}) fp32 x~N(0,1), {reps} reps in {el:.1f} s; "
                      f"fwd = reference FuseLSE-CPU (fused_fp32_cpu.cpp) at::parallel_for, "
                      f"bwd = C port of grad*exp(x-lse), rows over {threads} threads",
            "rows_per_s": rows / per, "cpu": _cpu_name()}


def cpu_reference_configs(reps=5):
    """BASELINE's CPU configuration on this host: (32, 128256) fp32, x ~ N(0, 1)
    from torch.Generator().manual_seed(0): the reference AVX2 IntLSE
    (lse_q16_2d_simd, intlse/cpu/lse_kernel_simd.c:232-236, single-threaded by
    design; "all cores" = rows over a thread pool), the reference FuseLSE-CPU
    (cpu_lse_float, fuselse/cpu/fused_fp32_cpu.cpp:28-46, at::parallel_for)
    and torch.logsumexp, each on 1 thread and on all host threads; median of
    `reps` timed runs after one warm-up (benchmark.py:36-44's form)."""
    from oracle import oracle as O
    B, N = 32, 128256
    xt = torch.randn(B, N, generator=torch.Generator().manual_seed(0))
    x = xt.numpy()
    nbytes = B * N * 4 + B * 4
    allt = O.host_threads()
    saved = torch.get_num_threads()
    out = {"config": f"({B},{N}) fp32 x~N(0,1) seed 0", "host_threads": allt, "cpu": _cpu_name(),
           "reps": reps}

    def med(fn):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        ms = statistics.median(ts) * 1e3
        return {"ms": ms, "GB_s": nbytes / (ms * 1e-3) / 1e9}

    try:
        if O.ref_available("simd"):
            out["intlse_avx2_1t"] = med(lambda: O.ref_simd_rows(x, threads=1))
            out["intlse_avx2_all"] = med(lambda: O.ref_simd_rows(x, threads=allt))
        if O.ref_available("ref_fused_cpu"):
            m = O.ref_ext("ref_fused_cpu")
            torch.set_num_threads(1)
            out["fuselse_cpu_1t"] = med(lambda: m.cpu_lse_float(xt))
            torch.set_num_threads(allt)
            out["fuselse_cpu_all"] = med(lambda: m.cpu_lse_float(xt))
        torch.set_num_threads(1)
        out["torch_logsumexp_1t"] = med(lambda: torch.logsumexp(xt, -1))
        torch.set_num_threads(allt)
        out["torch_logsumexp_all"] = med(lambda: torch.logsumexp(xt, -1))
    finally:
        torch.set_num_threads(saved)
    return out


def _cpu_name():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    threads = O.host_threads()
    rows = B_ROWS
    x = np.random.default_rng(0).standard_normal((rows, N_COLS)).astype(np.float32)
    for _ in range(args.warmup):
        kind = cpu_fwdbwd_step(x, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        kind = cpu_fwdbwd_step(x, threads)
        times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    bytes_ = 3 * rows * N_COLS * 4 + 3 * rows * 4
    value = bytes_ / per / 1e9
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": HEADLINE_WORKLOAD, "B": rows, "N": N_COLS,
                       "device": f"host CPU, {threads} threads"},
            "rows_per_s": rows / per,
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": kind,
                             "sample": f"full ({rows},{N_COLS}) fwd+bwd per step; fwd = reference "
                                       "FuseLSE-CPU built from source, bwd = C port (the reference "
                                       "has no CPU backward)", "cpu": _cpu_name()},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="fwdbwd_f32")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the `strong` and `vocab_exchange` measurements")
    ap.add_argument("--flush-l2", action="store_true", help="evict L2 between timed steps")
    ap.add_argument("--kernel-graphs", action="store_true",
                    help="report the step as the sum of the per-kernel pass (a graph per kernel, "
                         "events between kernels) instead of the step pass (one graph per step)")
    ap.add_argument("--same-input", action="store_true",
                    help="fwd/bwd workloads: one input batch every step instead of two alternating")
    ap.add_argument("--eager", action="store_true",
                    help="launch the timed kernels eagerly instead of from CUDA graphs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist_on = world > 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if dist_on:
        from datetime import timedelta
        torch.distributed.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    wl = make_workload(args.workload, dev, seed=rank, world=world, rank=rank,
                       same_input=args.same_input)
    with ClockSampler(local) as clk:
        # per-kernel pass: a graph per kernel, CUDA events between kernels
        step_ms, per_kernel = run_timed(wl, args.steps, args.warmup, dev, dist_on, args.flush_l2,
                                        graphs=not args.eager)
        kernel_pass_ms = step_ms
        step_graph = not (args.eager or args.kernel_graphs)
        if step_graph:  # step pass: one graph per step, events at step boundaries
            step_ms = run_step_graphs(wl, args.steps, args.warmup, dev, dist_on, args.flush_l2)
    clocks = clk.summary()
    step_ms = max_over_ranks(step_ms, dist_on, dev)
    kernel_pass_ms = max_over_ranks(kernel_pass_ms, dist_on, dev)
    per_kernel = [max_over_ranks(v, dist_on, dev) for v in per_kernel]
    ks = wl.kernels()
    bytes_step = sum(b for _, _, b in ks)
    value = world * bytes_step / (step_ms * 1e-3) / 1e9
    peaks = measured_peaks()

    # dominant kernel roofline
    i_dom = int(np.argmax(per_kernel))
    lab, _, b_dom = ks[i_dom]
    ach = b_dom / (per_kernel[i_dom] * 1e-3) / 1e9
    roofline = {"bound": "hbm", "kernel": lab, "achieved": ach, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": ach / peaks["hbm_gbs"], "peak_source": peaks["source"],
                "traffic": profiled_traffic(lab)}
    kernels = {l: {"ms": t, "algorithmic_bytes": b, "GB_s": b / (t * 1e-3) / 1e9,
                   "frac_of_peak": b / (t * 1e-3) / 1e9 / peaks["hbm_gbs"]}
               for (l, _, b), t in zip(ks, per_kernel)}

    extra = {}
    if args.workload == "fwdbwd_f32" and not args.no_extra:
        # the forward kernel timed on its own (a graph per call, the two input
        # batches alternating): inside the step it also pays the write-back of
        # the backward's last gradient lines, still dirty in L2 when it starts
        wf = FwdBwdF32(dev, seed=rank, do_bwd=False)
        f_ms = max_over_ranks(run_step_graphs(wf, args.steps, args.warmup, dev, dist_on), dist_on, dev)
        del wf
        torch.cuda.empty_cache()
        fb = ks[0][2]
        kernels["fwd"]["in_step"] = ("inside the step the forward also writes back the backward's "
                                     "last gradient lines (~54 MB left dirty in L2)")
        kernels["fwd"]["alone"] = {"ms": f_ms, "GB_s": fb / (f_ms * 1e-3) / 1e9,
                                   "frac_of_peak": fb / (f_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                                   "how": "forward only, one graph per call, two input batches "
                                          "alternating, same run"}
        extra["strong"] = strong_record(dev, world, rank, args.steps, args.warmup, dist_on, step_ms)
        extra["vocab_exchange"] = vocab_exchange_record(dev, world, rank, args.steps, args.warmup,
                                                        dist_on)

    e2e = None
    if not args.no_e2e and hasattr(wl, "e2e_step"):
        e2e_ms = max_over_ranks(run_e2e(wl, max(3, args.steps // 4), 3, dev, dist_on), dist_on, dev)
        floor_ms = max_over_ranks(copy_floor(wl, 6, dev, dist_on), dist_on, dev)
        e2e = {"value": world * bytes_step / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": wl.h2d, "d2h_bytes_per_step": wl.d2h, "ms_per_step": e2e_ms,
               "api": getattr(wl, "e2e_api", "public API"),
               "copy_floor_ms": floor_ms,
               "copy_floor_value": world * bytes_step / (floor_ms * 1e-3) / 1e9,
               "copy_floor": "the step's input uploaded and a buffer of its output's size downloaded, "
                             "pinned host memory, concurrently on two streams, no kernel, all ranks "
                             "at once: the host link's bound on e2e"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "fwdbwd_f32":
        try:
            cpu = cpu_baseline(rows=B_ROWS)
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "error": repr(exc)}
        try:
            cpu["reference_cpu_configs"] = cpu_reference_configs()
        except Exception as exc:
            cpu["reference_cpu_configs"] = {"error": repr(exc)}

    if rank == 0:
        line = {"metric": METRIC if args.workload == "fwdbwd_f32" else f"{wl.name} HBM GB/s",
                "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
                "config": dict(wl.config, parallelism=f"rows x{world}" if world > 1 else "1 GPU",
                               launch=("eager" if args.eager else
                                       "one CUDA graph per step (all its kernels), events at step "
                                       "boundaries" if step_graph else "CUDA graph per kernel"),
                               l2_flush=bool(args.flush_l2)),
                "ms_per_step_kernel_pass": kernel_pass_ms,
                "rows_per_s": world * wl.rows() / (step_ms * 1e-3),
                "pct_of_peak": 100.0 * value / (world * peaks["hbm_gbs"]),
                "roofline": roofline, "kernels": kernels, "cpu_baseline": cpu, "e2e": e2e,
                "clocks": clocks, "gpu_launches": wl.launches_per_step * args.steps,
                "gpu": torch.cuda.get_device_name(dev), **extra}
        print(json.dumps(line), flush=True)
    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
