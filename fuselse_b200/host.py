"""Host-resident rows: log-sum-exp forward + backward straight from pinned host memory.

The reference's entry points take CUDA tensors, so a caller holding logits in
host memory copies them in, runs the kernels and copies the results out, one
after the other.  `HostRowPipeline` does the same work with the copies hidden:
the rows go through the GPU in chunks on three streams, so chunk k+1 is
uploaded while chunk k is reduced and chunk k-1's results are downloaded (the
PCIe link carries both directions at once).  The kernels are the library's
own (fl_lse_f32_fwd / fl_lse_f32_bwd through the C ABI); each call starts
after the work already queued on the caller's current stream and the current
stream waits for the call's last download, so the call is ordered like any
other operation on that stream.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib


class HostRowPipeline:
    """Chunked, copy-overlapped forward (+ backward) over rows of N fp32 values
    held in pinned host memory.  Device buffers for `depth` chunks of
    `chunk_rows` rows (by default about 16 MB of rows: 32 rows of 128256) are
    allocated once and reused by every call; the (B,) vectors g and lse grow
    once to the largest B seen and go up / come down in one copy per call.
    (Measured on B200 for (512, 128256) forward + backward: 32-row chunks
    5.97 ms per call, 64-row 6.05 ms, 128-row 6.50 ms; a copy of g and lse per
    chunk cost a further 0.25-0.5 ms.)"""

    def __init__(self, N: int, device=None, chunk_rows: int | None = None, depth: int = 3,
                 robust: bool = True):
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if chunk_rows is None:
            chunk_rows = max(1, (16 << 20) // (4 * max(N, 1)))
        self.N, self.rows, self.depth, self.robust = N, chunk_rows, depth, robust
        f = dict(dtype=torch.float32, device=self.device)
        self.x = [torch.empty(chunk_rows, N, **f) for _ in range(depth)]
        self.gx = [torch.empty(chunk_rows, N, **f) for _ in range(depth)]
        self.g = torch.empty(0, **f)
        self.lse = torch.empty(0, **f)
        self.up, self.comp, self.down = (torch.cuda.Stream(self.device) for _ in range(3))
        self.free = [torch.cuda.Event() for _ in range(depth)]

    def _check(self, t: torch.Tensor, shape, name: str):
        if not (t.device.type == "cpu" and t.dtype == torch.float32 and t.is_contiguous()
                and tuple(t.shape) == tuple(shape)):
            raise RuntimeError(f"{name} must be a contiguous fp32 host tensor of shape {tuple(shape)}")
        if not t.is_pinned():
            raise RuntimeError(f"{name} must be in pinned host memory")

    def run(self, x_host: torch.Tensor, lse_host: torch.Tensor, g_host: torch.Tensor = None,
            gx_host: torch.Tensor = None) -> None:
        """lse_host[b] = LSE(x_host[b, :]); with g_host and gx_host also
        gx_host = g_host[:, None] * exp(x_host - lse[:, None]).  All four are
        pinned fp32 host tensors; the results are in place once the caller's
        current stream has reached this point (e.g. after synchronize)."""
        B = x_host.shape[0] if x_host.dim() == 2 else -1
        self._check(x_host, (B, self.N), "x_host")
        self._check(lse_host, (B,), "lse_host")
        bwd = g_host is not None
        if bwd != (gx_host is not None):
            raise RuntimeError("g_host and gx_host go together")
        if bwd:
            self._check(g_host, (B,), "g_host")
            self._check(gx_host, (B, self.N), "gx_host")
        if B == 0:
            return
        if self.lse.numel() < B:
            self.lse = torch.empty(B, dtype=torch.float32, device=self.device)
            self.g = torch.empty(B, dtype=torch.float32, device=self.device)
        cur = torch.cuda.current_stream(self.device)
        self.up.wait_stream(cur)
        if bwd:
            with torch.cuda.stream(self.up):
                self.g[:B].copy_(g_host, non_blocking=True)
        N = self.N
        for i, r0 in enumerate(range(0, B, self.rows)):
            n = min(self.rows, B - r0)
            k = i % self.depth
            xs, gxs = self.x[k], self.gx[k]
            if i >= self.depth:
                self.up.wait_event(self.free[k])  # slot k's last download is done
            with torch.cuda.stream(self.up):
                xs[:n].copy_(x_host[r0:r0 + n], non_blocking=True)
            self.comp.wait_stream(self.up)
            s = ctypes.c_void_p(self.comp.cuda_stream)
            ls = self.lse[r0:r0 + n]
            _lib.call("fl_lse_f32_fwd", _lib.ptr(xs), _lib.ptr(ls), n, N, int(self.robust), s)
            if bwd:
                _lib.call("fl_lse_f32_bwd", _lib.ptr(self.g[r0:r0 + n]), _lib.ptr(xs), _lib.ptr(ls),
                          _lib.ptr(gxs), n, N, s)
                self.down.wait_stream(self.comp)
                with torch.cuda.stream(self.down):
                    gx_host[r0:r0 + n].copy_(gxs[:n], non_blocking=True)
            else:
                self.down.wait_stream(self.comp)
            self.free[k].record(self.down)
        self.down.wait_stream(self.comp)
        with torch.cuda.stream(self.down):
            lse_host.copy_(self.lse[:B], non_blocking=True)
        cur.wait_stream(self.down)


def logsumexp_fwd_bwd_host(x_host: torch.Tensor, g_host: torch.Tensor, robust: bool = True,
                           chunk_rows: int | None = None):
    """One-shot form: (lse_host, gx_host) for pinned fp32 host rows, synchronised."""
    B, N = x_host.shape
    pipe = HostRowPipeline(N, chunk_rows=chunk_rows, robust=robust)
    lse = torch.empty(B, dtype=torch.float32).pin_memory()
    gx = torch.empty(B, N, dtype=torch.float32).pin_memory()
    pipe.run(x_host, lse, g_host, gx)
    torch.cuda.current_stream(pipe.device).synchronize()
    return lse, gx
