"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configurations (no dataset is involved; every input is generated on the device).

  fp32 rows      x ~ N(0, 1), (B, N) = (512, 128256) / (512, 256)
  robust rows    same x, 1% of entries -inf, row 0 all -inf, row 1 one +inf and one NaN
  fp16 logits    x ~ N(0, 3^2) plus +15 at one random column per row, cast to fp16,
                 (8192, 128256) split into 8 contiguous vocab shards of 16032
  IntLSE         x ~ N(0, 2^2); Q16.16 int32 = round(x * 65536),
                 Q10.6 int16 = clamp(round(x * 64), -32768, 32767)
  sparse layer   element_mars (P, batch) ~ N(-20, 5^2); S sum nodes with E children
                 drawn uniformly without replacement from [0, P); weights
                 Dirichlet(1) per node; block_size 1, nids = arange(S),
                 pids = arange(S*E).view(S, E)
"""
from __future__ import annotations

import torch


def _gen(seed: int, device) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def fp32_rows(B: int, N: int, seed: int = 0, device="cuda") -> torch.Tensor:
    return torch.randn(B, N, generator=_gen(seed, device), device=device)


def robust_rows(B: int, N: int, seed: int = 0, device="cuda") -> torch.Tensor:
    x = fp32_rows(B, N, seed, device)
    mask = torch.rand(B, N, generator=_gen(1, device), device=device) < 0.01
    x[mask] = float("-inf")
    x[0] = float("-inf")
    if B > 1 and N > 1:
        x[1, 0] = float("inf")
        x[1, N - 1] = float("nan")
    return x


def fp16_logits(B: int, N: int, seed: int = 0, device="cuda") -> torch.Tensor:
    g = _gen(seed, device)
    x = torch.randn(B, N, generator=g, device=device) * 3.0
    col = torch.randint(0, N, (B,), generator=g, device=device)
    x[torch.arange(B, device=device), col] += 15.0
    return x.half()


def vocab_shard(x: torch.Tensor, shards: int, index: int) -> torch.Tensor:
    """Contiguous column block `index` of `shards`, materialised contiguous."""
    from .distributed import split_range
    lo, hi = split_range(x.size(1), shards, index)
    return x[:, lo:hi].contiguous()


def intlse_inputs(B: int, N: int, seed: int = 0, device="cuda"):
    x = torch.randn(B, N, generator=_gen(seed, device), device=device) * 2.0
    q16 = (x * 65536.0).round().to(torch.int32)
    q106 = (x * 64.0).round().clamp(-32768, 32767).to(torch.int16)
    return x, q16, q106


def sample_children(S: int, E: int, P: int, seed: int = 0, device="cuda") -> torch.Tensor:
    """(S, E) int64: each row E distinct indices uniform over [0, P) (row-wise rejection)."""
    if E > P:
        raise ValueError("more children than elements")
    g = _gen(seed, device)
    c = torch.randint(0, P, (S, E), generator=g, device=device)
    while True:
        s, _ = torch.sort(c, dim=1)
        dup = (s[:, 1:] == s[:, :-1]).any(dim=1)
        n = int(dup.sum())
        if n == 0:
            return c
        c[dup] = torch.randint(0, P, (n, E), generator=g, device=device)


def sparse_layer(P: int = 262144, S: int = 65536, E: int = 32, batch: int = 512, seed: int = 0,
                 device="cuda"):
    """Returns node_mars (S, batch) zeros, element_mars, params, nids, cids, pids, block_size."""
    g = _gen(seed, device)
    em = torch.randn(P, batch, generator=g, device=device) * 5.0 - 20.0
    cids = sample_children(S, E, P, seed + 1, device)
    gam = -torch.log(torch.rand(S, E, generator=g, device=device).clamp_min(1e-30))  # Gamma(1)
    params = (gam / gam.sum(dim=1, keepdim=True)).reshape(-1).contiguous()       # Dirichlet(1)
    nids = torch.arange(S, device=device)
    pids = torch.arange(S * E, device=device).view(S, E)
    node_mars = torch.zeros(S, batch, device=device)
    return node_mars, em, params, nids, cids, pids, 1
