"""Oracle API — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker (or the timed CPU baseline); the product never does.

  * integer paths: the C restatement in lse_oracle.c (bit-exact reference order);
  * float paths: float64 numpy evaluation of log(sum(exp(x))) with the
    reference's IEEE rules (run_microbenchmark.py:141-146 uses the same fp64
    max-shifted form);
  * reference builds in oracle/_ref (built by oracle/build.py from the
    reference sources): the AVX2 IntLSE library, the FuseLSE-CPU extension and
    the six GPU extensions, loadable on the GPU box without the sources.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import sys
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_void_p
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liblse_oracle.so"
REF_DIR = HERE / "_ref"

Q16_F32, Q16_I32, Q10_6_I16 = 0, 1, 2
Q_NEG_INF = -0x3FFFFFFF

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            from .build import build_oracle
            build_oracle()
        L = ctypes.CDLL(str(ORACLE_SO))
        L.orc_pair_q16.argtypes = [c_int32, c_int32, c_int]
        L.orc_pair_q16.restype = c_int32
        L.orc_pair_q10_6.argtypes = [c_int32, c_int32]
        L.orc_pair_q10_6.restype = c_int32
        L.orc_pair_q16_capped.argtypes = [c_int32, c_int32]
        L.orc_pair_q16_capped.restype = c_int32
        L.orc_f2i_rn.argtypes = [c_float]
        L.orc_f2i_rn.restype = c_int32
        L.orc_f32_to_q16.argtypes = [c_float]
        L.orc_f32_to_q16.restype = c_int32
        L.orc_intlse_rows.argtypes = [c_int, c_int, c_void_p, c_int64, c_int64, c_int,
                                      POINTER(c_float), POINTER(c_int32)]
        L.orc_intlse_rows.restype = None
        L.orc_sparse_q16.argtypes = [POINTER(c_float), POINTER(c_float), POINTER(c_float),
                                     POINTER(c_int64), POINTER(c_int64), c_int64, c_int64,
                                     c_int64, c_int64]
        L.orc_sparse_q16.restype = None
        L.orc_simd_q16_rows.argtypes = [POINTER(c_float), c_int, c_int, POINTER(c_float)]
        L.orc_simd_q16_rows.restype = None
        L.orc_fuselse_cpu_rows.argtypes = [POINTER(c_float), c_int64, c_int64, c_int64,
                                           POINTER(c_float)]
        L.orc_fuselse_cpu_rows.restype = None
        L.orc_lse_bwd_rows.argtypes = [POINTER(c_float)] * 4 + [c_int64, c_int64, c_int64]
        L.orc_lse_bwd_rows.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray, ct=c_float):
    return a.ctypes.data_as(POINTER(ct))


# ---------------------------------------------------------------- integer paths
def intlse_rows(x: np.ndarray, kind: int, use_lut: bool = True, base_phase: int = 0):
    """Reference GPU-order IntLSE of a dense (B, N) array whose first element
    sits at device address phase `base_phase` (address mod 16).
    Returns (out float32 (B,), acc int32 (B,))."""
    dt = {Q16_F32: np.float32, Q16_I32: np.int32, Q10_6_I16: np.int16}[kind]
    x = np.ascontiguousarray(x, dtype=dt)
    B, N = x.shape
    out = np.empty(B, np.float32)
    acc = np.empty(B, np.int32)
    lib().orc_intlse_rows(kind, int(use_lut), x.ctypes.data_as(c_void_p), B, N, base_phase,
                          _p(out), _p(acc, c_int32))
    return out, acc


def f32_to_q16(x: np.ndarray) -> np.ndarray:
    """Elementwise __float2int_rn(x * CONV) (lse_kernel.cu:114)."""
    f = np.vectorize(lambda v: lib().orc_f32_to_q16(float(v)), otypes=[np.int32])
    return f(np.asarray(x, np.float32))


def pair_q16(a: int, b: int, use_lut: bool = True) -> int:
    return lib().orc_pair_q16(a, b, int(use_lut))


def pair_q10_6(a: int, b: int) -> int:
    return lib().orc_pair_q10_6(a, b)


def sparse_q16(node_mars: np.ndarray, element_mars: np.ndarray, logw: np.ndarray,
               nids: np.ndarray, cids: np.ndarray, block_size: int) -> np.ndarray:
    """Sparse Q16.16 layer with device-formed log-weights logw (num_nblocks*block_size, E).
    Writes into (a copy of) node_mars and returns it."""
    out = np.array(node_mars, np.float32, copy=True, order="C")
    em = np.ascontiguousarray(element_mars, np.float32)
    lw = np.ascontiguousarray(logw, np.float32)
    nids = np.ascontiguousarray(nids, np.int64)
    cids = np.ascontiguousarray(cids, np.int64)
    K, E = cids.shape
    lib().orc_sparse_q16(_p(out), _p(em), _p(lw), _p(nids, c_int64), _p(cids, c_int64), K, E,
                         out.shape[1], block_size)
    return out


def simd_q16_rows(x: np.ndarray) -> np.ndarray:
    """AVX2 CPU IntLSE order (lse_kernel_simd.c:166-236) restated."""
    x = np.ascontiguousarray(x, np.float32)
    B, N = x.shape
    out = np.empty(B, np.float32)
    lib().orc_simd_q16_rows(_p(x), B, N, _p(out))
    return out


# ---------------------------------------------------------------- float paths
def lse_f64(x: np.ndarray) -> np.ndarray:
    """fp64 log-sum-exp over the last axis with the robust IEEE rules:
    NaN anywhere -> NaN, else +inf -> +inf, all -inf (or empty) -> -inf."""
    x = np.asarray(x, np.float64)
    if x.shape[-1] == 0:
        return np.full(x.shape[:-1], -np.inf)
    with np.errstate(invalid="ignore", over="ignore"):
        m = np.max(x, axis=-1)
        has_nan = np.isnan(x).any(axis=-1)
        ms = np.where(np.isfinite(m), m, 0.0)
        s = np.sum(np.exp(x - ms[..., None]), axis=-1)
        with np.errstate(divide="ignore"):
            r = ms + np.log(s)
    r = np.where(m == np.inf, np.inf, r)
    r = np.where(m == -np.inf, -np.inf, r)
    r = np.where(has_nan, np.nan, r)
    return r


def lse_bwd_f64(g: np.ndarray, x: np.ndarray, lse: np.ndarray) -> np.ndarray:
    """grad_input = g[:, None] * exp(x - lse[:, None]) in fp64."""
    x = np.asarray(x, np.float64)
    with np.errstate(invalid="ignore", over="ignore"):
        return np.asarray(g, np.float64)[:, None] * np.exp(x - np.asarray(lse, np.float64)[:, None])


def selective_f64(x: np.ndarray, index: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(logp, lse) in fp64: logp[b] = x[b, index[b]] - LSE(x[b, :]) — the value of
    trl.trainer.utils.selective_log_softmax (trl 1.0.0) as run_rlhf.py:145-157 calls
    it; an index outside [0, N) gives NaN."""
    x = np.asarray(x, np.float64)
    index = np.asarray(index, np.int64)
    lse = lse_f64(x)
    ok = (index >= 0) & (index < x.shape[-1])
    picked = np.take_along_axis(x, np.where(ok, index, 0)[..., None], -1)[..., 0]
    with np.errstate(invalid="ignore"):
        logp = np.where(ok, picked - lse, np.nan)
    return logp, lse


def selective_bwd_f64(g: np.ndarray, x: np.ndarray, lse: np.ndarray, index: np.ndarray) -> np.ndarray:
    """d logp / d x scaled by g: g[b] * (onehot(index[b]) - exp(x - lse)) in fp64;
    an index outside [0, N) adds no one-hot term."""
    gx = -lse_bwd_f64(g, x, lse)
    g = np.asarray(g, np.float64)
    index = np.asarray(index, np.int64)
    rows = np.nonzero((index >= 0) & (index < gx.shape[-1]))[0]
    gx[rows, index[rows]] += g[rows]
    return gx


def sparse_f64(node_mars, element_mars, params, nids, cids, pids, block_size, floor=1e-45):
    """fp64 sparse layer: LSE_e(log(max(w, floor)) + child) for every output row
    (the formula of run_pyjuice.py:90-119, with the kernels' 1e-45 floor)."""
    out = np.array(node_mars, np.float64, copy=True)
    em = np.asarray(element_mars, np.float64)
    w = np.asarray(params, np.float64)
    K, E = cids.shape
    for p in range(block_size):
        lw = np.log(np.maximum(w[pids + p], floor))          # (K, E)
        logits = em[cids] + lw[:, :, None]                   # (K, E, batch)
        out[nids + p] = lse_f64(np.moveaxis(logits, 1, -1))
    return out


# ---------------------------------------------------------------- CPU baseline (C port)
def sparse_bwd_f64(node_mars, node_grads, element_mars, params, nids, cids, pids, block_size,
                   floor=1e-45):
    """fp64 gradient of the sparse layer (the reference has a forward only):
    element grads sum over edges G[n] * w * exp(em[c] - nm[n]) into row c,
    param grads sum over the batch G[n] * exp(em[c] - nm[n]) into params[q]
    (0 for weights at or below the floor); nodes with nm = -inf pass nothing."""
    nm = np.asarray(node_mars, np.float64)
    G = np.asarray(node_grads, np.float64)
    em = np.asarray(element_mars, np.float64)
    w = np.asarray(params, np.float64)
    gem = np.zeros_like(em)
    gw = np.zeros_like(w)
    K, E = cids.shape
    for p in range(block_size):
        n = nids + p                                          # (K,)
        q = pids + p                                          # (K, E)
        lw = np.log(np.maximum(w[q], floor))                  # (K, E)
        dead = np.isneginf(nm[n])                             # (K, batch)
        Gn = np.where(dead, 0.0, G[n])
        with np.errstate(invalid="ignore", over="ignore"):
            d = em[cids] - np.where(dead, 0.0, nm[n])[:, None, :]  # (K, E, batch)
            r = Gn[:, None, :] * np.exp(d)
        r = np.where(Gn[:, None, :] == 0.0, 0.0, r)
        np.add.at(gem, cids.reshape(-1), (np.exp(lw)[:, :, None] * r).reshape(K * E, -1))
        np.add.at(gw, q.reshape(-1), np.where(w[q] > floor, r.sum(-1), 0.0).reshape(-1))
    return gem, gw


def fuselse_cpu_port(x: np.ndarray, threads: int = 1) -> np.ndarray:
    """Reference FuseLSE-CPU pair chain, restated in C; rows split over threads."""
    x = np.ascontiguousarray(x, np.float32)
    B, N = x.shape
    out = np.empty(B, np.float32)
    _rows_parallel(lambda r0, r1: lib().orc_fuselse_cpu_rows(_p(x), N, r0, r1, _p(out)), B, threads)
    return out


def lse_bwd_port(g, x, lse, threads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    g = np.ascontiguousarray(g, np.float32)
    lse = np.ascontiguousarray(lse, np.float32)
    B, N = x.shape
    gx = np.empty_like(x)
    _rows_parallel(lambda r0, r1: lib().orc_lse_bwd_rows(_p(g), _p(x), _p(lse), _p(gx), N, r0, r1),
                   B, threads)
    return gx


def _rows_parallel(fn, B: int, threads: int) -> None:
    threads = max(1, min(threads, B))
    if threads == 1:
        fn(0, B)
        return
    bounds = [(B * i // threads, B * (i + 1) // threads) for i in range(threads)]
    with ThreadPoolExecutor(threads) as ex:  # ctypes releases the GIL
        list(ex.map(lambda rr: fn(*rr), bounds))


def host_threads() -> int:
    return len(os.sched_getaffinity(0))


# ---------------------------------------------------------------- reference builds
def ref_available(name: str) -> bool:
    if name == "simd":
        return (REF_DIR / "lse_kernel_simd.so").exists()
    return (REF_DIR / name / f"{name}.so").exists()


_ref_simd = None


def ref_simd() -> ctypes.CDLL:
    """The reference AVX2 IntLSE library (intlse/cpu/lse_kernel_simd.c), built from source."""
    global _ref_simd
    if _ref_simd is None:
        L = ctypes.CDLL(str(REF_DIR / "lse_kernel_simd.so"))
        L.lse_q16_2d_simd.argtypes = [POINTER(c_float), c_int, c_int, POINTER(c_float)]
        L.lse_q16_2d_simd.restype = None
        L.lse_q16_2d_simd_neg_inf.argtypes = [POINTER(c_float), c_int, c_int, POINTER(c_float)]
        L.lse_q16_2d_simd_neg_inf.restype = None
        _ref_simd = L
    return _ref_simd


def ref_simd_rows(x: np.ndarray, threads: int = 1, neg_inf: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    B, N = x.shape
    out = np.empty(B, np.float32)
    f = ref_simd().lse_q16_2d_simd_neg_inf if neg_inf else ref_simd().lse_q16_2d_simd

    def run(r0, r1):
        f(_p(x[r0:r1]), r1 - r0, N, _p(out[r0:r1]))

    _rows_parallel(run, B, threads)
    return out


_ref_mods: dict = {}


def ref_ext(name: str):
    """A reference torch extension from oracle/_ref (torch must be importable)."""
    if name not in _ref_mods:
        import torch  # noqa: F401  (extension symbols resolve against libtorch)
        path = REF_DIR / name / f"{name}.so"
        if not path.exists():
            raise FileNotFoundError(f"reference build {path} missing; run python -m oracle.build")
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _ref_mods[name] = mod
    return _ref_mods[name]
