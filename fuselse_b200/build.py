"""Build recipe for libfuselse_b200.so (sm_100a), in-tree.

    python -m fuselse_b200.build [--verbose] [--ptxas-info]
    python -m fuselse_b200.build --define FL_FLAT_ROWS=2 --out /tmp/v/libfuselse_b200.so

Each csrc/*.cu is compiled with nvcc for `-gencode arch=compute_100a,code=sm_100a`
into build objects under fuselse_b200/_build/, then linked into
fuselse_b200/libfuselse_b200.so (CUDA runtime linked statically, so the
library only needs the driver).  Objects are rebuilt when their source or a
header changed.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libfuselse_b200.so"
HEADERS = [ROOT / "include" / "fuselse_b200.h", *sorted(CSRC.glob("*.cuh"))]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "-I", str(ROOT / "include")]
# Per-file extra flags.  sparse.cu matches the reference kernels' fast-math
# build so its log-weights and Q16.16 conversions round identically.
EXTRA = {"sparse.cu": ["--use_fast_math"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin on PATH")


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *HEADERS])


def _compile(cc: str, src: Path, obj: Path, verbose: bool, ptxas_info: bool, defines=()):
    cmd = [cc, *ARCH, *COMMON, *EXTRA.get(src.name, []), *(f"-D{d}" for d in defines),
           "-c", str(src), "-o", str(obj)]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, cmd, r


def build(verbose: bool = False, ptxas_info: bool = False, defines=(), out: Path | None = None) -> Path:
    """Build the library.  `defines` (NAME=VALUE strings, e.g. the FL_* shape
    macros of csrc/*.cuh) build a variant instead: every source is compiled with
    them into a build folder of its own beside `out`, which must then name the
    variant library (the in-tree library is left as it is)."""
    defines = tuple(defines)
    if defines and out is None:
        raise ValueError("a build with defines needs an output path of its own")
    lib = Path(out) if out is not None else LIB
    build_dir = BUILD if out is None else lib.parent / (lib.stem + "_build")
    build_dir.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    objs, todo = [], []
    for src in sorted(CSRC.glob("*.cu")):
        obj = build_dir / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, src) or ptxas_info or defines:
            todo.append((src, obj))
    # the translation units are independent: compile them side by side
    workers = max(1, min(len(todo), os.cpu_count() or 1))
    failed = []
    with ThreadPoolExecutor(max_workers=workers) as pool:
        for src, cmd, r in pool.map(lambda t: _compile(cc, t[0], t[1], verbose, ptxas_info, defines),
                                    todo):
            if verbose:
                print(" ".join(cmd), flush=True)
            if r.returncode != 0 or verbose or ptxas_info:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed on {', '.join(failed)}")
    if not lib.exists() or any(o.stat().st_mtime > lib.stat().st_mtime for o in objs):
        tmp = lib.with_suffix(".so.tmp")
        cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("linking libfuselse_b200.so failed")
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills per kernel")
    ap.add_argument("--define", action="append", default=[], metavar="NAME=VALUE",
                    help="build a variant with this macro (repeatable; needs --out)")
    ap.add_argument("--out", default=None, help="variant library path (load it with FUSELSE_B200_LIB)")
    args = ap.parse_args()
    print(build(verbose=args.verbose, ptxas_info=args.ptxas_info, defines=args.define,
                out=Path(args.out) if args.out else None))
