"""Build recipe for the oracle (TEST INFRASTRUCTURE ONLY).

    python -m oracle.build            # oracle C restatement + reference builds
    python -m oracle.build --no-ref   # oracle only

1. oracle/lse_oracle.c -> oracle/_build/liblse_oracle.so (gcc, strict IEEE:
   no fast-math, no FMA contraction).
2. When the reference sources are present (this container, not the GPU box),
   the reference's own files are compiled where they lie into oracle/_ref/:
     - intlse/cpu/lse_kernel_simd.c      -> lse_kernel_simd.so (gcc, AVX2/FMA)
     - fuselse/cpu/fused_fp32_cpu.cpp    -> torch extension (g++, OpenMP)
     - the six GPU .cu files             -> torch extensions for sm_100a,
       with the reference's flags (-O3 --use_fast_math)
   The built files travel to the GPU box with the repository snapshot; nothing
   there reads the reference sources.  Sources are never copied.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
ORACLE_SO = BUILD / "liblse_oracle.so"
# the reference checkout: FUSELSE_REFERENCE, else a `reference` directory
# beside this repository's root
REF_SRC = Path(os.environ.get("FUSELSE_REFERENCE", HERE.parent.parent / "reference"))

# reference GPU sources -> extension module names
REF_CUDA = {
    "ref_fused_fp32": "fuselse/gpu/fused_fp32_kernel.cu",
    "ref_fused_fp16": "fuselse/gpu/fused_fp16_kernel.cu",
    "ref_lse_q16": "intlse/gpu/lse_kernel.cu",
    "ref_lse_q10_6": "intlse/gpu/lse_kernel_q10_6.cu",
    "ref_sparse_float": "experiment_pyjuice/sparse_float_kernel.cu",
    "ref_sparse_q16": "experiment_pyjuice/sparse_q16_kernel.cu",
}
REF_CPU_EXT = {"ref_fused_cpu": "fuselse/cpu/fused_fp32_cpu.cpp"}
REF_SIMD_SO = REF_OUT / "lse_kernel_simd.so"


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"command failed: {' '.join(map(str, cmd))}")


def build_oracle() -> Path:
    BUILD.mkdir(exist_ok=True)
    src = HERE / "lse_oracle.c"
    if ORACLE_SO.exists() and ORACLE_SO.stat().st_mtime > src.stat().st_mtime:
        return ORACLE_SO
    _run(["gcc", "-O2", "-fPIC", "-shared", "-fno-fast-math", "-ffp-contract=off",
          "-std=c11", "-o", str(ORACLE_SO), str(src), "-lm"])
    return ORACLE_SO


def ext_path(name: str) -> Path:
    return REF_OUT / name / f"{name}.so"


def _build_torch_ext(name: str, src: Path, cuda: bool) -> None:
    out = ext_path(name)
    if out.exists():
        return
    os.environ["CXX"] = "/usr/bin/g++"  # the /opt/gcc wrapper lacks libgomp.spec
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import load

    bdir = REF_OUT / name
    bdir.mkdir(parents=True, exist_ok=True)
    kw = dict(name=name, sources=[str(src)], build_directory=str(bdir), verbose=False)
    if cuda:
        kw["extra_cuda_cflags"] = ["-O3", "--use_fast_math",
                                   "-gencode", "arch=compute_100a,code=sm_100a"]
    else:
        kw["extra_cflags"] = ["-O3", "-mavx2", "-mfma", "-fopenmp"]
        kw["extra_ldflags"] = ["-fopenmp"]
    load(**kw)
    if not out.exists():
        raise RuntimeError(f"reference extension {name} did not produce {out}")


def build_ref() -> bool:
    """Build what the reference sources give; False if they are absent."""
    if not (REF_SRC / "intlse" / "cpu" / "lse_kernel_simd.c").exists():
        return False
    REF_OUT.mkdir(exist_ok=True)
    if not REF_SIMD_SO.exists():
        _run(["gcc", "-O3", "-fPIC", "-shared", "-mavx2", "-mfma",
              str(REF_SRC / "intlse/cpu/lse_kernel_simd.c"), "-o", str(REF_SIMD_SO), "-lm"])
    jobs = [(name, str(REF_SRC / rel), False) for name, rel in REF_CPU_EXT.items()]
    jobs += [(name, str(REF_SRC / rel), True) for name, rel in REF_CUDA.items()]
    jobs = [j for j in jobs if not ext_path(j[0]).exists()]
    if len(jobs) <= 1:
        for j in jobs:
            _build_torch_ext(j[0], Path(j[1]), j[2])
        return True
    # independent extensions: one worker process each (spawned, so no CUDA or
    # torch state is inherited), as many at a time as there are cores
    import multiprocessing as mp
    from concurrent.futures import ProcessPoolExecutor
    workers = max(1, min(len(jobs), os.cpu_count() or 1))
    with ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn")) as pool:
        for f in [pool.submit(_build_torch_ext_job, *j) for j in jobs]:
            f.result()
    return True


def _build_torch_ext_job(name: str, src: str, cuda: bool) -> None:
    _build_torch_ext(name, Path(src), cuda)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--no-ref", action="store_true")
    a = ap.parse_args()
    print(build_oracle())
    if not a.no_ref:
        print("reference built" if build_ref() else "reference sources absent")
