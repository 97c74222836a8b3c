"""Multi-GPU path on real GPUs: NCCL vocab-shard combine and batch-row sharding
against the single-GPU kernels (tests/dist_worker.py under torchrun).
Skipped when fewer than two GPUs are visible."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_paths_match_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_port()), str(ROOT / "tests" / "dist_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT,
                       env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    # the workers' own error lines first (torchrun's summary follows them)
    errors = [l for l in r.stderr.splitlines() if "Error" in l and "elastic" not in l]
    assert r.returncode == 0, "\n".join(errors[:20]) + "\n" + r.stdout[-2000:] + r.stderr[-2000:]
    assert f"dist ok: world {world}" in r.stdout
