import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")
    config.addinivalue_line("markers", "slow: full-size configurations")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def dev():
    import torch
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ext():
    import fuselse_b200
    return fuselse_b200.ext


def ref_ext_or_skip(name: str):
    from oracle import oracle as O
    if not O.ref_available(name):
        pytest.skip(f"reference build {name} absent (python -m oracle.build)")
    return O.ref_ext(name)
