"""Shared test setup: repo root on sys.path, the engine package, the `gpu` marker."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402

load_package()

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running (full 30B-shape model)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    if not O.LIB_PATH.exists():
        O.build()
    return O


@pytest.fixture(scope="session")
def tools():
    from qwen30brust_b200 import build, tools as T
    if not T.LIB_PATH.exists():
        build.build_tools()
    return T


@pytest.fixture(scope="session")
def cuda_engine():
    """The ctypes binding of libqwen_cuda.so; a GPU test fails (not skips) if it is missing."""
    from qwen30brust_b200 import engine as E
    assert E.LIB_PATH.exists(), "libqwen_cuda.so is not built"
    return E


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "gpu test without a CUDA device"
    return torch
