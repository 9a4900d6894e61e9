"""Shared fixtures.  `-m gpu` tests need a B200 and the built CUDA library;
`-m "not gpu"` tests run anywhere (oracle, host logic, ABI symbol table)."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and libheadshot_cuda.so")


@pytest.fixture(scope="session")
def gpu_ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from headshot_b200.engine import GpuContext

    ctx = GpuContext(0)
    yield ctx
    ctx.close()
