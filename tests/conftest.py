"""Shared test set-up.

``-m gpu`` tests need a CUDA device (a B200) and call the kernels through the C ABI; the rest
run on CPU (oracle vs the reference's goldens, host logic, library load / exports). The CPU
oracle in ``oracle/`` is the checker only.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); calls the CUDA kernels")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    import mlx_dspark_b200  # noqa: F401  (loads libdspark.so or raises)
    from mlx_dspark_b200 import _lib

    _lib.ensure_init(torch.cuda.current_device())
    yield torch.device("cuda", torch.cuda.current_device())
    torch.cuda.synchronize()
    assert _lib.device_status(torch.cuda.current_device()) == 0, "a bounded device wait ran out"


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.build()
    return o


def pytest_collection_modifyitems(config, items):
    # keep GPU tests after CPU tests within the run (cheap failures first)
    items.sort(key=lambda it: (1 if it.get_closest_marker("gpu") else 0))
    if os.environ.get("DSPARK_TEST_FAST"):
        for it in items:
            if it.get_closest_marker("slow"):
                it.add_marker(pytest.mark.skip(reason="DSPARK_TEST_FAST"))
