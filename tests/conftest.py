"""Shared test setup: the `gpu` marker, import paths and library builds.

Tests marked `gpu` need a B200 and run the CUDA path through the C ABI; everything
else runs on the CPU (the oracle, the host logic, the ABI's exported symbols).
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "sense-nova-server_b200"
for p in (str(PKG), str(ROOT / "oracle"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running (full-size shapes)")


def _ensure_built():
    import build  # sense-nova-server_b200/build.py

    build.build_oracle()
    if not build.LIB.exists():
        build.build_lib()


_ensure_built()


def has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def lib():
    from sensenova_b200 import ffi

    return ffi.load()


@pytest.fixture(scope="session")
def orc():
    import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def torch_cuda(request):
    if not has_gpu():
        # Under `-m gpu` a missing device is a failure, not a skip: a silent skip would
        # hide a broken device path.
        if "gpu" in (request.config.getoption("-m") or "") and "not gpu" not in request.config.getoption("-m"):
            pytest.fail("no CUDA device on this host")
        pytest.skip("no CUDA device")
    import torch

    torch.cuda.init()
    return torch
