"""Shared pytest setup: import paths, the `gpu` marker, and in-tree builds.

CPU tests (`-m "not gpu"`) need the oracle (gcc) and the C-ABI library
(nvcc cross-compiles sm_100a without a GPU); both are built here on demand
with the committed Makefiles if missing.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "slang-gemm_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (ROOT, PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def _ensure_built():
    if not os.path.exists(os.path.join(ORACLE, "liboracle_gemm.so")):
        subprocess.run(["make", "-s", "-C", ORACLE], check=True)
    if not os.path.exists(os.path.join(PKG, "libgemm_sm100.so")):
        subprocess.run(["make", "-s", "-j8", "-C", PKG], check=True)


_ensure_built()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    """Skips (rather than fails) GPU tests on a machine without a B200."""
    if not gpu_available():
        pytest.skip("no sm_100 GPU")
    import torch

    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def handle(cuda):
    import gemm_sm100 as gs

    h = gs.Handle()
    yield h
    h.close()
