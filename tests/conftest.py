"""Test configuration: puts the repository root (oracle/) and the package
directory (opencl_tf) on sys.path and registers the ``gpu`` marker."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "opencl-tensorflow_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; parity tests against the oracle")


@pytest.fixture(scope="session")
def port():
    from oracle.oracle import Oracle, build, available
    if not available("port"):
        build()
    return Oracle("port")


@pytest.fixture(scope="session")
def port1():
    """The restated oracle on one thread: the order a single-threaded reference run adds in."""
    from oracle.oracle import Oracle, build, available
    if not available("port"):
        build()
    return Oracle("port", threads=1)


@pytest.fixture(scope="session")
def ref():
    from oracle.oracle import Oracle, available, build
    if not available("ref"):
        try:
            build()
        except Exception:
            pass
    if not available("ref"):
        pytest.skip("oracle/_ref (the reference kernels compiled on the host) is not built")
    return Oracle("ref", threads=1)


@pytest.fixture(scope="session")
def otf():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import opencl_tf
    return opencl_tf
