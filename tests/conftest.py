"""Shared pytest setup: the `gpu` marker, import paths, on-demand builds."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flash1017-engine_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def _make(path):
    subprocess.run(["make", "-s", "-C", path, "-j4"], check=True)


@pytest.fixture(scope="session")
def oracle():
    _make(os.path.join(ROOT, "oracle"))
    import oracle as O
    return O


@pytest.fixture(scope="session")
def ffn():
    """The CUDA library binding (built in-tree if missing; loading needs no GPU)."""
    lib = os.path.join(PKG, "_build", "libffn_b200.so")
    if not os.path.exists(lib):
        _make(PKG)
    import ffn_b200
    ffn_b200.lib()
    return ffn_b200


@pytest.fixture(autouse=True)
def _release_host_weight_copies(request):
    """The reference ABI keeps one HBM copy per host weight range, valid while
    the host keeps those weights alive (the reference's mmap'd shards live for
    the whole process).  A test's numpy weights are freed when it ends, and a
    later test's arrays can reuse their addresses, so the copies are dropped
    after every GPU test."""
    yield
    if request.node.get_closest_marker("gpu") and "ffn_b200" in sys.modules:
        sys.modules["ffn_b200"].lib().ffn_b200_release_host_ranges()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
