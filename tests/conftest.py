"""Test configuration: import paths, the `gpu` marker, and the library build.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's golden
vectors, the host-side planner and math, the stream topology, the C ABI's
exports and error paths, and the multi-process host logic (gloo).  GPU tests
(`-m gpu`) are the parity tests proper: every op through the C ABI on a
B200 against the golden fixtures and the oracle.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "best-tts-godot_b200"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on a B200)")


@pytest.fixture(scope="session")
def lib():
    """The C-ABI library, built in-tree first if it is missing or stale."""
    import build  # best-tts-godot_b200/build.py
    build.build()
    from bt_b200 import _lib
    return _lib.load()


@pytest.fixture(scope="session")
def gpu_runtime(lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    from bt_b200.runtime import BtRuntime
    return BtRuntime(0)
