"""Shared test setup.

Markers: `gpu` tests need a B200 and the built engine (libazb200.so); the
rest run on any machine. GPU tests never skip for a missing library: the
engine must load, or the test fails.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("alphazero-go_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built engine")


@pytest.fixture(scope="session")
def engine():
    """The azb200 module with a usable device 0 (fails, never skips, on a GPU run)."""
    import azb200

    ok, why = azb200.cuda_available(0)
    assert ok, f"no usable GPU for the engine: {why}"
    return azb200


@pytest.fixture(scope="session")
def oracle():
    import oracle as O

    O.lib()   # built by __graft_entry__.build() / `make -C oracle`
    return O
