"""pytest configuration: the `gpu` marker and a one-time native build."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on B200)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA GPUs")


def pytest_sessionstart(session):
    # The native libraries are git-ignored build products: build them once if
    # this checkout has none (a no-op when they are already up to date).
    try:
        import commux_b200._C  # noqa: F401
        import commux_b200._ops  # noqa: F401
    except ImportError:
        from commux_b200.build import build

        build()


def cuda_count():
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.fixture
def ngpus():
    return cuda_count()
