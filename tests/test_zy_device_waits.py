"""Failure detection on the GPU without a fault: waits on flags that nothing
sets give up after their limit, record their status and return, and the
context stays usable (csrc/cuda/wait_selftest.cu). Runs in its own process."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_device_waits_give_up_and_report():
    worker = os.path.join(ROOT, "tests", "workers", "device_wait.py")
    r = subprocess.run([sys.executable, worker], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
