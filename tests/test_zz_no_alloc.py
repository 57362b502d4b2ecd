"""The allocation-free strided copy entry point (commux_strided_copy_noalloc in
libcommux_cuda.so), called through ctypes and compared with the backend's
CUDA self send/recv, which runs the same pull kernel with allocated scratch.
Runs in its own process, so it passes alone or after every other test."""

import pytest

from mp import check, run

pytestmark = pytest.mark.gpu


def test_noalloc_copy_matches_existing_path():
    check(run("no_alloc.py", 1, env={"CMX_DEVICE": "cuda"}, timeout=240))
