"""The pull kernel's copy descriptors, checked on the host: FastDiv against
exact division, and the descriptors built for random strided views walked
the way the kernel walks them against a brute-force enumeration
(tests/cpp/test_layout.cpp). Needs a C++ compiler and the CUDA headers only."""

import os
import shutil
import subprocess
import tempfile

import pytest

from mp import ROOT

CUDA_INC = "/usr/local/cuda/include"


def test_descriptor_walks_match_brute_force():
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None or not os.path.exists(os.path.join(CUDA_INC, "cuda_runtime.h")):
        pytest.skip("no C++ compiler or CUDA headers")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "test_layout")
        r = subprocess.run([cxx, "-std=c++17", "-O2", "-Wall", "-Wno-unused-function",
                            "-I", os.path.join(ROOT, "commux_b200", "csrc", "cuda"), "-I", CUDA_INC,
                            "-I", os.path.join(ROOT, "commux_b200", "include"),
                            os.path.join(ROOT, "tests", "cpp", "test_layout.cpp"), "-o", exe],
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
        r = subprocess.run([exe, "20000"], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0 and "ALL LAYOUT CHECKS PASSED" in r.stdout, r.stdout[-3000:]


def test_descriptor_code_has_no_undefined_behaviour():
    """The same checks built with AddressSanitizer and UndefinedBehaviorSanitizer
    (signed overflow, shifts, misaligned or out-of-range accesses abort)."""
    cxx = shutil.which("g++")
    if cxx is None or not os.path.exists(os.path.join(CUDA_INC, "cuda_runtime.h")):
        pytest.skip("no g++ or CUDA headers")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "test_layout_san")
        r = subprocess.run([cxx, "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined",
                            "-fno-sanitize-recover=undefined",
                            "-I", os.path.join(ROOT, "commux_b200", "csrc", "cuda"), "-I", CUDA_INC,
                            "-I", os.path.join(ROOT, "commux_b200", "include"),
                            os.path.join(ROOT, "tests", "cpp", "test_layout.cpp"), "-o", exe],
                           capture_output=True, text=True, timeout=600)
        if r.returncode != 0 and "sanitize" in (r.stdout + r.stderr):
            pytest.skip("sanitizer runtime unavailable: " + (r.stdout + r.stderr)[-300:])
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
        r = subprocess.run([exe, "3000"], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0 and "ALL LAYOUT CHECKS PASSED" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
