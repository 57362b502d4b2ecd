"""C++ consumers: `cmake --install` of the in-tree build, then a separate
project that does find_package(commux) and links commux::commux and
commux::commux_io (the reference documents the same consumer flow with its
installed headers and libcommux.so)."""

import os
import shutil
import subprocess
import tempfile

import pytest

from mp import ROOT

BUILD = os.path.join(ROOT, "build")

CONSUMER_CMAKE = """cmake_minimum_required(VERSION 3.22)
project(consumer CXX)
set(CMAKE_CXX_STANDARD 17)
find_package(commux REQUIRED)
add_executable(consumer main.cpp)
target_compile_definitions(consumer PRIVATE _GLIBCXX_USE_CXX11_ABI=1)
target_link_libraries(consumer PRIVATE commux::commux commux::commux_io)
"""

CONSUMER_MAIN = """#include <commux/io.hpp>
#include <commux/process_group_ucx.hpp>
#include <cstdio>
int main() {
  auto t = commux::make_ucp_tag(1, 7, 2, true);
  std::printf("tag %llx\\n", static_cast<unsigned long long>(t));
  return t == ((1ull << 48) | (2ull << 33) | (1ull << 32) | 7ull) ? 0 : 1;
}
"""


def test_find_package_consumer():
    if not os.path.exists(os.path.join(BUILD, "CMakeCache.txt")) or shutil.which("cmake") is None:
        pytest.skip("no in-tree CMake build")
    with tempfile.TemporaryDirectory() as d:
        prefix = os.path.join(d, "install")
        r = subprocess.run(["cmake", "--install", BUILD, "--prefix", prefix], capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        assert os.path.exists(os.path.join(prefix, "lib", "cmake", "commux", "commuxConfig.cmake"))
        src = os.path.join(d, "consumer")
        os.makedirs(src)
        with open(os.path.join(src, "CMakeLists.txt"), "w") as f:
            f.write(CONSUMER_CMAKE)
        with open(os.path.join(src, "main.cpp"), "w") as f:
            f.write(CONSUMER_MAIN)
        env = dict(os.environ, CXX="/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++")
        b = os.path.join(d, "b")
        r = subprocess.run(["cmake", "-S", src, "-B", b, f"-DCMAKE_PREFIX_PATH={prefix}"], env=env,
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        r = subprocess.run(["cmake", "--build", b], env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout + r.stderr
        r = subprocess.run([os.path.join(b, "consumer")], capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        assert "tag 1000500000007" in r.stdout
