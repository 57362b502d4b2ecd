"""C++ consumers. (1) `cmake --install` of the in-tree build, then a separate
project that does find_package(commux) and links commux::commux and
commux::commux_io. (2) A project that pulls the source tree in with
FetchContent and links the same targets. (3) A project that finds the library
and headers inside the installed `commux` Python package, as the reference's
README shows. The reference documents all three flows
(reference: README.md:83-114)."""

import sys

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


FETCH_CMAKE = """cmake_minimum_required(VERSION 3.26)
project(fetch_consumer CXX)
set(CMAKE_CXX_STANDARD 17)
include(FetchContent)
FetchContent_Declare(commux SOURCE_DIR "{root}")
set(COMMUX_CUDA OFF CACHE BOOL "" FORCE)
FetchContent_MakeAvailable(commux)
add_executable(consumer main.cpp)
target_link_libraries(consumer PRIVATE commux::commux commux::commux_io)
"""


def _tree_state(root):
    """Modification times of the package's build outputs (must not change)."""
    out = {}
    for d in (os.path.join(root, "commux_b200", "lib"), os.path.join(root, "commux_b200")):
        if os.path.isdir(d):
            for f in os.listdir(d):
                if f.endswith(".so") or f == "test_commux":
                    out[os.path.join(d, f)] = os.stat(os.path.join(d, f)).st_mtime_ns
    return out


def test_fetchcontent_consumer():
    if shutil.which("cmake") is None:
        pytest.skip("no cmake")
    before = _tree_state(ROOT)
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "consumer")
        os.makedirs(src)
        with open(os.path.join(src, "CMakeLists.txt"), "w") as f:
            f.write(FETCH_CMAKE.format(root=ROOT))
        with open(os.path.join(src, "main.cpp"), "w") as f:
            f.write(CONSUMER_MAIN)
        env = dict(os.environ, CXX="/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++",
                   CC="/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc")
        b = os.path.join(d, "b")
        gen = ["-G", "Ninja"] if shutil.which("ninja") else []
        r = subprocess.run(["cmake", "-S", src, "-B", b, *gen, f"-DPython3_EXECUTABLE={sys.executable}"],
                           env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
        r = subprocess.run(["cmake", "--build", b, "-j", str(os.cpu_count() or 4)], env=env,
                           capture_output=True, text=True, timeout=1200)
        assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
        # the commux libraries built for the consumer live in its own tree
        assert os.path.exists(os.path.join(b, "_deps", "commux-build", "lib", "libcommux.so"))
        r = subprocess.run([os.path.join(b, "consumer")], capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        assert "tag 1000500000007" in r.stdout
    assert _tree_state(ROOT) == before, "a build inside another project wrote into the package"


PROBE_CMAKE = """cmake_minimum_required(VERSION 3.22)
project(probe_consumer CXX)
set(CMAKE_CXX_STANDARD 17)
find_package(Python3 REQUIRED COMPONENTS Interpreter)
execute_process(
  COMMAND ${{Python3_EXECUTABLE}} -c "import commux,os;print(os.path.dirname(commux.__file__))"
  OUTPUT_VARIABLE COMMUX_DIR OUTPUT_STRIP_TRAILING_WHITESPACE)
find_library(COMMUX_LIBRARY commux HINTS ${{COMMUX_DIR}}/lib REQUIRED NO_DEFAULT_PATH)
add_executable(consumer main.cpp)
target_include_directories(consumer PRIVATE ${{COMMUX_DIR}}/include {torch_inc})
target_compile_definitions(consumer PRIVATE _GLIBCXX_USE_CXX11_ABI={abi})
target_link_directories(consumer PRIVATE {torch_lib})
target_link_libraries(consumer PRIVATE ${{COMMUX_LIBRARY}} torch torch_cpu c10)
set_target_properties(consumer PROPERTIES BUILD_RPATH "${{COMMUX_DIR}}/lib;{torch_lib}")
"""


def test_python_package_probe_consumer():
    """The reference README's route: locate lib/ and include/ from the
    installed `commux` package (here the in-tree package, on PYTHONPATH)."""
    if shutil.which("cmake") is None:
        pytest.skip("no cmake")
    if not os.path.exists(os.path.join(ROOT, "commux", "lib", "libcommux.so")):
        pytest.skip("no in-tree build")
    import torch
    from torch.utils import cpp_extension

    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "consumer")
        os.makedirs(src)
        with open(os.path.join(src, "CMakeLists.txt"), "w") as f:
            f.write(PROBE_CMAKE.format(torch_inc=" ".join(cpp_extension.include_paths()), torch_lib=torch_lib,
                                       abi=int(torch._C._GLIBCXX_USE_CXX11_ABI)))
        with open(os.path.join(src, "main.cpp"), "w") as f:
            f.write(CONSUMER_MAIN)
        env = dict(os.environ, PYTHONPATH=ROOT,
                   CXX="/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++")
        b = os.path.join(d, "b")
        r = subprocess.run(["cmake", "-S", src, "-B", b, f"-DPython3_EXECUTABLE={sys.executable}"], env=env,
                           capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
        r = subprocess.run(["cmake", "--build", b], env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
        r = subprocess.run([os.path.join(b, "consumer")], capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        assert "tag 1000500000007" in r.stdout
