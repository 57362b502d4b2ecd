"""Build the native libraries in-tree (``python -m commux_b200.build``).

Runs CMake + Ninja into ``<repo>/build`` and places the outputs inside the
package: ``commux_b200/lib/libcommux{,_io,_cuda}.so``, ``commux_b200/_C*.so``
and the C++ test driver ``commux_b200/lib/test_commux``. CUDA code is compiled
for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``); nvcc
cross-compiles, so no GPU is needed to build.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_DIR)


def _has_cuda_sources() -> bool:
    d = os.path.join(PKG_DIR, "csrc", "cuda")
    return os.path.isdir(d) and any(f.endswith(".cu") for f in os.listdir(d))


def build(build_dir: str | None = None, jobs: int | None = None, verbose: bool = False,
          sanitize: str = "", device_checks: bool = False, cuda: bool | None = None) -> None:
    if build_dir is None:
        build_dir = os.path.join(REPO, f"build-{sanitize}" if sanitize else
                                 "build-devchecks" if device_checks else "build")
    os.makedirs(build_dir, exist_ok=True)
    if cuda is None:
        cuda = _has_cuda_sources() and os.path.exists("/usr/local/cuda/bin/nvcc") and not sanitize
    gen = ["-G", "Ninja"] if shutil.which("ninja") else []
    cfg = ["cmake", "-S", REPO, "-B", build_dir, *gen,
           f"-DPython3_EXECUTABLE={sys.executable}",
           f"-DCOMMUX_CUDA={'ON' if cuda else 'OFF'}",
           f"-DCOMMUX_DEVICE_CHECKS={'ON' if device_checks else 'OFF'}",
           "-DCMAKE_BUILD_TYPE=Release"]
    if sanitize:
        # host libraries and the C++ test driver only, inside the build tree
        cfg += [f"-DCOMMUX_SANITIZE={sanitize}", "-DCOMMUX_BUILD_PYTHON=OFF"]
    elif device_checks:
        # the libraries with bounds-checking kernels, inside the build tree
        # (<build_dir>/lib); the package keeps the production kernels
        cfg += ["-DCOMMUX_BUILD_PYTHON=OFF"]
    env = dict(os.environ)
    env.setdefault("CUDACXX", "/usr/local/cuda/bin/nvcc")
    # Use the system compiler, which links the shared libstdc++ that torch
    # uses. A toolchain that links libstdc++ statically gives each library
    # private iostream/locale state, and that crashes as soon as one of them
    # formats an exception message coming from torch.
    cxx = os.environ.get("COMMUX_CXX", "/usr/bin/g++")
    cc = os.environ.get("COMMUX_CC", "/usr/bin/gcc")
    if os.path.exists(cxx):
        env["CXX"] = cxx
        cfg.append(f"-DCMAKE_CUDA_HOST_COMPILER={cxx}")
    if os.path.exists(cc):
        env["CC"] = cc
    out = None if verbose else subprocess.PIPE
    r = subprocess.run(cfg, env=env, stdout=out, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout or "")
        raise RuntimeError("commux: cmake configure failed")
    cmd = ["cmake", "--build", build_dir, "-j", str(jobs or os.cpu_count() or 4)]
    r = subprocess.run(cmd, env=env, stdout=out, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout or "")
        raise RuntimeError("commux: native build failed")
    if not verbose and r.stdout:
        # keep the ptxas register/spill report around for inspection
        with open(os.path.join(build_dir, "build.log"), "w") as f:
            f.write(r.stdout)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--build-dir")
    ap.add_argument("-j", "--jobs", type=int)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--sanitize", default="", help="thread, address or undefined (host code)")
    ap.add_argument("--device-checks", action="store_true",
                    help="kernels bounds-check descriptors and report instead of faulting")
    ap.add_argument("--no-cuda", action="store_true")
    a = ap.parse_args()
    build(a.build_dir, a.jobs, a.verbose, a.sanitize, a.device_checks,
          cuda=False if a.no_cuda else None)
    print("commux: build ok")


if __name__ == "__main__":
    main()
