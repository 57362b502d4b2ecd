"""Wheel / editable install of commux_b200 (and the ``commux`` alias package).

The native libraries are built by CMake through ``commux_b200.build`` (the same
build ``python -m commux_b200.build`` runs in-tree): ``libcommux.so``,
``libcommux_io.so`` and ``libcommux_cuda.so`` under ``commux_b200/lib``, the
pybind modules ``commux_b200/_C`` and ``commux_b200/_ops``, and the C++ headers
under ``commux_b200/include/commux`` for C++ consumers. torch must be
importable at build time (install with ``--no-build-isolation``).

    pip install --no-build-isolation .
"""

import os
import subprocess
import sys

from setuptools import find_packages, setup
from setuptools.command.build_py import build_py
from setuptools.dist import Distribution


def _version() -> str:
    """COMMUX_VERSION, else the latest `vX.Y.Z` git tag, else 0.1.0."""
    v = os.environ.get("COMMUX_VERSION")
    if v:
        return v.lstrip("v")
    try:
        tag = subprocess.run(["git", "describe", "--tags", "--abbrev=0", "--match", "v[0-9]*"],
                             capture_output=True, text=True, cwd=os.path.dirname(os.path.abspath(__file__)),
                             timeout=30)
        if tag.returncode == 0 and tag.stdout.strip():
            return tag.stdout.strip().lstrip("v")
    except (OSError, subprocess.SubprocessError):
        pass
    return "0.1.0"


class BuildNative(build_py):
    def run(self):
        subprocess.check_call([sys.executable, "-m", "commux_b200.build"])
        super().run()


class BinaryDistribution(Distribution):
    def has_ext_modules(self):
        return True


setup(
    name="commux-b200",
    version=_version(),
    description="MPI-style tagged p2p and collectives for torch.distributed on B200 (NVLink 5 / NVSwitch)",
    packages=find_packages(include=["commux_b200", "commux_b200.*", "commux"]),
    # `commux` (the reference's package name) carries the libraries and
    # headers too, where C++ consumers of the reference look for them
    package_data={"commux_b200": ["_C*.so", "_ops*.so", "lib/*.so", "lib/test_commux",
                                  "include/commux/*.hpp", "include/commux/*.h"],
                  "commux": ["lib/*.so", "include/commux/*.hpp", "include/commux/*.h"]},
    python_requires=">=3.10",
    cmdclass={"build_py": BuildNative},
    distclass=BinaryDistribution,
    zip_safe=False,
)
