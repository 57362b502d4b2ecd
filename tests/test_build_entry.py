"""The package and both extensions import on a machine without a GPU driver
(the build host): libcommux.so loads the CUDA library only on first CUDA use,
and the compute-kernel extension resolves its driver entry points at run time.
`__graft_entry__.build()` relies on this when it imports what it built."""

import os
import subprocess
import sys

from mp import ROOT

CODE = """
import commux_b200 as c
from commux_b200 import _C, _ops
c.register()
print("import ok", c.preferred_backend())
"""


def test_extensions_import_without_driver():
    r = subprocess.run([sys.executable, "-c", CODE], cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "import ok ucx" in r.stdout


def test_commux_alias_exports_the_api():
    code = ("import commux, commux_b200\n"
            "missing = [n for n in commux_b200.__all__ if not hasattr(commux, n)]\n"
            "assert not missing, missing\n"
            "assert commux.register is commux_b200.register and commux.p2p_plan is commux_b200.p2p_plan\n"
            "print('alias ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0 and "alias ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_halo_helper_under_both_names():
    code = ("import commux.halo as a, commux_b200.halo as b, commux_b200.parallel.halo as c\n"
            "assert a.HaloExchange is b.HaloExchange is c.HaloExchange\n"
            "g = a.CartGrid((2, 2, 2), 5)\n"
            "assert len(a.DIRECTIONS) == 26 and a.TAG_BASE == 1000 and g.neighbor((1, 0, 0)) != 5\n"
            "print('halo ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0 and "halo ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_empty_batches_are_rejected_clearly():
    code = ("import commux_b200 as c, torch.distributed as dist, os\n"
            "from commux_b200.utils import free_port\n"
            "os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(free_port()))\n"
            "c.register(); dist.init_process_group('ucx', rank=0, world_size=1)\n"
            "for f in (c.batch_p2p, c.p2p_plan):\n"
            "    try:\n"
            "        f()\n"
            "        raise SystemExit('accepted')\n"
            "    except ValueError as e:\n"
            "        assert 'no sends and no receives' in str(e)\n"
            "dist.destroy_process_group(); print('empty ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0 and "empty ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_reload_after_in_process_build_finds_the_extension():
    # build() imports the package before the extension exists (the package
    # then holds a stand-in for _C) and reloads it once the build is done.
    code = ("import importlib, commux_b200 as c\n"
            "c._C = c._Unbuilt(ImportError('not built yet'))\n"
            "importlib.reload(c)\n"
            "assert not isinstance(c._C, c._Unbuilt), c._C\n"
            "assert c.make_ucp_tag(1, 2) is not None\n"
            "print('reload ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0 and "reload ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
