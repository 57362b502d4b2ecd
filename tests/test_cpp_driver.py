"""The C++ test driver (commux_b200/lib/test_commux): tag matching, collectives,
vector p2p, group window, multi-threaded posting and parked-waiter wakeups
through the C++ ProcessGroupUCX API (reference: tests/test_commux.cpp)."""

import os
import subprocess

import pytest

from mp import ROOT, free_port

BIN = os.path.join(ROOT, "commux_b200", "lib", "test_commux")


def run_driver(world, env=None, timeout=180):
    port = free_port()
    e = dict(os.environ)
    e.update(env or {})
    procs = [subprocess.Popen([BIN, str(r), str(world), "127.0.0.1", str(port)], env=e,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(world)]
    outs = []
    for p in procs:
        try:
            outs.append((p.communicate(timeout=timeout)[0], p.returncode))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    for out, rc in outs:
        assert rc == 0, out[-3000:]
    return outs


@pytest.fixture(autouse=True)
def _need_binary():
    if not os.path.exists(BIN):
        pytest.skip("C++ test driver not built")


@pytest.mark.parametrize("world", [2, 3])
def test_driver_basic(world):
    out = run_driver(world)
    assert "ALL TESTS PASSED" in out[0][0]


@pytest.mark.parametrize("coalesce,group", [("1", "0"), ("0", "1")])
def test_driver_coalesce_group(coalesce, group):
    run_driver(2, {"COMMUX_COALESCE": coalesce, "COMMUX_GROUP": group})


def test_driver_threads():
    out = run_driver(2, {"COMMUX_MT": "1", "COMMUX_DEADLOCK": "1"}, timeout=240)
    assert "parked waiters all wake" in out[0][0] or "parked waiters all wake" in out[1][0]


def test_driver_pingpong_bench():
    out = run_driver(2, {"COMMUX_BENCH": "1", "COMMUX_BENCH_V": "2"})
    assert "[bench] V=2" in out[0][0]
