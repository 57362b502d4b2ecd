"""Multi-rank CPU tests of the commux backend (gloo-free: every rank talks
through commux's shared-memory engine). Mirrors the reference's Python tests
(tests/test_torch_dist.py, test_collectives.py, test_reduce_op.py) and adds
the mixed tagged p2p + collectives workload, coalescing/grouping, halo, DDP,
IOContext and
host-side failure detection."""

import os
import tempfile

import pytest

from mp import check, run


@pytest.mark.parametrize("world", [3, 4])
def test_subgroups(world):
    check(run("subgroups.py", world, timeout=180))


@pytest.mark.parametrize("world", [2, 3])
def test_p2p_fuzz(world):
    check(run("fuzz_p2p.py", world, timeout=240))


@pytest.mark.parametrize("world,transport", [(3, "shm"), (2, "tcp")])
def test_no_engine_state_left_behind(world, transport):
    check(run("resource_stability.py", world, env={"COMMUX_TRANSPORT": transport}, timeout=180))


@pytest.mark.parametrize("transport", ["shm", "tcp"])
def test_buffer_reuse_after_wait(transport):
    check(run("reuse_after_wait.py", 2, env={"COMMUX_TRANSPORT": transport}, timeout=180))


def test_p2p_fuzz_tcp():
    check(run("fuzz_p2p.py", 2, env={"COMMUX_TRANSPORT": "tcp"}, timeout=240))


def test_torch_dist_2ranks():
    check(run("torch_dist.py", 2))


@pytest.mark.parametrize("world", [1, 2, 3, 4, 7])
def test_collectives(world):
    check(run("collectives.py", world, timeout=180))


@pytest.mark.parametrize("world", [1, 3, 4])
def test_reduce_op_rejected_everywhere(world):
    check(run("reduce_op.py", world, timeout=120))


def test_mixed_tagged_bit_exact():
    out = check(run("mixed_tagged.py", 2, timeout=180))
    assert "PASSED" in out[0][1]


def test_mixed_tagged_bit_exact_4ranks():
    check(run("mixed_tagged.py", 4, timeout=240))


def test_mixed_tagged_two_copy_rendezvous():
    # same workload with the single-copy read switched off (ring + CTS path)
    out = check(run("mixed_tagged.py", 2, env={"COMMUX_CMA": "0"}, timeout=180))
    assert "PASSED" in out[0][1]


@pytest.mark.parametrize("coalesce,group", [("0", "0"), ("1", "0"), ("0", "1"), ("1", "1")])
def test_coalesce_and_group(coalesce, group):
    check(run("coalesce.py", 3, env={"COMMUX_COALESCE": coalesce, "COMMUX_GROUP": group}))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_halo_cpu(world):
    check(run("halo.py", world, timeout=240))


def test_ddp_cpu():
    check(run("ddp.py", 2, timeout=180))


def test_iocontext():
    with tempfile.TemporaryDirectory() as d:
        check(run("io_ctx.py", 3, env={"CMX_IO_PATH": os.path.join(d, "f.bin")}))


def test_wait_timeout_raises():
    check(run("fault.py", 2, "timeout", timeout=90))


def test_fault_drop_times_out():
    check(run("fault.py", 2, "drop", env={"COMMUX_FAULT": "drop:1:77"}, timeout=90))


def test_fault_kill_detected():
    res = run("fault.py", 2, "kill", env={"COMMUX_FAULT": "kill:1:1"}, timeout=90)
    assert res[0][0] == 0, res[0][1][-3000:]
    assert res[1][0] == 77, res[1][1][-3000:]


# --- the TCP transport (peers on other hosts), forced on this one host -------

TCP = {"COMMUX_TRANSPORT": "tcp"}


def test_tcp_torch_dist():
    check(run("torch_dist.py", 2, env=TCP))


@pytest.mark.parametrize("world", [2, 3])
def test_tcp_collectives(world):
    check(run("collectives.py", world, env=TCP, timeout=180))


def test_tcp_mixed_tagged_bit_exact():
    out = check(run("mixed_tagged.py", 2, env=TCP, timeout=180))
    assert "PASSED" in out[0][1]


@pytest.mark.parametrize("coalesce,group", [("0", "0"), ("1", "1")])
def test_tcp_coalesce_and_group(coalesce, group):
    check(run("coalesce.py", 3, env=dict(TCP, COMMUX_COALESCE=coalesce, COMMUX_GROUP=group)))


def test_tcp_halo():
    check(run("halo.py", 4, env=TCP, timeout=240))


def test_tcp_fault_kill_detected():
    # a peer that exits closes its socket: the survivor's wait raises
    res = run("fault.py", 2, "kill", env=dict(TCP, COMMUX_FAULT="kill:1:1"), timeout=90)
    assert res[0][0] == 0, res[0][1][-3000:]
    assert res[1][0] == 77, res[1][1][-3000:]
