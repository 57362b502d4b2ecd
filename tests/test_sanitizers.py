"""The host engine under ThreadSanitizer, AddressSanitizer and
UndefinedBehaviorSanitizer: instrumented builds of libcommux and the C++ test
driver (their own build trees, the
package keeps the production libraries), run as 2 ranks, including the
multi-threaded posting, parked-waiter and large-message tests. ThreadSanitizer
runs over shared memory and over TCP; any data race or memory error report
fails."""

import os
import subprocess
import sys

import pytest

from mp import ROOT, free_port

BUILD = os.path.join(ROOT, "build-thread")
BIN = os.path.join(BUILD, "lib", "test_commux")


@pytest.fixture(scope="module")
def tsan_driver():
    r = subprocess.run([sys.executable, "-m", "commux_b200.build", "--sanitize", "thread"], cwd=ROOT,
                       capture_output=True, text=True, timeout=1500)
    if r.returncode != 0 or not os.path.exists(BIN):
        pytest.skip("ThreadSanitizer build unavailable: " + (r.stdout + r.stderr)[-500:])
    return BIN


@pytest.mark.parametrize("transport", ["shm", "tcp"])
def test_engine_has_no_data_races(tsan_driver, transport):
    port = free_port()
    env = dict(os.environ, COMMUX_MT="1", COMMUX_DEADLOCK="1", COMMUX_TRANSPORT=transport,
               TSAN_OPTIONS="halt_on_error=0 report_signal_unsafe=0")
    procs = [subprocess.Popen([tsan_driver, str(r), "2", "127.0.0.1", str(port)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append((p.communicate(timeout=600)[0], p.returncode))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    for out, rc in outs:
        assert "WARNING: ThreadSanitizer" not in out, out[-4000:]
        assert rc == 0, out[-3000:]
    assert "ALL TESTS PASSED" in outs[0][0]


ASAN_BUILD = os.path.join(ROOT, "build-address")
ASAN_BIN = os.path.join(ASAN_BUILD, "lib", "test_commux")


@pytest.fixture(scope="module")
def asan_driver():
    r = subprocess.run([sys.executable, "-m", "commux_b200.build", "--sanitize", "address"], cwd=ROOT,
                       capture_output=True, text=True, timeout=1500)
    if r.returncode != 0 or not os.path.exists(ASAN_BIN):
        pytest.skip("AddressSanitizer build unavailable: " + (r.stdout + r.stderr)[-500:])
    return ASAN_BIN


def test_engine_has_no_memory_errors(asan_driver):
    """The same driver under AddressSanitizer over shared memory (leak checks
    off: torch's own allocations live until exit)."""
    port = free_port()
    env = dict(os.environ, COMMUX_MT="1", COMMUX_DEADLOCK="1", ASAN_OPTIONS="detect_leaks=0")
    procs = [subprocess.Popen([asan_driver, str(r), "2", "127.0.0.1", str(port)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append((p.communicate(timeout=600)[0], p.returncode))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    for out, rc in outs:
        assert "ERROR: AddressSanitizer" not in out, out[-4000:]
        assert rc == 0, out[-3000:]
    assert "ALL TESTS PASSED" in outs[0][0]


UB_BUILD = os.path.join(ROOT, "build-undefined")
UB_BIN = os.path.join(UB_BUILD, "lib", "test_commux")


@pytest.fixture(scope="module")
def ubsan_driver():
    r = subprocess.run([sys.executable, "-m", "commux_b200.build", "--sanitize", "undefined"], cwd=ROOT,
                       capture_output=True, text=True, timeout=1500)
    if r.returncode != 0 or not os.path.exists(UB_BIN):
        pytest.skip("UndefinedBehaviorSanitizer build unavailable: " + (r.stdout + r.stderr)[-500:])
    return UB_BIN


@pytest.mark.parametrize("transport", ["shm", "tcp"])
def test_engine_has_no_undefined_behaviour(ubsan_driver, transport):
    port = free_port()
    env = dict(os.environ, COMMUX_MT="1", COMMUX_DEADLOCK="1", COMMUX_TRANSPORT=transport,
               UBSAN_OPTIONS="print_stacktrace=1")
    procs = [subprocess.Popen([ubsan_driver, str(r), "2", "127.0.0.1", str(port)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append((p.communicate(timeout=600)[0], p.returncode))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    for out, rc in outs:
        assert "runtime error" not in out, out[-4000:]
        assert rc == 0, out[-3000:]
    assert "ALL TESTS PASSED" in outs[0][0]
