"""Launch a worker script as N ranks on localhost (one process per rank).

Each rank gets RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR=127.0.0.1 /
MASTER_PORT like torchrun would set. Returns (returncode, output) per rank;
every process is killed if the group does not finish within the timeout.
"""

import os
import signal
import socket
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run(script, nprocs, *args, env=None, timeout=120):
    port = free_port()
    path = script if os.path.isabs(script) else os.path.join(HERE, "workers", script)
    procs = []
    for r in range(nprocs):
        e = dict(os.environ)
        e.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(r), WORLD_SIZE=str(nprocs),
                 LOCAL_RANK=str(r), LOCAL_WORLD_SIZE=str(nprocs), PYTHONPATH=ROOT)
        e.update(env or {})
        procs.append(subprocess.Popen([sys.executable, path, *map(str, args)], env=e,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                                      start_new_session=True))
    deadline = time.time() + timeout
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=max(1, deadline - time.time()))
        except subprocess.TimeoutExpired:
            for q in procs:
                try:
                    os.killpg(q.pid, signal.SIGKILL)
                except ProcessLookupError:
                    pass
            out = (p.communicate()[0] or "") + "\n[timed out]"
        outs.append((p.returncode, out))
    return outs


def check(results, expect=0):
    bad = [(i, rc, out) for i, (rc, out) in enumerate(results) if rc != expect]
    if bad:
        msg = "\n".join(f"--- rank {i} rc={rc}\n{out[-4000:]}" for i, rc, out in bad)
        raise AssertionError(f"{len(bad)} rank(s) failed:\n{msg}")
    return results
