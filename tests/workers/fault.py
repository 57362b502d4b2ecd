"""Failure detection on the host (no GPU involved).

mode=timeout: rank 0 receives a message rank 1 never sends; the wait must
raise DistBackendError within its timeout. mode=drop: COMMUX_FAULT drops one
send on rank 1; rank 0's matching wait times out. mode=kill: COMMUX_FAULT
makes rank 1 exit mid-run; rank 0's pending receive must fail with a
"peer ... failed/exited" error instead of hanging."""
import datetime
import os
import sys
import time

from common import init, torch, dist

mode = sys.argv[1]
rank, world, dev = init(timeout_s=30)
ok = True
t0 = time.time()
if mode in ("timeout", "drop"):
    if rank == 0:
        buf = torch.zeros(4)
        w = dist.irecv(buf, 1, tag=77)
        try:
            w.wait(timeout=datetime.timedelta(seconds=2))
            ok = False
            print("FAIL wait returned", flush=True)
        except Exception as e:
            print("raised:", type(e).__name__, str(e)[:200], flush=True)
            ok = "timed out" in str(e) and time.time() - t0 < 20
    elif rank == 1 and mode == "drop":
        dist.send(torch.ones(4), 0, tag=77)  # dropped by COMMUX_FAULT=drop:1:77
    dist.barrier()
elif mode == "kill":
    if rank == 0:
        buf = torch.zeros(4)
        w = dist.irecv(buf, 1, tag=88)
        try:
            w.wait(timeout=datetime.timedelta(seconds=20))
            ok = False
        except Exception as e:
            print("raised:", str(e)[:200], flush=True)
            ok = ("failed" in str(e) or "exited" in str(e)) and time.time() - t0 < 15
        print("ok" if ok else "FAIL", flush=True)
        os._exit(0 if ok else 1)
    else:
        dist.barrier  # noqa: B018
        # the COMMUX_FAULT kill trigger fires on this rank's next posted op
        dist.isend(torch.ones(4), 0, tag=99)
        time.sleep(30)
        os._exit(3)
print("ok" if ok else "FAIL", flush=True)
dist.destroy_process_group()
sys.exit(0 if ok else 1)
