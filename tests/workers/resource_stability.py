"""No engine state outlives the messages that created it. The counterpart of
the reference's regression test on host send addresses
(reference: tests/test_host_coll_addresses.py:18-56: 100 all_reduces and 20
barriers on fresh tensors): the same workload, plus tagged p2p of fresh
tensors at eager and rendezvous sizes, then every queue and table of the
engine (posted receives, unexpected messages, partly received messages,
sends waiting for their FIN, sends queued for the TCP pump) must be empty."""
import time

from common import Checker, init, torch, dist

import commux_b200 as commux

rank, world, dev = init(timeout_s=120)
c = Checker(rank)
sizes = [1, 1000, 20000, 300000]  # floats: eager and rendezvous
for k in range(100):
    t = torch.full((sizes[k % len(sizes)],), float(rank + 1))
    dist.all_reduce(t)
    if k % 5 == 0:
        dist.barrier()
peer, src = (rank + 1) % world, (rank - 1) % world
for k in range(50):
    n = sizes[k % len(sizes)]
    r = dist.irecv(torch.empty(n), src, tag=40 + k % 3)
    s = dist.isend(torch.full((n,), float(k)), peer, tag=40 + k % 3)
    s.wait()
    r.wait()
dist.barrier()
time.sleep(0.2)  # FIN records of the last rendezvous messages land
st = commux.stats()
# every rank reads its gauges before any rank sends the next message (the
# agreement all_reduce of finish() would otherwise land in a slower rank's
# unexpected queue before that rank read its gauges)
dist.barrier()
c.check("at least 100 host sends", st["sends"] >= 100, str(st["sends"]))
for g in ("posted_now", "unexpected_now", "partial_now", "sends_waiting_now", "pump_waiting_now"):
    c.check(f"{g} back to zero", st[g] == 0, f"{g}={st[g]}")
c.finish()
