"""A sender may reuse its buffer as soon as its send's wait() returns. Rank 0
sends 2 MiB messages from one buffer, overwriting it right after each wait;
rank 1 checks that every message holds the values it had when it was sent.
Over TCP this checks that a large send (which the pump sends straight from
the sender's memory) completes only once its last byte has left."""
from common import Checker, init, torch, dist

rank, world, dev = init(timeout_s=90)
c = Checker(rank)
n = 1 << 19  # fp32: 2 MiB
rounds = 12
if rank == 0:
    buf = torch.empty(n)
    for k in range(rounds):
        buf.fill_(float(k + 1))
        dist.isend(buf, 1, tag=30).wait()
        buf.fill_(-1.0)  # reused at once
elif rank == 1:
    got = torch.empty(n)
    for k in range(rounds):
        dist.recv(got, 0, tag=30)
        c.check(f"message {k} intact", bool((got == float(k + 1)).all()), f"min {float(got.min())}")
c.finish()
