"""Vector p2p (COMMUX_COALESCE on/off), the group window (COMMUX_GROUP), the
batch_isend_irecv aggregate Work, any-source receive with sourceRank, and
strided receive views (reference: tests/test_commux.cpp:151-200)."""

from common import Checker, init, torch, dist

rank, world, dev = init()
c = Checker(rank)
pg = dist.distributed_c10d._get_default_group()
if world >= 2 and rank < 2:
    peer = 1 - rank
    shapes = [5, 1, 8]
    if rank == 0:
        v = [torch.full((s,), float(10 + k), dtype=torch.float64, device=dev) for k, s in enumerate(shapes)]
        pg.send(v, 1, 300).wait()
    else:
        v = [torch.zeros(s, dtype=torch.float64, device=dev) for s in shapes]
        pg.recv(v, 0, 300).wait()
        for k in range(3):
            c.equal(f"vector p2p[{k}]", v[k], torch.full((shapes[k],), float(10 + k), dtype=torch.float64))
    # batch window: recv + send deferred together, one aggregate Work
    out = torch.zeros(4, dtype=torch.float64, device=dev)
    mine = torch.full((4,), float(rank + 1), dtype=torch.float64, device=dev)
    ops = [dist.P2POp(dist.irecv, out, peer, tag=410 if rank == 1 else 420),
           dist.P2POp(dist.isend, mine, peer, tag=410 if rank == 0 else 420)]
    for w in dist.batch_isend_irecv(ops):
        w.wait()
    c.equal("batch window", out, torch.full((4,), float(peer + 1), dtype=torch.float64))
    # strided receive into a view (superset of the reference: recv may be strided)
    big = torch.zeros(6, 8, dtype=torch.float32, device=dev)
    if rank == 0:
        dist.send(torch.arange(12, dtype=torch.float32, device=dev).view(6, 2), 1, tag=500)
    else:
        dist.recv(big[:, 3:5], 0, tag=500)
        want = torch.zeros(6, 8)
        want[:, 3:5] = torch.arange(12, dtype=torch.float32).view(6, 2)
        c.equal("strided recv view", big, want)
    # strided send view
    if rank == 0:
        m = torch.arange(40, dtype=torch.float32, device=dev).view(5, 8)
        dist.send(m[:, 1::3], 1, tag=510)
    else:
        r = torch.empty(5, 3, device=dev)
        dist.recv(r, 0, tag=510)
        c.equal("strided send view", r, torch.arange(40, dtype=torch.float32).view(5, 8)[:, 1::3])
# any source: every rank > 0 sends to 0 with tag 600; rank 0 learns the sources
if world >= 2:
    if rank == 0:
        seen = []
        for _ in range(world - 1):
            buf = torch.zeros(2, device=dev)
            w = pg.recv_anysource([buf], 600)
            w.wait()
            src = w._source_rank()
            seen.append(src)
            c.equal(f"anysource payload from {src}", buf, torch.full((2,), float(src)))
        c.check("anysource sources", sorted(seen) == list(range(1, world)), str(seen))
    else:
        dist.send(torch.full((2,), float(rank), device=dev), 0, tag=600)
    # the same through torch.distributed: recv without src returns the sender
    if rank == 0:
        seen = []
        for _ in range(world - 1):
            buf = torch.zeros(3, device=dev)
            src = dist.recv(buf, tag=601)
            seen.append(src)
            c.equal(f"dist.recv any source from {src}", buf, torch.full((3,), float(10 * src)))
        c.check("dist.recv any source senders", sorted(seen) == list(range(1, world)), str(seen))
    else:
        dist.send(torch.full((3,), float(10 * rank), device=dev), 0, tag=601)
c.finish()
