"""allreduce SUM, out-of-order tagged isend/irecv, barrier through torch.distributed
(reference: tests/test_torch_dist.py:22-70). CMX_DEVICE=cuda runs on GPUs."""
from common import Checker, init, torch, dist

rank, world, dev = init()
c = Checker(rank)
c.check("backend name", dist.get_backend() == "ucx", dist.get_backend())
t = torch.full((4,), float(rank + 1), device=dev)
dist.all_reduce(t)
c.equal("all_reduce SUM", t, torch.full((4,), world * (world + 1) / 2.0))
if world >= 2:
    if rank == 0:
        reqs = [dist.isend(torch.full((3,), 1.0, device=dev), 1, tag=100),
                dist.isend(torch.full((3,), 2.0, device=dev), 1, tag=200)]
        for r in reqs:
            r.wait()
    elif rank == 1:
        b = torch.zeros(3, device=dev)
        a = torch.zeros(3, device=dev)
        rb = dist.irecv(b, 0, tag=200)  # the second-sent message first
        ra = dist.irecv(a, 0, tag=100)
        rb.wait()
        ra.wait()
        c.equal("tag-matched B", b, torch.full((3,), 2.0))
        c.equal("tag-matched A", a, torch.full((3,), 1.0))
    # blocking send/recv in matching order
    x = torch.arange(10, dtype=torch.float32, device=dev) + rank
    y = torch.empty_like(x)
    peer = (rank + 1) % world
    src = (rank - 1) % world
    rr = dist.irecv(y, src, tag=7)
    dist.send(x, peer, tag=7)
    rr.wait()
    c.equal("ring p2p", y, torch.arange(10, dtype=torch.float32) + src)
dist.barrier()
c.finish()
