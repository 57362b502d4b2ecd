"""Process subgroups on this backend: dist.new_group builds a second backend
instance over a prefixed store. Checks an all_reduce and a tagged p2p inside
a subgroup (group ranks translated to global ones), a broadcast in a second,
overlapping subgroup, and that destroying a subgroup leaves the default group
working."""
from common import Checker, init, torch, dist

rank, world, dev = init(timeout_s=90)
c = Checker(rank)
a = [0, world - 1]
b = list(range(1, world))
ga = dist.new_group(a)
gb = dist.new_group(b)
if rank in a:
    t = torch.full((3,), float(rank + 1), device=dev)
    dist.all_reduce(t, group=ga)
    c.equal("subgroup all_reduce", t, torch.full((3,), float(sum(r + 1 for r in a))))
    if rank == a[0]:
        dist.send(torch.full((2,), 7.0, device=dev), a[1], group=ga, tag=5)
    else:
        y = torch.zeros(2, device=dev)
        dist.recv(y, a[0], group=ga, tag=5)
        c.equal("subgroup p2p", y, torch.full((2,), 7.0))
if rank in b:
    t = torch.full((1,), float(rank), device=dev)
    dist.broadcast(t, src=b[0], group=gb)
    c.equal("second subgroup broadcast", t, torch.full((1,), float(b[0])))
dist.destroy_process_group(ga)
t = torch.ones(2, device=dev)
dist.all_reduce(t)
c.equal("default group after destroying a subgroup", t, torch.full((2,), float(world)))
c.finish()
