"""reduce/broadcast at every root, all_reduce SUM/PRODUCT/MIN/MAX/AVG, a 2 MiB
all_reduce (rendezvous path), a 3-tensor all_reduce, allgather, reduce_scatter,
all_to_all, gather, scatter (reference: tests/test_collectives.py:38-89)."""
import os

from common import Checker, init, torch, dist

rank, world, dev = init()
c = Checker(rank)


def mine(r):
    return torch.arange(5, dtype=torch.float64) + 10.0 * (r + 1)


total = sum(mine(r) for r in range(world))
for root in range(world):
    t = mine(rank).to(dev)
    dist.reduce(t, dst=root)
    c.equal(f"reduce root={root}", t, total if rank == root else mine(rank))
    t = (mine(rank) if rank == root else torch.zeros(5, dtype=torch.float64)).to(dev)
    dist.broadcast(t, src=root)
    c.equal(f"broadcast root={root}", t, mine(root))
t = mine(rank).to(dev)
dist.all_reduce(t)
c.equal("all_reduce", t, total)
for op, fold in ((dist.ReduceOp.PRODUCT, torch.mul), (dist.ReduceOp.MIN, torch.minimum),
                 (dist.ReduceOp.MAX, torch.maximum)):
    want = mine(0)
    for r in range(1, world):
        want = fold(want, mine(r))
    for root in range(world):
        t = mine(rank).to(dev)
        dist.reduce(t, dst=root, op=op)
        c.equal(f"reduce {op} root={root}", t, want if rank == root else mine(rank))
    t = mine(rank).to(dev)
    dist.all_reduce(t, op=op)
    c.equal(f"all_reduce {op}", t, want)
t = mine(rank).to(dev)
dist.all_reduce(t, op=dist.ReduceOp.AVG)
c.equal("all_reduce AVG", t, total / world)
big = torch.arange(1 << 18, dtype=torch.float64)
t = (big + rank).to(dev)
dist.all_reduce(t)
c.equal("all_reduce 2 MiB", t, world * big + world * (world - 1) / 2)
ts = [(mine(rank) * (k + 1)).to(dev) for k in range(3)]
dist.distributed_c10d._get_default_group().allreduce(ts).wait()
for k in range(3):
    c.equal(f"all_reduce list[{k}]", ts[k], total * (k + 1))
# allgather family
x = (torch.arange(6, dtype=torch.float32) + 100 * rank).to(dev)
outs = [torch.empty(6, device=dev) for _ in range(world)]
dist.all_gather(outs, x)
for r in range(world):
    c.equal(f"all_gather[{r}]", outs[r], torch.arange(6, dtype=torch.float32) + 100 * r)
flat = torch.empty(6 * world, device=dev)
dist.all_gather_into_tensor(flat, x)
c.equal("all_gather_into_tensor", flat, torch.cat([torch.arange(6, dtype=torch.float32) + 100 * r for r in range(world)]))
objs = [None] * world
dist.all_gather_object(objs, {"rank": rank})
c.check("all_gather_object", objs == [{"rank": r} for r in range(world)], str(objs))
# reduce_scatter
inp = (torch.arange(4 * world, dtype=torch.float32) * (rank + 1)).to(dev)
out = torch.empty(4, device=dev)
dist.reduce_scatter_tensor(out, inp)
s = world * (world + 1) / 2
c.equal("reduce_scatter_tensor", out, torch.arange(4 * rank, 4 * rank + 4, dtype=torch.float32) * s)
# all_to_all
if dev.type == "cpu" or os.environ.get("CMX_A2A", "1") == "1":
    inp = (torch.arange(world * 2, dtype=torch.float32) + 1000 * rank).to(dev)
    out = torch.empty(world * 2, device=dev)
    dist.all_to_all_single(out, inp)
    want = torch.cat([torch.arange(2 * rank, 2 * rank + 2, dtype=torch.float32) + 1000 * r for r in range(world)])
    c.equal("all_to_all_single", out, want)
    # list form: outs[p] receives rank p's ins[me]
    ins = [torch.full((3,), float(100 * rank + p), device=dev) for p in range(world)]
    if dev.type == "cpu":  # a strided output view too
        base = torch.zeros(world, 6)
        outs = [base[p, ::2] for p in range(world)]
    else:
        outs = [torch.empty(3, device=dev) for _ in range(world)]
    dist.all_to_all(outs, ins)
    for p in range(world):
        c.equal(f"all_to_all list from {p}", outs[p], torch.full((3,), float(100 * p + rank)))
if dev.type == "cpu":
    # object collectives (torch pickles into byte tensors over this backend)
    o = [{"rank": rank, "v": [rank] * 3}] if rank == 0 else [None]
    dist.broadcast_object_list(o, src=0)
    c.check("broadcast_object_list", o[0] == {"rank": 0, "v": [0, 0, 0]}, str(o))
    allo = [None] * world
    dist.all_gather_object(allo, ("r", rank))
    c.check("all_gather_object", allo == [("r", r) for r in range(world)], str(allo))
    got = [None]
    dist.scatter_object_list(got, [f"x{r}" for r in range(world)] if rank == 0 else None, src=0)
    c.check("scatter_object_list", got[0] == f"x{rank}", str(got))
if dev.type == "cpu":
    g = [torch.empty(3) for _ in range(world)] if rank == 0 else None
    dist.gather(torch.full((3,), float(rank)), g, dst=0)
    if rank == 0:
        for r in range(world):
            c.equal(f"gather[{r}]", g[r], torch.full((3,), float(r)))
    o = torch.empty(2)
    dist.scatter(o, [torch.full((2,), float(r * 7)) for r in range(world)] if rank == 0 else None, src=0)
    c.equal("scatter", o, torch.full((2,), float(rank * 7)))
# integer and fp64 payloads (exact): SUM / MIN / MAX / PRODUCT
for dtype in (torch.int64, torch.int32, torch.uint8, torch.float64):
    for op, fold in ((dist.ReduceOp.SUM, lambda a, b: a + b), (dist.ReduceOp.MIN, torch.minimum),
                     (dist.ReduceOp.MAX, torch.maximum), (dist.ReduceOp.PRODUCT, lambda a, b: a * b)):
        def mk(r):
            return ((torch.arange(9) * (r + 1)) % 5 + (1 if op == dist.ReduceOp.PRODUCT else 0)).to(dtype)
        want = mk(0)
        for r in range(1, world):
            want = fold(want, mk(r))
        t = mk(rank).to(dev)
        dist.all_reduce(t, op=op)
        c.equal(f"all_reduce {dtype} {op}", t, want.to(dtype))
c.finish()
