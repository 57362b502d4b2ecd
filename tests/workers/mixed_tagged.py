"""Mixed tagged workload on CPU tensors: each rank posts 64 non-blocking irecv
then 64 isend of fp32 tensors (1..1M elements, log-spaced) with tags 100..163
in shuffled order (seed 0); all_reduce SUM and MAX of a 1M-element fp32 tensor
~N(0,1) seeded by rank; broadcast from rank 0. Results are checked bit-exact
against a reference computation: the left fold over ranks in rank order."""
import random
import time

from common import Checker, init, torch, dist

rank, world, dev = init(timeout_s=120)
c = Checker(rank)
sizes = sorted({max(1, int(round(10 ** (6 * i / 63)))) for i in range(64)})
while len(sizes) < 64:
    sizes.append(sizes[-1] + 1)
tags = list(range(100, 164))
order = list(range(64))
random.Random(0).shuffle(order)


def payload(src, i):
    g = torch.Generator().manual_seed(1000 * src + i)
    return torch.randn(sizes[i], generator=g, dtype=torch.float32)


t0 = time.perf_counter()
if world >= 2:
    peer = (rank + 1) % world
    src = (rank - 1) % world
    bufs = [torch.empty(sizes[i], device=dev) for i in range(64)]
    recvs = [dist.irecv(bufs[i], src, tag=tags[i]) for i in order]
    sends = [dist.isend(payload(rank, i).to(dev), peer, tag=tags[i]) for i in reversed(order)]
    for w in recvs + sends:
        w.wait()
    for i in range(64):
        c.equal(f"p2p tag {tags[i]}", bufs[i], payload(src, i))
t_p2p = time.perf_counter() - t0


def data(r):
    return torch.randn(1 << 20, generator=torch.Generator().manual_seed(r), dtype=torch.float32)


for op, fold in ((dist.ReduceOp.SUM, torch.add), (dist.ReduceOp.MAX, torch.maximum)):
    want = data(0)
    for r in range(1, world):
        want = fold(want, data(r))
    t = data(rank).to(dev)
    dist.all_reduce(t, op=op)
    c.equal(f"all_reduce {op} bit-exact", t, want)
b = data(rank).to(dev)
dist.broadcast(b, src=0)
c.equal("broadcast", b, data(0))
if rank == 0:
    print(f"p2p phase {t_p2p * 1e3:.2f} ms", flush=True)
c.finish()
