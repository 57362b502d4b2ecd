"""Persistent p2p plans: matched once, started many times with new data.

Every rank sends three tensors (contiguous, strided view, transposed) to
(rank+1) % world and receives from (rank-1) % world; after each start() the
receive buffers must hold the sender's data of that step."""
from common import Checker, init, torch
import commux_b200 as commux

rank, world, dev = init(timeout_s=90)
c = Checker(rank)
peer, src = (rank + 1) % world, (rank - 1) % world
a = torch.zeros(1000, device=dev)
b_full = torch.zeros(40, 64, device=dev, dtype=torch.float64)
b = b_full[:, 8:40:2]
t_full = torch.zeros(24, 36, device=dev, dtype=torch.bfloat16)
ra = torch.zeros(1000, device=dev)
rb = torch.zeros(40, 16, device=dev, dtype=torch.float64)
rt_full = torch.zeros(36, 30, device=dev, dtype=torch.bfloat16)
rt = rt_full[:, 3:27]
plan = commux.p2p_plan(sends=[(a, peer, 5), (b, peer, 6), (t_full.t(), peer, 7)],
                       recvs=[(ra, src, 5), (rb, src, 6), (rt, src, 7)])
for step in range(20):
    a.copy_(torch.arange(1000, device=dev) + 1000 * rank + step)
    b_full.copy_(torch.arange(40 * 64, device=dev, dtype=torch.float64).view(40, 64) * (rank + 1) + step)
    t_full.copy_(((torch.arange(24 * 36, device=dev) % 97) + rank + step).view(24, 36).to(torch.bfloat16))
    plan.start()
    ra_h, rb_h, rt_h = ra.cpu(), rb.cpu(), rt.cpu()
    want_a = torch.arange(1000) + 1000 * src + step
    want_b = (torch.arange(40 * 64, dtype=torch.float64).view(40, 64) * (src + 1) + step)[:, 8:40:2]
    want_t = ((torch.arange(24 * 36) % 97) + src + step).view(24, 36).to(torch.bfloat16).t()
    c.equal(f"plan contiguous step {step}", ra_h, want_a.float())
    c.equal(f"plan strided step {step}", rb_h, want_b)
    c.equal(f"plan transposed step {step}", rt_h, want_t)
if rank == 0:
    print("plan info", plan.info(), flush=True)
c.finish()
