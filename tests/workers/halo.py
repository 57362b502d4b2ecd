"""Multi-rank 26-direction halo exchange against the single-process oracle."""
import os

from common import Checker, init, torch, dist
from commux_b200.parallel.halo import CartGrid, HaloExchange, factor3, reference_exchange

rank, world, dev = init()
c = Checker(rank)
dims = factor3(world)
n, h = 6, 2
G = tuple(n * d for d in dims)
glob = torch.arange(G[0] * G[1] * G[2], dtype=torch.float64).view(*G)
grid = CartGrid(dims, rank)
cz, cy, cx = grid.coords
u = torch.full((n + 2 * h,) * 3, -1.0, dtype=torch.float64)
u[h:-h, h:-h, h:-h] = glob[cz * n:(cz + 1) * n, cy * n:(cy + 1) * n, cx * n:(cx + 1) * n]
u = u.to(dev)
ex = HaloExchange((n, n, n), h, grid)
for _ in range(2):
    ex.exchange(u)
want = reference_exchange(glob, dims, h)[rank]
c.equal("halo exchange", u, want)
c.finish()
