"""Multi-rank 26-direction halo exchange against the single-process oracle,
for several dtypes and halo widths: fp64 with halo 2 (16-byte x-face rows),
fp32 with halo 2 (8-byte rows: the narrow rows and the wide ones fall in
different copy classes), int16 with halo 3 (6-byte rows). Each field is
exchanged twice (a persistent plan is matched once, then started again)."""

from common import Checker, init, torch
from commux_b200.parallel.halo import CartGrid, HaloExchange, factor3, reference_exchange

rank, world, dev = init()
c = Checker(rank)
dims = factor3(world)
grid = CartGrid(dims, rank)
cz, cy, cx = grid.coords
for dtype, n, h in ((torch.float64, 6, 2), (torch.float32, 8, 2), (torch.int16, 7, 3)):
    G = tuple(n * d for d in dims)
    glob = (torch.arange(G[0] * G[1] * G[2], dtype=torch.float64).view(*G) % 30000).to(dtype)
    u = torch.full((n + 2 * h,) * 3, -1, dtype=dtype)
    u[h:-h, h:-h, h:-h] = glob[cz * n:(cz + 1) * n, cy * n:(cy + 1) * n, cx * n:(cx + 1) * n]
    u = u.to(dev)
    ex = HaloExchange((n, n, n), h, grid)
    for _ in range(2):
        ex.exchange(u)
    want = reference_exchange(glob, dims, h)[rank]
    c.equal(f"halo exchange {dtype} n={n} h={h}", u, want)
c.finish()
