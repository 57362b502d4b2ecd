"""Jacobi steps with the exchange overlapped with the core update give the
same field as sequential steps (exchange, then the whole update), bit for
bit, at any world size (one rank per GPU where the box has enough)."""
from common import Checker, init, torch
from commux_b200.models.halo3d import Jacobi3D

rank, world, dev = init(timeout_s=120)
c = Checker(rank)
for dtype, n in ((torch.float64, 40), (torch.float32, 37)):
    a = Jacobi3D(n * world, halo=2, dims=(world, 1, 1), dtype=dtype, seed=3)
    b = Jacobi3D(n * world, halo=2, dims=(world, 1, 1), dtype=dtype, seed=3)
    c.equal(f"{dtype} same start", a.u.cpu(), b.u.cpu())
    for k in range(4):
        a.step()
        b.step_overlapped()
        torch.cuda.synchronize()
        ra, rb = float(a.residual), float(b.residual)
        c.check(f"{dtype} step {k} residual", abs(ra - rb) <= 1e-9 * max(1.0, abs(ra)), f"{ra} vs {rb}")
    h = a.h
    c.equal(f"{dtype} interior after 4 steps", a.u[h:-h, h:-h, h:-h].cpu(), b.u[h:-h, h:-h, h:-h].cpu())
c.finish()
