"""3-D Jacobi stencil with domain decomposition: the flagship halo workload.

A global periodic field of ``global_n``^3 points (fp64 by default) is split
over a near-cubic grid of ranks (1024^3 over 2x2x2 -> 512^3 per rank), with a
ghost shell of width ``halo``. One timestep exchanges the 26 halo slabs with
the neighbours through commux's tagged p2p (tags 1000 + direction) and then
applies one 7-point Jacobi sweep (``commux_b200.ops.jacobi7``, an sm_100a
kernel) from ``u`` into ``v``; the fields swap roles each step.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import jacobi7
from ..parallel.halo import CartGrid, HaloExchange, factor3


class Jacobi3D:
    def __init__(self, global_n: int = 1024, halo: int = 2, dims=None, dtype=torch.float64,
                 device=None, group=None, seed: int = 0, overlap_ctas: int | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dims = tuple(dims) if dims is not None else factor3(self.world)
        if self.dims[0] * self.dims[1] * self.dims[2] != self.world:
            raise ValueError(f"process grid {self.dims} does not match world size {self.world}")
        gn = (global_n,) * 3 if isinstance(global_n, int) else tuple(global_n)
        for g, d in zip(gn, self.dims):
            if g % d:
                raise ValueError(f"global size {gn} is not divisible by the grid {self.dims}")
        self.interior = tuple(g // d for g, d in zip(gn, self.dims))
        self.h = halo
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        shape = tuple(n + 2 * halo for n in self.interior)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed * 1000003 + self.rank)
        self.u = torch.empty(shape, dtype=dtype, device=self.device)
        self.u.uniform_(-1.0, 1.0, generator=gen)
        self.v = self.u.clone()
        self.residual = torch.zeros(1, dtype=torch.float64, device=self.device)
        self.grid = CartGrid(self.dims, self.rank)
        self.halo = HaloExchange(self.interior, halo, self.grid, group=group)
        # step_overlapped() exchanges through its own plans, whose launches
        # take at most `overlap_ctas` CTAs (default one per SM) so the core
        # update keeps most of every SM while the exchange runs
        if overlap_ctas is None:
            overlap_ctas = int(os.environ.get(
                "COMMUX_OVERLAP_CTAS", torch.cuda.get_device_properties(self.device).multi_processor_count))
        self.halo_overlap = HaloExchange(self.interior, halo, self.grid, group=group, max_ctas=overlap_ctas)
        self._xstream = None  # side stream of step_overlapped()

    @property
    def halo_bytes(self) -> int:
        """Bytes this rank sends (and receives) per exchange."""
        return self.halo.message_bytes(self.u.element_size())

    def exchange(self) -> None:
        self.halo.exchange(self.u)

    def update(self) -> None:
        self.residual.zero_()
        jacobi7(self.u, self.v, self.h, self.residual)
        self.u, self.v = self.v, self.u

    def step(self) -> None:
        self.exchange()
        self.update()

    def step_overlapped(self) -> None:
        """One timestep with the exchange hidden behind the core update.

        The exchange (reads u's boundary slabs, writes u's ghost cells) runs on
        a high-priority side stream while the core cells -- whose stencil
        reads no ghost cell -- are updated on the current stream; the
        one-cell boundary layer follows once the ghosts have arrived. Writes
        the same v as ``step()`` (bit for bit; the residual's summation order
        differs).
        """
        h = self.h
        if min(self.interior) < 3:
            self.step()
            return
        main = torch.cuda.current_stream(self.device)
        if self._xstream is None:
            self._xstream = torch.cuda.Stream(device=self.device, priority=-1)
        xs = self._xstream
        xs.wait_stream(main)  # u complete (the previous step's update)
        with torch.cuda.stream(xs):
            self.halo_overlap.exchange(self.u)
        self.residual.zero_()
        jacobi7(self.u, self.v, h, self.residual, part="core")
        main.wait_stream(xs)
        jacobi7(self.u, self.v, h, self.residual, part="shell")
        self.u, self.v = self.v, self.u

    def inject(self, forcing: torch.Tensor, scale: float = 1e-6) -> None:
        """Add a per-step source plane (shape interior[1:]) to the middle z-plane."""
        h = self.h
        z = h + self.interior[0] // 2
        self.u[z, h:h + self.interior[1], h:h + self.interior[2]].add_(forcing, alpha=scale)
