"""Halo exchange over commux's tagged p2p (domain decomposition of a 3-D field).

A field of interior size (nz, ny, nx) per rank carries a ghost shell of width
``halo``. Ranks form a periodic Cartesian grid; each rank exchanges with its
26 neighbours (6 faces, 12 edges, 8 corners). A message that travels in
direction d = (dz, dy, dx) carries tag ``1000 + index(d)``: the sender's
interior slab next to its d side lands in the receiver's ghost slab on its -d
side. Both are passed as strided views -- the CUDA transport gathers the
sender's slab and scatters into the receiver's ghost region inside its copy
kernel, with no pack/unpack buffers. The reference backend ships no halo
driver (its consumer "snapy" hands it per-variable ghost tensors, reference:
src/process_group_ucx.cpp:131-134); this module is that driver.
"""

from __future__ import annotations

import itertools
import math
import os

import torch
import torch.distributed as dist

DIRECTIONS = [d for d in itertools.product((-1, 0, 1), repeat=3) if d != (0, 0, 0)]
TAG_BASE = 1000


def dir_index(d) -> int:
    """Index of direction d in the 3x3x3 stencil (0..26, the centre is 13)."""
    return (d[0] + 1) * 9 + (d[1] + 1) * 3 + (d[2] + 1)


def factor3(n: int) -> tuple[int, int, int]:
    """Near-cubic process grid (dz, dy, dx) with dz*dy*dx == n, dz >= dy >= dx."""
    dims = [1, 1, 1]
    f, m = 2, n
    primes = []
    while m > 1:
        while m % f == 0:
            primes.append(f)
            m //= f
        f += 1
    for p in sorted(primes, reverse=True):
        i = dims.index(min(dims))
        dims[i] *= p
    dims.sort(reverse=True)
    return tuple(dims)


class CartGrid:
    """Periodic Cartesian process grid; rank = (cz * Dy + cy) * Dx + cx."""

    def __init__(self, dims, rank: int):
        self.dims = tuple(dims)
        self.rank = rank
        Dz, Dy, Dx = self.dims
        self.coords = (rank // (Dy * Dx), (rank // Dx) % Dy, rank % Dx)

    def rank_of(self, coords) -> int:
        Dz, Dy, Dx = self.dims
        cz, cy, cx = (c % D for c, D in zip(coords, self.dims))
        return (cz * Dy + cy) * Dx + cx

    def neighbor(self, d) -> int:
        return self.rank_of(tuple(c + o for c, o in zip(self.coords, d)))


def _axis_send(o: int, n: int, h: int) -> slice:
    return slice(h, 2 * h) if o < 0 else (slice(n, n + h) if o > 0 else slice(h, h + n))


def _axis_recv(o: int, n: int, h: int) -> slice:
    # data travelling in +o lands in the ghost slab on the receiver's -o side
    return slice(0, h) if o > 0 else (slice(n + h, n + 2 * h) if o < 0 else slice(h, h + n))


class HaloExchange:
    """26-direction tagged halo exchange of halo-padded fields.

    ``exchange(u)`` posts every receive and send of one field as one
    ``batch_isend_irecv`` (a coalescing window, so with ``COMMUX_GROUP=1`` the
    CUDA transport launches one copy per batch) and waits for completion on
    the current stream.
    """

    def __init__(self, interior, halo: int, grid: CartGrid, group=None, directions=None, max_ctas: int = 0):
        self.max_ctas = max_ctas  # grid cap of the persistent plans (0: default)
        self.n = tuple(interior)
        self.h = halo
        self.grid = grid
        self.group = group
        self.directions = list(directions or DIRECTIONS)
        self._native = None
        self._plans = {}  # views (+ persistent plan) per field; fields alternate
        self.use_plans = os.environ.get("COMMUX_HALO_PLAN", "1") != "0"
        for n in self.n:
            if n < halo:
                raise ValueError("interior must be at least as wide as the halo")

    def send_view(self, u: torch.Tensor, d) -> torch.Tensor:
        return u[tuple(_axis_send(o, n, self.h) for o, n in zip(d, self.n))]

    def recv_view(self, u: torch.Tensor, d) -> torch.Tensor:
        return u[tuple(_axis_recv(o, n, self.h) for o, n in zip(d, self.n))]

    def message_bytes(self, elem_size: int) -> int:
        """Bytes this rank sends per exchange (= bytes it receives)."""
        total = 0
        for d in self.directions:
            total += math.prod(self.h if o else n for o, n in zip(d, self.n)) * elem_size
        return total

    def remote_bytes(self, elem_size: int, rank: int) -> int:
        """Bytes this rank receives from other ranks per exchange (with one
        GPU per rank: the bytes that cross NVLink into this GPU)."""
        total = 0
        for d in self.directions:
            if self.grid.neighbor(tuple(-o for o in d)) != rank:
                total += math.prod(self.h if o else n for o, n in zip(d, self.n)) * elem_size
        return total

    def ops(self, u: torch.Tensor) -> list:
        ops = []
        for d in self.directions:
            src = self.grid.neighbor(tuple(-o for o in d))
            ops.append(dist.P2POp(dist.irecv, self.recv_view(u, d), src,
                                  group=self.group, tag=TAG_BASE + dir_index(d)))
        for d in self.directions:
            ops.append(dist.P2POp(dist.isend, self.send_view(u, d), self.grid.neighbor(d),
                                  group=self.group, tag=TAG_BASE + dir_index(d)))
        return ops

    def start(self, u: torch.Tensor) -> list:
        """Post the 26 receives and 26 sends; returns the Works to wait on.

        On the commux backend this is one native batch call; on any other
        backend it goes through ``torch.distributed.batch_isend_irecv``.
        """
        if self._native is None:
            import commux_b200

            self._native = commux_b200.is_commux(self.group, u.device)
        if not self._native:
            return dist.batch_isend_irecv(self.ops(u))
        import commux_b200

        key = (u.data_ptr(), tuple(u.shape), tuple(u.stride()))
        plan = self._plans.get(key)
        if plan is None:
            recvs, sends = [], []
            for d in self.directions:
                tag = TAG_BASE + dir_index(d)
                recvs.append((self.recv_view(u, d), self.grid.neighbor(tuple(-o for o in d)), tag))
                sends.append((self.send_view(u, d), self.grid.neighbor(d), tag))
            if len(self._plans) >= 8:
                self._plans.clear()
            persistent = None
            if u.is_cuda and self.use_plans and "tcp" not in commux_b200.transports(self.group):
                # matched once; every later exchange of this field replays
                # one CUDA graph (collective: all ranks reach this together)
                persistent = commux_b200.p2p_plan(sends=sends, recvs=recvs, group=self.group,
                                                  max_ctas=self.max_ctas)
            plan = self._plans[key] = (sends, recvs, persistent)
        if plan[2] is not None:
            plan[2].start()
            return []
        return [commux_b200.batch_p2p(sends=plan[0], recvs=plan[1], group=self.group)]

    def exchange(self, u: torch.Tensor) -> None:
        for w in self.start(u):
            w.wait()


def reference_exchange(global_field: torch.Tensor, dims, halo: int) -> list[torch.Tensor]:
    """Single-process oracle: split a periodic global interior field into the
    padded blocks of a ``dims`` grid with ghost shells filled from the
    periodic neighbours (what a correct exchange must produce)."""
    Gz, Gy, Gx = global_field.shape
    Dz, Dy, Dx = dims
    nz, ny, nx = Gz // Dz, Gy // Dy, Gx // Dx
    h = halo
    blocks = []
    for r in range(Dz * Dy * Dx):
        cz, cy, cx = r // (Dy * Dx), (r // Dx) % Dy, r % Dx
        iz = (torch.arange(cz * nz - h, (cz + 1) * nz + h) % Gz)
        iy = (torch.arange(cy * ny - h, (cy + 1) * ny + h) % Gy)
        ix = (torch.arange(cx * nx - h, (cx + 1) * nx + h) % Gx)
        blocks.append(global_field[iz][:, iy][:, :, ix].clone())
    return blocks
