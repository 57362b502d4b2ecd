"""Compute kernels of the workloads (sm_100a, in commux_b200._ops) and their
plain-PyTorch references used by the numerics tests."""

from __future__ import annotations

import torch

try:
    from .. import _ops as _native
except ImportError as _e:  # pragma: no cover - only when the extension is unbuilt
    _native = None
    _err = _e


def _need_native():
    if _native is None:
        raise ImportError("commux_b200._ops is not built; run `python -m commux_b200.build` "
                          f"({_err})")
    return _native


_PARTS = {"all": 0, "core": 1, "shell": 2}


def jacobi7(u: torch.Tensor, v: torch.Tensor, halo: int, residual: torch.Tensor | None = None,
            part: str = "all") -> None:
    """v[interior] = mean of the 6 face neighbours of u; residual += sum((v-u)^2).

    ``part`` selects the cells: "all" (the interior), "core" (cells whose
    stencil reads no ghost cell, so it may run while the halo exchange fills
    the ghosts) or "shell" (the one-cell layer around the core). "core" and
    "shell" together write exactly what "all" writes.

    CUDA only (sm_100a kernel); fails loudly if the extension is missing.
    """
    _need_native().jacobi7(u, v, halo, residual, _PARTS[part])


def launches() -> int:
    """Number of kernels this extension launched in this process."""
    return _need_native().launches() if _native is not None else 0


def jacobi7_reference(u: torch.Tensor, v: torch.Tensor, halo: int) -> float:
    """fp64 PyTorch reference of jacobi7 (writes v's interior, returns the residual)."""
    h = halo
    c = u[h:-h, h:-h, h:-h]
    s = (u[h - 1:-h - 1, h:-h, h:-h] + u[h + 1:u.shape[0] - h + 1, h:-h, h:-h]
         + u[h:-h, h - 1:-h - 1, h:-h] + u[h:-h, h + 1:u.shape[1] - h + 1, h:-h]
         + u[h:-h, h:-h, h - 1:-h - 1] + u[h:-h, h:-h, h + 1:u.shape[2] - h + 1])
    new = s / 6
    v[h:-h, h:-h, h:-h] = new
    return float(((new.double() - c.double()) ** 2).sum())
