"""commux (B200-native): a torch.distributed backend with MPI-style tag matching.

Gives real ``(sender, tag)`` point-to-point matching (which NCCL lacks) plus
allreduce / reduce / broadcast / barrier / allgather / reduce_scatter /
all_to_all, on CPU and CUDA tensors. Host bytes move through POSIX
shared-memory rings; CUDA bytes move by hand-written sm_100a kernels that read
the matched peer's buffer over NVLink (CUDA IPC) and signal completion through
bounded device flags.

Usage::

    import commux            # or: import commux_b200 as commux
    commux.register()        # registers backends "ucx" and "commux"
    torch.distributed.init_process_group(backend="ucx", init_method="env://")

Public API of the reference package (reference: python/commux/__init__.py:
1-75): ``register``, ``create_backend``, ``preferred_backend``. Added here:
``stats``, ``reset_stats``, ``IOContext``, ``make_tcp_io_context`` and the
``halo`` helpers.
"""

from __future__ import annotations

import os

import torch  # noqa: F401  (loads libtorch/libc10 before the extension)
import torch.distributed as dist

_PKG = os.path.dirname(os.path.abspath(__file__))


class _Unbuilt:
    """Stand-in for the native module when it is not built: every use raises."""

    def __init__(self, err):
        self._err = err

    def __getattr__(self, name):
        raise ImportError(
            "commux_b200 native libraries are not built; run "
            "`python -m commux_b200.build` (or __graft_entry__.build()). "
            f"Original error: {self._err}")


# On a reload after an in-process build the module still holds the stand-in
# of the first import; drop it so the import below finds the built module.
globals().pop("_C", None)
try:
    from . import _C  # noqa: F401
except ImportError as _e:  # the build module itself imports this package
    _C = _Unbuilt(_e)

__all__ = [
    "register", "create_backend", "preferred_backend", "stats", "reset_stats",
    "make_ucp_tag", "TAG_MASK_ANY_SOURCE", "IOContext", "make_tcp_io_context",
    "library_paths", "batch_p2p", "p2p_plan", "transports", "is_commux",
]

_REGISTERED = False
if isinstance(_C, _Unbuilt):
    make_ucp_tag = IOContext = make_tcp_io_context = None
    TAG_MASK_ANY_SOURCE = 0x0000FFFFFFFFFFFF
else:
    make_ucp_tag = _C.make_ucp_tag
    TAG_MASK_ANY_SOURCE = _C.TAG_MASK_ANY_SOURCE
    IOContext = _C.IOContext
    make_tcp_io_context = _C.make_tcp_io_context
    import atexit as _atexit

    # Release CUDA state of groups still alive at exit while the CUDA context
    # exists (interpreter teardown would otherwise free it too late).
    if hasattr(_C, "_release_all"):
        _atexit.register(_C._release_all)


def create_backend(store, rank, size, timeout):
    """torch.distributed creator: returns a c10d::Backend (ProcessGroupUCX)."""
    return _C.create_backend(store, rank, size, timeout)


def register(names=("ucx", "commux")):
    """Register commux with torch.distributed under the given backend name(s).

    Idempotent. Afterwards ``backend="ucx"`` (or ``"commux"``) works anywhere
    torch.distributed expects a backend, for CPU and CUDA tensors.
    """
    global _REGISTERED
    if _REGISTERED:
        return
    for name in names:
        try:
            dist.Backend.register_backend(name, create_backend, devices=["cpu", "cuda"])
        except ValueError:
            # already registered in this process (e.g. by another import path)
            pass
    _REGISTERED = True


def preferred_backend(name="ucx"):
    """Register commux and return the backend name to pass to init_process_group.

    The portable pattern keeps Gloo as the fallback where commux is absent::

        try:
            from commux import preferred_backend
            backend = preferred_backend()   # "ucx"
        except ImportError:
            backend = "gloo"
    """
    register()
    return name


def _backend_of(group=None, device=None):
    group = group if group is not None else dist.distributed_c10d._get_default_group()
    if device is None:
        device = torch.device("cpu")
    return group._get_backend(torch.device(device))


def stats(group=None, device=None) -> dict:
    """Engine counters of this rank's commux backend (messages, bytes, eager vs
    rendezvous, unexpected-queue peak, device launches, IPC cache, ...)."""
    return dict(_C.stats(_backend_of(group, device)))


def reset_stats(group=None, device=None) -> None:
    _C.reset_stats(_backend_of(group, device))


def batch_p2p(sends=(), recvs=(), group=None):
    """Post tagged sends and receives as one batch and return one Work.

    ``sends`` and ``recvs`` are sequences of ``(tensor, peer, tag)`` with peer
    ranks of ``group`` (default group if None). Receives are posted first. This
    is the native form of ``torch.distributed.batch_isend_irecv``: one call
    into the backend for the whole exchange, one readiness event and (for
    messages to self) one copy launch on CUDA.
    """
    group = group if group is not None else dist.distributed_c10d._get_default_group()
    r = list(recvs)
    s = list(sends)
    if not r and not s:
        raise ValueError("commux.batch_p2p: no sends and no receives")
    first = (r + s)[0][0]
    backend = group._get_backend(first.device)
    return _C.batch_p2p(backend, [t for t, _, _ in r], [int(p) for _, p, _ in r], [int(g) for _, _, g in r],
                        [t for t, _, _ in s], [int(p) for _, p, _ in s], [int(g) for _, _, g in s])


def p2p_plan(sends=(), recvs=(), group=None, max_ctas=0):
    """Persistent plan of CUDA sends and receives, matched once.

    ``sends``/``recvs`` are ``(tensor, peer, tag)`` like :func:`batch_p2p`.
    ``plan.start()`` enqueues one exchange of the same buffers on the current
    stream as one CUDA graph: a pull launch that stores this rank's "ready"
    signals, packs narrow rows for peers on other GPUs and copies every
    receive (waiting on the peers' ready flags on the device); when peers on
    other GPUs read this rank's data, its last CTA waits for their
    "consumed" flags. No host matching and no host round trip per step.
    Every rank the plan talks to creates its side in the same order and calls
    start() the same number of times (the analogue of MPI_Startall).
    ``max_ctas`` (or ``plan.set_max_ctas``) caps the launches' grid, leaving
    SMs to kernels that run beside the exchange.
    """
    group = group if group is not None else dist.distributed_c10d._get_default_group()
    r = list(recvs)
    s = list(sends)
    if not r and not s:
        raise ValueError("commux.p2p_plan: no sends and no receives")
    first = (r + s)[0][0]
    backend = group._get_backend(first.device)
    plan = _C.p2p_plan(backend, [t for t, _, _ in r], [int(p) for _, p, _ in r], [int(g) for _, _, g in r],
                       [t for t, _, _ in s], [int(p) for _, p, _ in s], [int(g) for _, _, g in s])
    if max_ctas:
        plan.set_max_ctas(int(max_ctas))
    return plan


def transports(group=None) -> list:
    """Transport to each rank of ``group``: ``"self"``, ``"shm"`` (shared
    memory and, for CUDA tensors, NVLink peer memory on this host) or
    ``"tcp"`` (another host, or ``COMMUX_TRANSPORT=tcp``; CUDA tensors are
    staged through host memory)."""
    return list(_C.transports(_backend_of(group, None)))


def is_commux(group=None, device="cpu") -> bool:
    """True if ``group`` runs on the commux backend."""
    try:
        return bool(_C.is_commux(_backend_of(group, device)))
    except Exception:
        return False


def library_paths() -> list[str]:
    """Paths of the native libraries this package loads."""
    lib = os.path.join(_PKG, "lib")
    return [os.path.join(lib, n) for n in ("libcommux.so", "libcommux_io.so", "libcommux_cuda.so")
            if os.path.exists(os.path.join(lib, n))]
