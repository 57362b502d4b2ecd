"""Shared setup of the multi-rank worker scripts."""

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import commux_b200 as commux  # noqa: E402


def init(timeout_s=60):
    """Register commux, init the default group, pick this rank's device."""
    commux.register()
    dist.init_process_group(os.environ.get("CMX_BACKEND", "ucx"),
                            timeout=datetime.timedelta(seconds=timeout_s))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cpu")
    if os.environ.get("CMX_DEVICE") == "cuda":
        n = torch.cuda.device_count()
        torch.cuda.set_device(rank % n)
        dev = torch.device("cuda", rank % n)
    return rank, world, dev


class Checker:
    """Counts failures and agrees on them with an all_reduce, so no rank
    leaves a collective early (reference idiom: tests/test_collectives.py:83-89)."""

    def __init__(self, rank):
        self.rank = rank
        self.failures = []

    def check(self, name, ok, detail=""):
        if not ok:
            self.failures.append(f"{name}: rank {self.rank} {detail}")

    def equal(self, name, got, want):
        ok = torch.equal(got.cpu(), want.cpu())
        self.check(name, ok, f"got {got.flatten()[:8].tolist()} want {want.flatten()[:8].tolist()}")

    def finish(self):
        for m in self.failures:
            print("FAIL", m, flush=True)
        n = torch.tensor([float(len(self.failures))])
        dist.all_reduce(n)
        total = int(n.item())
        if self.rank == 0:
            print(f"{total} failure(s)" + ("" if total else " -- PASSED"), flush=True)
        dist.destroy_process_group()
        sys.exit(1 if total else 0)
