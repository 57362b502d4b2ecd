"""Shared setup of the multi-rank worker scripts."""

import datetime
import operator
import os
import re
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import commux_b200 as commux  # noqa: E402


def init(timeout_s=60):
    """Register commux, init the default group, pick this rank's device:
    GPU rank % count, or GPU 0 for every rank with CMX_SHARED_GPU=1 (ranks
    sharing one GPU take the host-gated paths)."""
    commux.register()
    dist.init_process_group(os.environ.get("CMX_BACKEND", "ucx"),
                            timeout=datetime.timedelta(seconds=timeout_s))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cpu")
    if os.environ.get("CMX_DEVICE") == "cuda":
        n = torch.cuda.device_count()
        idx = 0 if os.environ.get("CMX_SHARED_GPU") == "1" else rank % n
        torch.cuda.set_device(idx)
        dev = torch.device("cuda", idx)
    return rank, world, dev


_OPS = {">": operator.gt, ">=": operator.ge, "==": operator.eq, "<": operator.lt, "<=": operator.le}


def expected_path_failures():
    """Checks of CMX_EXPECT against this rank's backend counters: a comma
    list of `<counter><op><int>` (e.g. "cuda_sends_device_flag>0,
    cuda_sends_host_fin==0"), so a test states which transport path must
    have run and fails when the work silently took another one."""
    spec = os.environ.get("CMX_EXPECT", "")
    if not spec:
        return []
    st = commux.stats()
    bad = []
    for cond in filter(None, (x.strip() for x in spec.split(","))):
        m = re.fullmatch(r"(\w+)(>=|<=|==|>|<)(-?\d+)", cond)
        if m is None:
            bad.append(f"malformed CMX_EXPECT condition {cond!r}")
            continue
        key, op, val = m.groups()
        got = st.get(key)
        if got is None or not _OPS[op](got, int(val)):
            bad.append(f"expected path {cond}: {key}={got}")
    return bad


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
        self.failures += [f"rank {self.rank} {m}" for m in expected_path_failures()]
        for m in self.failures:
            print("FAIL", m, flush=True)
        n = torch.tensor([float(len(self.failures))])
        dist.all_reduce(n)
        total = int(n.item())
        if self.rank == 0:
            print(f"{total} failure(s)" + ("" if total else " -- PASSED"), flush=True)
        dist.destroy_process_group()
        sys.exit(1 if total else 0)
