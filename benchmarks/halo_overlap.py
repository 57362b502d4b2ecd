#!/usr/bin/env python
"""Sequential against overlapped Jacobi timesteps (one process per GPU,
512^3 fp64 per GPU, halo 2), for several grid caps of the overlapped step's
exchange: the exchange runs on a high-priority side stream with at most
`cap` CTAs while the core cells update, then the one-cell boundary layer.
Step times are device-timed with CUDA events, median over 20 steps of the
per-step max over ranks. Prints one JSON line.

    torchrun --nproc-per-node N benchmarks/halo_overlap.py
"""

from __future__ import annotations

import datetime
import json
import os
import statistics
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    os.environ.setdefault("COMMUX_GROUP", "1")
    import torch
    import torch.distributed as dist

    import commux_b200 as commux
    from commux_b200.models.halo3d import Jacobi3D
    from commux_b200.parallel.halo import factor3
    from commux_b200.utils import env_rank, free_port, rank_max

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    commux.register()
    if "MASTER_ADDR" not in os.environ:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group("ucx", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    dims = factor3(world)
    m = Jacobi3D(tuple(512 * d for d in dims), halo=2, dims=dims, seed=0)

    def timed(fn, k=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(k + 1)]
        ev[0].record()
        for i in range(k):
            fn()
            ev[i + 1].record()
        torch.cuda.synchronize()
        return round(statistics.median(rank_max([ev[i].elapsed_time(ev[i + 1]) for i in range(k)])), 4)

    res = {"n_gpus": world, "sequential_step_ms": timed(m.step)}
    for cap in (32, 74, 148, 296, 592):
        m.halo_overlap.max_ctas = cap
        m.halo_overlap._plans.clear()
        res[f"overlapped_step_ms_cap{cap}"] = timed(m.step_overlapped)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
