#!/usr/bin/env python
"""Timing of the mixed tagged workload on CPU tensors, on this backend or on
Gloo (the comparator; the reference UCX backend cannot be
built offline). One iteration: every rank posts 64 non-blocking irecv, then
64 isend of fp32 tensors (1..1M elements, log-spaced, tags 100..163 in
shuffled order, seed 0), then all_reduce SUM and MAX of a 1M-element fp32
tensor and a broadcast from rank 0. Reports the max over ranks of the mean
iteration time after warm-up (host wall clock: CPU tensors).

    torchrun --nproc-per-node 2 benchmarks/cpu_mixed_tagged.py --backend ucx
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import random
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--backend", default="ucx", choices=["ucx", "gloo"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    import commux_b200 as commux
    from commux_b200.utils import env_rank, free_port

    rank, world, _ = env_rank()
    commux.register()
    if "MASTER_ADDR" not in os.environ:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group(args.backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    sizes = sorted({max(1, int(round(10 ** (6 * i / 63)))) for i in range(64)})
    while len(sizes) < 64:
        sizes.append(sizes[-1] + 1)
    tags = list(range(100, 164))
    order = list(range(64))
    random.Random(0).shuffle(order)
    peer, src = (rank + 1) % world, (rank - 1) % world
    sends = [torch.randn(sizes[i], generator=torch.Generator().manual_seed(1000 * rank + i)) for i in range(64)]
    bufs = [torch.empty(sizes[i]) for i in range(64)]
    data = torch.randn(1 << 20, generator=torch.Generator().manual_seed(rank))

    def one():
        recvs = [dist.irecv(bufs[i], src, tag=tags[i]) for i in order]
        outs = [dist.isend(sends[i], peer, tag=tags[i]) for i in reversed(order)]
        for w in recvs + outs:
            w.wait()
        for op in (dist.ReduceOp.SUM, dist.ReduceOp.MAX):
            t = data.clone()
            dist.all_reduce(t, op=op)
        b = data.clone()
        dist.broadcast(b, src=0)

    for _ in range(args.warmup):
        one()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.iters):
        one()
    dt = (time.perf_counter() - t0) / args.iters
    t = torch.tensor([dt], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        moved = sum(sizes) * 4 + 3 * (1 << 22)
        print(json.dumps({"workload": "cpu mixed tagged p2p + allreduce + broadcast", "backend": args.backend, "world": world,
                          "ms_per_iter": round(float(t) * 1e3, 3),
                          "payload_MB_per_rank": round(moved / 1e6, 2)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
