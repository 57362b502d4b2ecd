#!/usr/bin/env python
"""Host-path latency and bandwidth on CPU tensors: all_reduce of one float,
barrier and broadcast of one float (median of --calls calls), and the
round-trip bandwidth of 1, 16 and 64 MiB tagged messages between ranks 0
and 1. Runs on this backend or on Gloo; COMMUX_TRANSPORT=tcp puts every
peer on the TCP transport. Prints one JSON line per measurement from rank 0
(host wall clock).

    torchrun --nproc-per-node 2 benchmarks/host_latency.py [--backend gloo]
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--backend", default="ucx", choices=["ucx", "gloo"])
    ap.add_argument("--calls", type=int, default=2000)
    ap.add_argument("--mib", default="1,16,64")
    ap.add_argument("--iters", type=int, default=10)
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
    transport = os.environ.get("COMMUX_TRANSPORT", "auto") if args.backend == "ucx" else "gloo"

    def emit(**kv):
        if rank == 0:
            print(json.dumps(dict(backend=args.backend, transport=transport, world=world, **kv)), flush=True)

    one = torch.ones(1)
    for name, f in (("all_reduce_1f", lambda: dist.all_reduce(one)), ("barrier", dist.barrier),
                    ("broadcast_1f", lambda: dist.broadcast(one, 0))):
        for _ in range(min(200, args.calls)):
            f()
        lat = []
        for _ in range(args.calls):
            t0 = time.perf_counter()
            f()
            lat.append(time.perf_counter() - t0)
        emit(op=name, us_p50=round(statistics.median(lat) * 1e6, 1))

    for mib in map(int, args.mib.split(",")):
        n = mib * (1 << 20) // 4
        x, y = torch.ones(n), torch.empty(n)
        dist.barrier()
        t0 = 0.0
        for it in range(3 + args.iters):
            if it == 3:
                dist.barrier()
                t0 = time.perf_counter()
            if rank == 0:
                dist.send(x, 1, tag=1)
                dist.recv(y, 1, tag=2)
            elif rank == 1:
                dist.recv(y, 0, tag=1)
                dist.send(x, 0, tag=2)
        dt = (time.perf_counter() - t0) / args.iters
        emit(op="p2p_round_trip", mib=mib, ms=round(dt * 1e3, 3), gib_per_s=round(2 * mib / 1024 / dt, 2))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
