#!/usr/bin/env python
"""Tagged p2p bandwidth over NVLink: every rank exchanges a buffer with a
partner (rank ^ 1) through a persistent plan, both directions at once, and
reports per-direction GB/s as the max-over-ranks device time (CUDA events
around K plan starts, after warm-up). Also runs a strided case shaped like a
halo face (rows of `--row` bytes at a pitch of `--pitch` bytes).

    torchrun --nproc-per-node 2 benchmarks/p2p_bandwidth.py
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes", default="1048576,4194304,16777216,67108864,268435456")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--row", type=int, default=16, help="bytes per row of the strided case")
    ap.add_argument("--pitch", type=int, default=4128, help="row pitch (bytes) of the strided case")
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    import commux_b200 as commux
    from commux_b200.utils import env_rank, free_port

    rank, world, local = env_rank()
    assert world % 2 == 0, "ranks pair up (rank ^ 1)"
    torch.cuda.set_device(local % torch.cuda.device_count())
    commux.register()
    if "MASTER_ADDR" not in os.environ:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group("ucx", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    peer = rank ^ 1
    cases = [("contiguous", int(s), None) for s in args.sizes.split(",")]
    for s in args.sizes.split(","):
        rows = int(s) // args.row
        cases.append((f"rows of {args.row} B at pitch {args.pitch} B", rows * args.row, rows))
    for name, nbytes, rows in cases:
        if rows is None:
            src = torch.ones(nbytes // 4, device="cuda")
            dst = torch.zeros_like(src)
            sv, rv = src, dst
        else:
            per = args.pitch // 4
            w = args.row // 4
            src = torch.ones(rows, per, device="cuda")
            dst = torch.zeros(rows, per, device="cuda")
            sv, rv = src[:, :w], dst[:, per - w:]
        plan = commux.p2p_plan(sends=[(sv, peer, 5)], recvs=[(rv, peer, 5)])
        for _ in range(args.warmup):
            plan.start()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            plan.start()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.iters], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
        if rank == 0:
            print(json.dumps({"case": name, "bytes": nbytes, "n_gpus": world, "us": round(ms * 1e3, 2),
                              "GBps_per_direction": round(nbytes / (ms * 1e-3) / 1e9, 1),
                              "frac_of_770": round(nbytes / (ms * 1e-3) / 770e9, 3)}), flush=True)
        del plan
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
