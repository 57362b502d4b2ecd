#!/usr/bin/env python
"""allreduce / reduce / broadcast sweep, commux device kernels vs NCCL.

Sizes 8 B .. 1 GB (powers of 4 by default), dtypes fp32/bf16/fp16, ops
SUM/MAX/AVG, on every GPU of the launch (torchrun --nproc-per-node N). Each
point is timed with CUDA events on the caller's stream (max over ranks, after
warm-up, inputs re-used: sizes above the 126 MB L2 stream from HBM) and
reported as algorithm bandwidth and bus bandwidth (allreduce: 2(P-1)/P x size
/ time; reduce/broadcast: size / time) and as the fraction of the NVLink
roofline (bus bandwidth / 770 GB/s, the measured peer-copy rate per direction).
NCCL runs in the same process on a second process group as the comparator.
Each row names the device algorithm the timed commux calls took on rank 0
(`commux_path`, from the backend's per-algorithm counters).

    torchrun --nproc-per-node 8 benchmarks/collectives_sweep.py --max-bytes 1073741824
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


# per-algorithm call counters of the device collectives (commux.stats());
# "gather" counts the allgather and broadcast kernels (root push, scatter +
# allgather)
PATHS = ("oneshot", "twoshot", "nvls", "gather", "chain")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-bytes", type=int, default=8)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--factor", type=int, default=4)
    ap.add_argument("--dtypes", default="fp32,bf16,fp16")
    ap.add_argument("--ops", default="sum,max,avg")
    ap.add_argument("--colls", default="allreduce,reduce,broadcast")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--no-nccl", action="store_true")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    import commux_b200 as commux
    from commux_b200.utils import env_rank, free_port

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    commux.register()
    if "MASTER_ADDR" not in os.environ:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group("ucx", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600))
    groups = {"commux": None}
    if not args.no_nccl and world > 1:
        groups["nccl"] = dist.new_group(backend="nccl")
    dt = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}
    ops = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "avg": dist.ReduceOp.AVG}
    def path_counters():
        return commux.stats()

    results = []
    size = args.min_bytes
    sizes = []
    while size <= args.max_bytes:
        sizes.append(size)
        size *= args.factor
    for coll in args.colls.split(","):
        for dname in args.dtypes.split(","):
            dtype = dt[dname]
            esz = torch.tensor([], dtype=dtype).element_size()
            for oname in (args.ops.split(",") if coll != "broadcast" else ["-"]):
                for nbytes in sizes:
                    n = max(1, nbytes // esz)
                    x = torch.randn(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(rank)).to(dtype)
                    row = {"coll": coll, "dtype": dname, "op": oname, "bytes": n * esz, "n_gpus": world}
                    for gname, g in groups.items():
                        if gname == "nccl" and coll == "reduce" and oname == "avg":
                            continue

                        def call():
                            if coll == "allreduce":
                                dist.all_reduce(x, op=ops[oname], group=g)
                            elif coll == "reduce":
                                dist.reduce(x, dst=0, op=ops[oname], group=g)
                            else:
                                dist.broadcast(x, src=0, group=g)

                        for _ in range(args.warmup):
                            call()
                        torch.cuda.synchronize()
                        dist.barrier()
                        before = path_counters() if gname == "commux" else None
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        e0.record()
                        for _ in range(args.iters):
                            call()
                        e1.record()
                        torch.cuda.synchronize()
                        t = torch.tensor([e0.elapsed_time(e1) / args.iters], dtype=torch.float64)
                        dist.all_reduce(t, op=dist.ReduceOp.MAX)
                        ms = float(t)
                        algbw = n * esz / (ms * 1e-3) / 1e9
                        busbw = algbw * (2 * (world - 1) / world if coll == "allreduce" else 1.0)
                        row[f"{gname}_us"] = round(ms * 1e3, 2)
                        row[f"{gname}_busbw_GBps"] = round(busbw, 2)
                        # NVLink roofline: bus bandwidth against the measured
                        # 770 GB/s per direction of one GPU's links
                        row[f"{gname}_frac_of_nvlink"] = round(busbw / 770.0, 3)
                        if before is not None:
                            # the device algorithm(s) the timed calls took on
                            # this rank (counter deltas); "none": no device
                            # kernel ran (host staging, e.g. ranks sharing a GPU)
                            after = path_counters()
                            row["commux_path"] = "+".join(
                                k for k in PATHS if after.get(f"coll_{k}", 0) > before.get(f"coll_{k}", 0)) or "none"
                    if rank == 0:
                        print(json.dumps(row), flush=True)
                    results.append(row)
    if rank == 0 and args.out:
        with open(args.out, "w") as f:
            json.dump(results, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
