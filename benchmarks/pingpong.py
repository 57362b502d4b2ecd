#!/usr/bin/env python
"""V-tensor ping-pong between two ranks (round-trip latency).

Rank 0 sends V tensors to rank 1 and receives V back; rank 1 mirrors. Each
iteration completes on the device before the next starts (stream synchronised
at the end of every round trip), so the host-timed round trip is comparable
to the reference's ping-pong numbers (reference: tests/test_commux.cpp:204-242,
published V=2/16 at 8 KiB per tensor in src/process_group_ucx.cpp:139-141).

Modes: ``pertensor`` (one message per tensor), ``coalesced`` (one message for
the V tensors; needs COMMUX_COALESCE=1 in the environment, which changes the
wire format on every rank), ``window`` (torch's batch_isend_irecv, i.e. the
backend's coalescing window; set COMMUX_GROUP=1 to defer the posts to its end),
``plan`` (a persistent plan started every iteration), ``batch`` (one
batch_p2p per direction).

    torchrun --nproc-per-node 2 benchmarks/pingpong.py --device cuda --mode plan
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
    ap.add_argument("--device", default="cuda", choices=["cuda", "cpu"])
    ap.add_argument("--mode", default="pertensor", choices=["pertensor", "coalesced", "window", "plan", "batch"])
    ap.add_argument("--V", default="1,8,64,512")
    ap.add_argument("--sizes", default="4096,65536,1048576,4194304")
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--max-total-bytes", type=int, default=2 << 30)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    import commux_b200 as commux
    from commux_b200.utils import env_rank, free_port

    rank, world, local = env_rank()
    assert world >= 2, "ping-pong needs two ranks"
    if args.device == "cuda":
        torch.cuda.set_device(local % torch.cuda.device_count())
    dev = torch.device(args.device, local % torch.cuda.device_count()) if args.device == "cuda" else torch.device("cpu")
    commux.register()
    if "MASTER_ADDR" not in os.environ:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group("ucx", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    pg = dist.distributed_c10d._get_default_group()
    sync = (lambda: torch.cuda.current_stream().synchronize()) if args.device == "cuda" else (lambda: None)
    for V in map(int, args.V.split(",")):
        for nbytes in map(int, args.sizes.split(",")):
            if V * nbytes > args.max_total_bytes:
                continue
            n = nbytes // 4
            sv = [torch.full((n,), float(k), device=dev) for k in range(V)]
            rv = [torch.zeros(n, device=dev) for _ in range(V)]
            peer = 1 - rank if rank < 2 else None
            if peer is None:
                dist.barrier()
                continue
            plans = None
            if args.mode == "plan":
                out = [(t, peer, 900 + k) for k, t in enumerate(sv)]
                inn = [(t, peer, 900 + k) for k, t in enumerate(rv)]
                # a ping-pong is two one-way plans started alternately
                ping = commux.p2p_plan(sends=out if rank == 0 else [], recvs=inn if rank == 1 else [])
                pong = commux.p2p_plan(sends=out if rank == 1 else [], recvs=inn if rank == 0 else [])
                plans = (ping, pong)

            def rt():
                if args.mode == "plan":
                    plans[0].start()
                    plans[1].start()
                elif args.mode == "window":
                    other = 1 - rank
                    if rank == 0:
                        ws = dist.batch_isend_irecv([dist.P2POp(dist.isend, t, other, tag=900 + k)
                                                     for k, t in enumerate(sv)])
                        for w in ws:
                            w.wait()
                        ws = dist.batch_isend_irecv([dist.P2POp(dist.irecv, t, other, tag=1900 + k)
                                                     for k, t in enumerate(rv)])
                    else:
                        ws = dist.batch_isend_irecv([dist.P2POp(dist.irecv, t, other, tag=900 + k)
                                                     for k, t in enumerate(rv)])
                        for w in ws:
                            w.wait()
                        ws = dist.batch_isend_irecv([dist.P2POp(dist.isend, t, other, tag=1900 + k)
                                                     for k, t in enumerate(sv)])
                    for w in ws:
                        w.wait()
                elif args.mode == "batch":
                    if rank == 0:
                        commux.batch_p2p(sends=[(t, 1, 900 + k) for k, t in enumerate(sv)]).wait()
                        commux.batch_p2p(recvs=[(t, 1, 901 + k) for k, t in enumerate(rv)]).wait()
                    else:
                        commux.batch_p2p(recvs=[(t, 0, 900 + k) for k, t in enumerate(rv)]).wait()
                        commux.batch_p2p(sends=[(t, 0, 901 + k) for k, t in enumerate(sv)]).wait()
                else:
                    if rank == 0:
                        pg.send(sv, 1, 900).wait()
                        pg.recv(rv, 1, 901).wait()
                    else:
                        pg.recv(rv, 0, 900).wait()
                        pg.send(sv, 0, 901).wait()
                sync()

            for _ in range(args.warmup):
                rt()
            dist.barrier()
            lat = []
            for _ in range(args.iters):
                t0 = time.perf_counter()
                rt()
                lat.append((time.perf_counter() - t0) * 1e6)
            if rank == 0:
                print(json.dumps({"mode": args.mode, "device": args.device, "V": V, "bytes_per_tensor": nbytes,
                                  "roundtrip_us_p50": round(statistics.median(lat), 2),
                                  "roundtrip_us_min": round(min(lat), 2),
                                  "coalesce": os.environ.get("COMMUX_COALESCE", "0"),
                                  "group": os.environ.get("COMMUX_GROUP", "0")}), flush=True)
            dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
