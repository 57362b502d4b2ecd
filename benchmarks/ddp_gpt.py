#!/usr/bin/env python
"""DDP training throughput of a 12-layer GPT over the commux backend.

Config: decoder-only transformer, d_model 768, 12 heads, FFN 3072, vocab
32000, seq 1024, micro-batch 8 per GPU, bf16 autocast (fp32 master weights),
random init (seeded), synthetic uniform token ids; DDP with 25 MB gradient
buckets, all-reduced by the backend on its collective stream while backward
runs. ``--backend nccl`` runs the same step on NCCL (the comparator: the
reference backend cannot run DDP at all -- no allgather, no getFuture).

    torchrun --nproc-per-node N benchmarks/ddp_gpt.py --backend ucx
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
    ap.add_argument("--backend", default="ucx", choices=["ucx", "nccl", "gloo"])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--bucket-mb", type=float, default=25.0)
    ap.add_argument("--layers", type=int, default=12)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel as DDP

    import commux_b200 as commux
    from commux_b200.models.gpt import GPT, GPTConfig
    from commux_b200.utils import env_rank, free_port, rank_max

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    commux.register()
    if "MASTER_ADDR" not in os.environ:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group(args.backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=600))
    torch.manual_seed(0)
    cfg = GPTConfig(n_layer=args.layers)
    model = GPT(cfg).cuda()
    ddp = DDP(model, device_ids=[local], bucket_cap_mb=args.bucket_mb, gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, fused=True)
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    B, T = args.micro_batch, cfg.seq_len
    x = torch.randint(0, cfg.vocab, (B, T), device="cuda", generator=g)
    y = torch.randint(0, cfg.vocab, (B, T), device="cuda", generator=g)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = ddp(x, y)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        loss = step()
    t1.record()
    torch.cuda.synchronize()
    ms = rank_max([t0.elapsed_time(t1) / args.steps])[0] if args.backend != "nccl" else None
    if ms is None:
        t = torch.tensor([t0.elapsed_time(t1) / args.steps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    if rank == 0:
        toks = world * B * T / (ms * 1e-3)
        print(json.dumps({"metric": "DDP GPT-12L tokens/s", "backend": args.backend, "n_gpus": world,
                          "value": round(toks, 1), "ms_per_step": round(ms, 3), "loss": float(loss),
                          "params_M": round(sum(p.numel() for p in model.parameters()) / 1e6, 2),
                          "micro_batch": B, "seq_len": T, "bucket_mb": args.bucket_mb}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
