#!/usr/bin/env python
"""Flagship benchmark: tagged 26-direction halo exchange of a 3-D stencil.

Workload: a global periodic 1024^3 fp64 field ~U(-1,1) (seeded), split over a near-cubic grid of
ranks (2x2x2 at 8 GPUs -> 512^3 per rank; 512^3 per GPU at every N, i.e.
weak scaling), halo width 2. One step = the 26-neighbour halo exchange
(tag = 1000 + direction, posted out of order as one isend/irecv batch through
torch.distributed with backend "ucx") followed by one 7-point Jacobi sweep.

Reported ``value``: halo-exchange GB/s of the whole job = bytes all ranks
send per step x steps / (max over ranks of the summed device time of the
exchange phase), timed with CUDA events on the compute stream. The fields
(1.1 GB each) exceed the 126 MB L2, so no flush is needed between steps.
``e2e`` repeats the steps through the same public API with, every step, a
host->device copy of a per-rank forcing plane from pinned memory and a
device->host read of the step's residual, timed by the host clock.

    python bench.py [--gpus N --steps K --warmup W]            # N=1
    torchrun --nproc-per-node N bench.py --gpus N ...          # N>1
    python bench.py --impl reference                           # reference arm
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

# every N runs 512^3 fp64 per GPU (weak scaling); the global size, which is
# 512^3 times the process grid (1024^3 at 8 GPUs), is in config.model
METRIC = "tagged halo-exchange GB/s (26-direction, halo 2, fp64, 512^3 per GPU, 7-point Jacobi)"
BASELINE_VALUE = None  # the reference publishes no halo-exchange GB/s number


NVLINK_GBS = 770.0  # measured peer copy per direction on this B200 model (GB/s)


def measured_hbm_gbs() -> tuple[float, str]:
    """HBM copy rate for the roofline: MEASURED_PEAKS.json beside this file
    when present, else an earlier measurement of the same B200 model."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            v = float(json.load(f)["hbm_gbs"])
        if v > 0:
            return v, "of measured"
    except (OSError, ValueError, KeyError, TypeError):
        pass
    return 6650.0, "of fallback"


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["commux", "reference"], default="commux")
    ap.add_argument("--global-n", type=int, default=1024)
    ap.add_argument("--halo", type=int, default=2)
    ap.add_argument("--dtype", choices=["fp64", "fp32"], default="fp64")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--clocks-raw", default=None, help="save the raw nvidia-smi samples here")
    ap.add_argument("--per-gpu-n", type=int, default=512,
                    help="interior points per GPU and axis (weak scaling); the global size is "
                         "per-gpu-n times the process grid")
    return ap.parse_args()


def reference_arm(args) -> None:
    """Run the unmodified reference through its own API, if it is installed."""
    ref = os.path.join(HERE, "baseline", "_ref")
    reason = None
    if not os.path.isdir(os.path.join(ref, "commux")):
        reason = ("reference not installable offline: its build needs setuptools_scm (absent from "
                  "the offline wheelhouse) and downloads UCX 1.18 + gdrcopy sources "
                  "(cmake/BuildUCX.cmake); no UCX exists on this image")
    else:
        try:
            sys.path.insert(0, ref)
            import commux as refmod  # noqa: F401
            reason = "reference package present but its UCX halo run is not wired (no UCX)"
        except Exception as e:  # pragma: no cover
            reason = f"reference import failed: {e}"
    print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    # one batched copy kernel per exchange (coalescing window of batch_isend_irecv)
    os.environ.setdefault("COMMUX_GROUP", "1")

    import torch
    import torch.distributed as dist

    import commux_b200 as commux
    from commux_b200 import ops
    from commux_b200.models.halo3d import Jacobi3D
    from commux_b200.parallel.halo import factor3
    from commux_b200.utils import env_rank, free_port, rank_max, rank_sum
    from commux_b200.utils.clocks import ClockSampler, gpu_uuid

    rank, world, local_rank = env_rank()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local_rank)
    commux.register()
    if "MASTER_ADDR" not in os.environ:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group("ucx", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=600))
    dims = factor3(world)
    gn = tuple(args.per_gpu_n * d for d in dims)
    dtype = torch.float64 if args.dtype == "fp64" else torch.float32
    model = Jacobi3D(gn, halo=args.halo, dims=dims, dtype=dtype, seed=0)
    bytes_rank = model.halo_bytes
    bytes_job = int(rank_sum([bytes_rank])[0])
    remote_rank = int(rank_max([model.halo.remote_bytes(model.u.element_size(), rank)])[0])

    def cuda_launches():
        s = commux.stats(device="cpu")
        return int(s.get("cuda_kernel_launches", 0)) + ops.launches()

    for _ in range(args.warmup):
        model.step()
    torch.cuda.synchronize()
    dist.barrier()

    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    uuid = gpu_uuid(local_rank)
    sampler = ClockSampler([uuid] if uuid else [], raw_path=args.clocks_raw).start()
    launches0 = cuda_launches()
    torch.cuda.synchronize()
    dist.barrier()
    for k in range(K):
        ev[k][0].record()
        model.exchange()
        ev[k][1].record()
        model.update()
        ev[k][2].record()
    torch.cuda.synchronize()
    dist.barrier()
    launches = cuda_launches() - launches0
    clocks = sampler.stop()
    # which transport path the timed exchanges took, summed over ranks, and
    # how many distinct GPUs the ranks drove
    st = commux.stats(device="cpu")
    path_keys = ("cuda_plan_device_msgs", "cuda_plan_shared_msgs", "cuda_plan_starts", "cuda_pulls_peer_gpu")
    path_sums = rank_sum([float(st.get(k, 0)) for k in path_keys])
    uuids = [None] * world
    dist.all_gather_object(uuids, uuid or f"rank{rank}")
    paths = {k: int(v) for k, v in zip(path_keys, path_sums)}
    paths["gpus_active"] = len(set(uuids))

    # the same steps with the exchange overlapped with the core update (side
    # stream) and the boundary layer after it: whole steps, device-timed
    for _ in range(2):
        model.step_overlapped()
    oev = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    torch.cuda.synchronize()
    dist.barrier()
    oev[0].record()
    for k in range(K):
        model.step_overlapped()
        oev[k + 1].record()
    torch.cuda.synchronize()
    dist.barrier()
    ostep_max = rank_max([oev[k].elapsed_time(oev[k + 1]) for k in range(K)])
    otot_max = rank_max([oev[0].elapsed_time(oev[K])])[0]

    # diagnostic: the same exchange back to back, no stencil in between (the
    # in-step exchange also absorbs the ranks' skew after each update)
    xev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(K)]
    torch.cuda.synchronize()
    dist.barrier()
    for k in range(K):
        xev[k][0].record()
        model.exchange()
        xev[k][1].record()
    torch.cuda.synchronize()
    xonly = rank_max([xev[k][0].elapsed_time(xev[k][1]) for k in range(K)])

    exch = [ev[k][0].elapsed_time(ev[k][1]) for k in range(K)]
    step = [ev[k][0].elapsed_time(ev[k][2]) for k in range(K)]
    total = ev[0][0].elapsed_time(ev[K - 1][2])
    exch_max = rank_max(exch)          # per-step max over ranks
    step_max = rank_max(step)
    tot_max, exch_sum_max = rank_max([total, sum(exch)])
    job_launches = int(rank_sum([launches])[0])

    # end to end through the public API: H2D input + exchange + D2H result
    Ke = args.e2e_steps or K
    forcing_h = torch.randn(model.interior[1], model.interior[2], dtype=dtype).pin_memory()
    forcing_d = torch.empty_like(forcing_h, device=model.device)
    res_h = torch.empty(1, dtype=torch.float64).pin_memory()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_wall = 0.0
    host_post = host_wait = 0.0
    for k in range(-2, Ke):  # two untimed warm-up steps (pinned copies, first launches)
        if k == 0:
            e2e_wall = host_post = host_wait = 0.0
        torch.cuda.current_stream().synchronize()  # previous update finished (not timed)
        t0 = time.perf_counter()
        forcing_d.copy_(forcing_h, non_blocking=True)
        model.inject(forcing_d)
        ta = time.perf_counter()
        works = model.halo.start(model.u)
        tb = time.perf_counter()
        for w in works:
            w.wait()
        tc = time.perf_counter()
        res_h.copy_(model.residual, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        _ = float(res_h[0])
        e2e_wall += time.perf_counter() - t0
        host_post += tb - ta
        host_wait += tc - tb
        model.update()
    torch.cuda.synchronize()
    e2e_wall_max = rank_max([e2e_wall])[0]

    value = bytes_job * K / (exch_sum_max * 1e-3) / 1e9
    # roofline of one exchange: the bytes that cross NVLink into the busiest
    # rank at the measured peer-copy rate, or every byte read and written
    # once in this GPU's HBM at the measured copy rate, whichever is slower
    hbm_gbs, hbm_src = measured_hbm_gbs()
    floor_us = max(remote_rank / NVLINK_GBS / 1e3, 2 * bytes_rank / hbm_gbs / 1e3)
    exch_p50_us = statistics.median(exch_max) * 1e3
    e2e_value = bytes_job * Ke / e2e_wall_max / 1e9
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(tot_max / K, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
            "dtype": args.dtype,
            "data": "synthetic: seeded U(-1,1) field, random-init; no dataset",
            "config": {
                "model": f"3-D 7-point Jacobi, {gn[0]}x{gn[1]}x{gn[2]} global, {model.interior[0]}^3 per GPU, "
                         f"halo {args.halo}, 26 neighbours, tags 1000+dir",
                "global_batch": 1,
                "seq_len": 0,
                "parallelism": f"domain decomposition {dims[0]}x{dims[1]}x{dims[2]} (periodic)",
                "halo_bytes_per_step_per_rank": bytes_rank,
                "nvlink_bytes_per_step_per_rank_max": remote_rank,
                "paths": paths,
                "exchange_only_us_p50": round(statistics.median(xonly) * 1e3, 2),
                "halo_bytes_per_step_job": bytes_job,
                "exchange_us_p50": round(exch_p50_us, 2),
                "roofline": {"nvlink_bytes_per_step_max_rank": remote_rank,
                             "floor_us": round(floor_us, 2),
                             "frac_of_roofline": round(floor_us / exch_p50_us, 3),
                             "basis": f"max(NVLink bytes / {NVLINK_GBS:.0f} GB/s measured peer copy, "
                                      f"2 x halo bytes / {hbm_gbs:.0f} GB/s HBM copy ({hbm_src})) "
                                      "against exchange_us_p50"},
                "exchange_us_min": round(min(exch_max) * 1e3, 2),
                "step_ms_p50": round(statistics.median(step_max), 4),
                "overlapped": {"step_ms_p50": round(statistics.median(ostep_max), 4),
                               "ms_per_step": round(otot_max / K, 4),
                               "jacobi_gcells_per_s_job": round(
                                   world * model.interior[0] * model.interior[1] * model.interior[2] * K
                                   / (otot_max * 1e-3) / 1e9, 3),
                               "how": "exchange on a high-priority side stream while the core cells "
                                      "(stencil reads no ghost) update, then the one-cell boundary layer; "
                                      "same field as the sequential step"},
                "jacobi_gcells_per_s_job": round(
                    world * model.interior[0] * model.interior[1] * model.interior[2] * K / (tot_max * 1e-3) / 1e9, 3),
                "value_basis": "bytes sent by all ranks / max-over-ranks sum of exchange-phase device time",
                "l2": "fields 1.1 GB each > 126 MB L2; no flush needed",
                "backend": "ucx (commux_b200)",
                "group_window": os.environ.get("COMMUX_GROUP"),
                "plan_order": os.environ.get("COMMUX_PLAN_ORDER", "plan"),
            },
            "e2e": {"value": round(e2e_value, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": forcing_h.numel() * forcing_h.element_size() * world,
                    "d2h_bytes_per_step": 8 * world,
                    "basis": "host wall clock per step around H2D forcing + exchange + D2H residual "
                             "(max over ranks), commux.batch_p2p public API",
                    "host_post_us": round(host_post / Ke * 1e6, 1),
                    "host_wait_us": round(host_wait / Ke * 1e6, 1)},
            "gpu_launches": job_launches,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
