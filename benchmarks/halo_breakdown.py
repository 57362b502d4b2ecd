#!/usr/bin/env python
"""One-GPU halo exchange by direction class (x-, y-, z-faces, edges,
corners, all 26), each as its own persistent plan, device-timed with CUDA
events: once back to back ("alone") and once right after a 7-point Jacobi
sweep ("after_sweep": the L2 then holds the sweep's dirty lines, as in a
real timestep). A plan of the eight 64-byte corners measures the fixed
cost of one exchange. 512^3 fp64 interior, halo 2, periodic (every message
is a copy within the GPU). Prints one JSON line.

    python benchmarks/halo_breakdown.py
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
    from commux_b200.parallel.halo import DIRECTIONS, HaloExchange
    from commux_b200.utils import free_port

    torch.cuda.set_device(0)
    commux.register()
    dist.init_process_group("ucx", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=120))
    m = Jacobi3D(512, halo=2, dims=(1, 1, 1), seed=0)
    nonzero = lambda d: sum(1 for o in d if o)  # noqa: E731
    classes = {
        "x_faces": [d for d in DIRECTIONS if nonzero(d) == 1 and d[2] != 0],
        "y_faces": [d for d in DIRECTIONS if nonzero(d) == 1 and d[1] != 0],
        "z_faces": [d for d in DIRECTIONS if nonzero(d) == 1 and d[0] != 0],
        "edges": [d for d in DIRECTIONS if nonzero(d) == 2],
        "corners": [d for d in DIRECTIONS if nonzero(d) == 3],
        "all": list(DIRECTIONS),
    }

    def span(fn):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3

    out = {}
    for name, dirs in classes.items():
        ex = HaloExchange(m.interior, 2, m.grid, directions=dirs)
        for _ in range(5):
            ex.exchange(m.u)
        torch.cuda.synchronize()
        alone = [span(lambda: ex.exchange(m.u)) for _ in range(30)]
        after = []
        for _ in range(10):
            m.update()
            after.append(span(lambda: ex.exchange(m.u)))
        out[name] = {"bytes": ex.message_bytes(8), "alone_us_p50": round(statistics.median(alone), 2),
                     "after_sweep_us_p50": round(statistics.median(after), 2)}
    out["env"] = {k: os.environ.get(k) for k in ("COMMUX_P2P_CTAS", "COMMUX_PLAN_INTERLEAVE")}
    print(json.dumps(out), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
