"""CUDA all_reduce / reduce / broadcast numerics across dtypes, ReduceOps and
sizes. The sizes cover every device algorithm: one-shot (small), two-shot
(large), and NVLS multimem (large f32/f16/bf16 sums, averages and f16/bf16
min/max, when every rank has its own GPU on an NVSwitch). Each result is
checked against an fp64 fold of every rank's input (the inputs are seeded by
rank, so every rank can rebuild all of them), and the ranks must agree bit for
bit."""
import os

from common import Checker, init, torch, dist

import commux_b200

rank, world, dev = init(timeout_s=180)
c = Checker(rank)
Op = dist.ReduceOp
sizes = [int(x) for x in os.environ.get("CMX_SIZES", "7,1000,70001,1048576,3145733").split(",")]
dtypes = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
tol = {torch.float32: 2e-5, torch.bfloat16: 2e-2, torch.float16: 2e-3}


def inputs(r, n, dtype, op):
    g = torch.Generator().manual_seed(1000 * r + n % 997)
    x = torch.randn(n, generator=g, dtype=torch.float64)
    if op == Op.PRODUCT:
        x = 1.0 + 0.01 * x
    return x.to(dtype)


def fold(n, dtype, op):
    xs = [inputs(r, n, dtype, op).double() for r in range(world)]
    acc = xs[0].clone()
    for x in xs[1:]:
        if op in (Op.SUM, Op.AVG):
            acc += x
        elif op == Op.PRODUCT:
            acc *= x
        elif op == Op.MIN:
            acc = torch.minimum(acc, x)
        else:
            acc = torch.maximum(acc, x)
    if op == Op.AVG:
        acc /= world
    return acc


def same_on_all_ranks(name, t):
    bits = t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32).to(torch.int64).cpu()
    h = torch.tensor([int((bits * torch.arange(1, bits.numel() + 1)).sum()) & ((1 << 52) - 1)], dtype=torch.float64)
    lo, hi = h.clone(), h.clone()
    dist.all_reduce(lo, op=Op.MIN)
    dist.all_reduce(hi, op=Op.MAX)
    c.check(name + " identical on every rank", float(lo) == float(hi))


for dname, dtype in dtypes.items():
    for op in (Op.SUM, Op.AVG, Op.MAX, Op.MIN, Op.PRODUCT):
        for n in sizes:
            name = f"all_reduce {dname} {op} n={n}"
            t = inputs(rank, n, dtype, op).to(dev)
            dist.all_reduce(t, op=op)
            want = fold(n, dtype, op)
            got = t.double().cpu()
            if op in (Op.MAX, Op.MIN):
                ok = torch.equal(got, want.to(dtype).double())
            else:
                scale = want.abs() + (world if op != Op.PRODUCT else 1.0)
                ok = bool(((got - want).abs() <= tol[dtype] * scale).all())
            c.check(name, ok, f"max err {float((got - want).abs().max())}")
            same_on_all_ranks(name, t)
    n = 1 << 20
    for root in range(world):
        t = inputs(rank, n, dtype, Op.SUM).to(dev)
        dist.reduce(t, dst=root)
        if rank == root:
            want = fold(n, dtype, Op.SUM)
            c.check(f"reduce {dname} root={root}",
                    bool(((t.double().cpu() - want).abs() <= tol[dtype] * (want.abs() + world)).all()))
        t = inputs(rank, n, dtype, Op.SUM).to(dev)
        dist.broadcast(t, src=root)
        c.equal(f"broadcast {dname} root={root}", t.cpu(), inputs(root, n, dtype, Op.SUM))
if rank == 0:
    st = commux_b200.stats()
    print({k: v for k, v in st.items() if k.startswith("cuda.coll") or k.startswith("coll")}, flush=True)
c.finish()
