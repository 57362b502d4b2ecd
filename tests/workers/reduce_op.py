"""Unsupported ReduceOps raise "unsupported ReduceOp" on every rank before any
message; AVG is supported on floating dtypes (reference: tests/test_reduce_op.py)."""
from common import Checker, init, torch, dist

rank, world, dev = init()
c = Checker(rank)


def expect_rejected(name, call):
    try:
        call()
    except (RuntimeError, ValueError) as e:
        if "unsupported ReduceOp" not in str(e):
            c.check(name, False, f"raised another error: {e}")
        return
    c.check(name, False, "returned without an error")


for op in (dist.ReduceOp.BAND, dist.ReduceOp.BXOR):
    for root in range(world):
        t = torch.ones(5, dtype=torch.float64, device=dev)
        expect_rejected(f"reduce {op} root={root}", lambda: dist.reduce(t, dst=root, op=op))
    t = torch.ones(5, dtype=torch.float64, device=dev)
    expect_rejected(f"all_reduce {op}", lambda: dist.all_reduce(t, op=op))
ti = torch.ones(5, dtype=torch.int64, device=dev)
expect_rejected("all_reduce AVG int64", lambda: dist.all_reduce(ti, op=dist.ReduceOp.AVG))
t = torch.full((5,), float(rank + 1), dtype=torch.float64, device=dev)
dist.all_reduce(t, op=dist.ReduceOp.AVG)
c.equal("AVG accepted", t, torch.full((5,), (world + 1) / 2.0, dtype=torch.float64))
t = torch.full((5,), float(rank + 1), dtype=torch.float64, device=dev)
dist.all_reduce(t)
c.equal("SUM after rejections", t, torch.full((5,), world * (world + 1) / 2.0, dtype=torch.float64))
c.finish()
