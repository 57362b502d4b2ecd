"""CUDA tagged p2p through the pull kernel, checked against torch copies.

Runs at any world size: every rank sends to (rank+1) % world and receives
from (rank-1) % world, so at world 1 every message is a self-send (launched
on the caller's stream), with ranks sharing one GPU the host-gated path runs,
and with one GPU per rank the device-flag path runs."""
import os
import zlib

from common import Checker, init, torch, dist

rank, world, dev = init(timeout_s=90)
c = Checker(rank)
peer, src = (rank + 1) % world, (rank - 1) % world
g = torch.Generator(device="cpu").manual_seed(0)


def data(shape, dtype, r):
    # crc32, not hash(): string hashing is randomised per process
    gg = torch.Generator().manual_seed(zlib.crc32(repr((shape, str(dtype), r)).encode()))
    if dtype.is_floating_point:
        return torch.randn(shape, generator=gg).to(dtype)
    return torch.randint(-100, 100, shape, generator=gg).to(dtype)


cases = [
    ("contig f32", (1000,), torch.float32, lambda t: t, lambda t: t),
    ("contig big bf16", (3, 1 << 20), torch.bfloat16, lambda t: t, lambda t: t),
    ("odd bytes u8", (1001,), torch.uint8, lambda t: t, lambda t: t),
    ("strided send", (64, 48), torch.float64, lambda t: t[:, 5:40:3], lambda t: t),
    ("strided recv", (40, 30), torch.float32, lambda t: t, lambda t: t[3:, ::2]),
    ("faces x", (20, 20, 20), torch.float64, lambda t: t[2:18, 2:18, 2:4], lambda t: t[2:18, 2:18, 18:20]),
    ("transpose", (33, 17), torch.float16, lambda t: t.t(), lambda t: t),
    ("6-dim", (2, 3, 2, 3, 2, 5), torch.float32, lambda t: t.permute(5, 4, 3, 2, 1, 0), lambda t: t),
    ("zero size", (0, 4), torch.float32, lambda t: t, lambda t: t),
    ("int64", (257,), torch.int64, lambda t: t, lambda t: t),
]
reqs, checks = [], []
for i, (name, shape, dtype, sview, rview) in enumerate(cases):
    s_full = data(shape, dtype, rank).to(dev)
    sv = sview(s_full)
    want_full = data(shape, dtype, src)
    want = sview(want_full).contiguous()
    # receive layout: rview applied to a buffer big enough; shapes must match the message
    rbuf = torch.zeros(shape, dtype=dtype, device=dev)
    rv = rview(rbuf)
    if rv.shape != want.shape:
        rbuf = torch.zeros(want.shape, dtype=dtype, device=dev)
        rv = rbuf
    reqs.append(dist.irecv(rv, src, tag=50 + i))
    reqs.append(dist.isend(sv, peer, tag=50 + i))
    checks.append((name, rv, want))
for w in reqs:
    w.wait()
torch.cuda.synchronize()
for name, rv, want in checks:
    c.equal(name, rv.cpu(), want)
# a layout with a 2 GiB stride (the kernel's 64-bit walk): rows of a 4 GiB field
big = torch.zeros((2, 1 << 28), dtype=torch.float64, device=dev)
big[:, 3:1003] = torch.arange(2000, dtype=torch.float64, device=dev).view(2, 1000) + 10000 * rank
wide_out = torch.zeros((2, 1000), dtype=torch.float64, device=dev)
rr = dist.irecv(wide_out, src, tag=40)
ss = dist.isend(big[:, 3:1003], peer, tag=40)
rr.wait()
ss.wait()
torch.cuda.synchronize()
c.equal("wide stride", wide_out.cpu(), torch.arange(2000, dtype=torch.float64).view(2, 1000) + 10000 * src)
del big
torch.cuda.empty_cache()
# repeated exchange into the same buffers (IPC caches, slot reuse)
x = torch.arange(4096, dtype=torch.float32, device=dev)
y = torch.zeros_like(x)
for it in range(50):
    x.fill_(rank * 1000 + it)
    rr = dist.irecv(y, src, tag=7)
    ss = dist.isend(x, peer, tag=7)
    rr.wait()
    ss.wait()
    if it % 10 == 9:
        c.equal(f"repeat {it}", y.cpu(), torch.full((4096,), float(src * 1000 + it)))
# coalesced window of 26 messages
ops, outs = [], []
for k in range(26):
    o = torch.zeros(100 + k, device=dev)
    outs.append(o)
    ops.append(dist.P2POp(dist.irecv, o, src, tag=1000 + k))
for k in range(26):
    ops.append(dist.P2POp(dist.isend, torch.full((100 + k,), float(src * 0 + rank * 10 + k), device=dev),
                          peer, tag=1000 + k))
for w in dist.batch_isend_irecv(ops):
    w.wait()
for k in range(26):
    c.equal(f"window {k}", outs[k].cpu(), torch.full((100 + k,), float(src * 10 + k)))
import commux_b200  # noqa: E402

st = commux_b200.stats(device=dev)
if os.environ.get("CMX_EXPECT_EXPORT_STAGING") == "1" and world > 1:
    # memory CUDA IPC cannot export (expandable segments) went through the pool
    c.check("export staging used", st.get("cuda_export_staged", 0) > 0, str(st))
if rank == 0:
    print({k: v for k, v in st.items() if k.startswith("cuda")}, flush=True)
c.finish()
