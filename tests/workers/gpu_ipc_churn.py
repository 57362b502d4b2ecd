"""Receivers keep a bounded number of CUDA-IPC mappings while senders free
and reallocate their buffers. This is the device counterpart of the
reference's regression test on host send addresses
(reference: tests/test_host_coll_addresses.py:18-56), which bounds the number
of distinct addresses over 100 all_reduces.

Every rank sends to (rank+1) % world and receives from (rank-1) % world, for
40 rounds. Each round the sender allocates a fresh 48 MiB tensor, which gets
its own cudaMalloc segment, sends it and waits. It then drops the tensor and
empties the allocator cache, so the segment is freed before the next round.
The data must arrive intact in every round. A receiver closes a mapping once
the sender's address range is reused, so its open mappings
(cuda_ipc_opens - cuda_ipc_closes) stay within the number of distinct
ranges the sender used, plus the mailbox."""
import zlib

from common import Checker, init, torch, dist

import commux_b200 as commux

rank, world, dev = init(timeout_s=120)
c = Checker(rank)
peer, src = (rank + 1) % world, (rank - 1) % world
n = 12 << 20  # fp32 elements: 48 MiB
rounds = 40
ptrs = set()
commux.reset_stats(device=dev)
for r in range(rounds):
    g = torch.Generator().manual_seed(zlib.crc32(repr((rank, r)).encode()))
    head = torch.randint(-1000, 1000, (1024,), generator=g).to(torch.float32)
    t = torch.full((n,), float(r + 1), device=dev)
    t[:1024] = head.to(dev)
    ptrs.add(t.data_ptr())
    out = torch.empty(n, device=dev)
    rq = dist.irecv(out, src=src, tag=r)
    sq = dist.isend(t, dst=peer, tag=r)
    sq.wait()
    rq.wait()
    torch.cuda.current_stream().synchronize()
    gs = torch.Generator().manual_seed(zlib.crc32(repr((src, r)).encode()))
    want_head = torch.randint(-1000, 1000, (1024,), generator=gs).to(torch.float32)
    c.equal(f"round {r} head", out[:1024], want_head)
    c.check(f"round {r} body", bool((out[1024:] == float(r + 1)).all().item()))
    del t, out, sq, rq
    torch.cuda.empty_cache()

# the sender's distinct ranges, as seen by its receiver
mine = torch.tensor([float(len(ptrs))])
theirs = torch.zeros(1)
lst = [torch.zeros(1) for _ in range(world)]
dist.all_gather(lst, mine)
theirs = int(lst[src].item())
s = commux.stats(device=dev)
opens, closes = int(s.get("cuda_ipc_opens", 0)), int(s.get("cuda_ipc_closes", 0))
live = opens - closes
if world > 1:
    c.check("live mappings bounded", live <= theirs + 1,
            f"opens {opens} closes {closes} live {live}, sender used {theirs} ranges")
print(f"rank {rank}: sender ranges {theirs}, ipc opens {opens}, closes {closes}", flush=True)
c.finish()
