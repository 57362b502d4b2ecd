"""Randomised tagged p2p: every rank knows the whole seeded schedule (who
sends what to whom, under which tag), posts its receives and sends in a
shuffled order, mixing single and vector posts, then checks every byte.
Sizes run from empty through eager (<= 64 KiB) and rendezvous messages up to
3 MiB, where same-host reads are split across the copy helpers. Several
messages share a (source, tag) pair to check MPI non-overtaking order."""
import random
import zlib

from common import Checker, init, torch, dist

rank, world, dev = init(timeout_s=120)
c = Checker(rank)
ROUNDS = 3
SIZES = [0, 1, 7, 64, 1000, 4096, 16384, 65536, 65537, 300000, 1 << 20, 3 << 20]


def payload(src, dst, tag, seq, n):
    # a value pattern unique to the message (exact in fp32 below 2^24)
    base = float(zlib.crc32(repr((src, dst, tag, seq)).encode()) % 4096)
    return (torch.arange(n, dtype=torch.float32) % 4093) + base


for rnd in range(ROUNDS):
    rng = random.Random(1234 + rnd)
    msgs = []  # (src, dst, tag, seq, elements)
    per_pair_tag = {}
    for _ in range(40 * world):
        src, dst = rng.randrange(world), rng.randrange(world)
        tag = rng.randrange(5)  # few tags: many messages share (src, tag)
        key = (src, dst, tag)
        seq = per_pair_tag.get(key, 0)
        per_pair_tag[key] = seq + 1
        msgs.append((src, dst, tag, seq, rng.choice(SIZES) // 4))
    local = random.Random(rank * 7919 + rnd)
    sends = [m for m in msgs if m[0] == rank]
    recvs = [m for m in msgs if m[1] == rank]
    # post in shuffled order, but keep each (peer, tag) stream in sequence:
    # MPI matches messages of one (source, tag) in posting order
    order = [("r", m) for m in recvs] + [("s", m) for m in sends]
    local.shuffle(order)
    streams = {}
    for kind, m in order:
        streams.setdefault((kind, m[0], m[1], m[2]), []).append(m)
    for k in streams:
        streams[k].sort(key=lambda m: m[3])
    cursor = {k: 0 for k in streams}
    works, checks = [], []
    for kind, m in order:
        k = (kind, m[0], m[1], m[2])
        m = streams[k][cursor[k]]
        cursor[k] += 1
        src, dst, tag, seq, n = m
        if kind == "s":
            t = payload(src, dst, tag, seq, n).to(dev)
            works.append(dist.isend(t, dst, tag=tag))
            checks.append(None)
        else:
            t = torch.full((n,), -1.0, device=dev)
            works.append(dist.irecv(t, src, tag=tag))
            checks.append((m, t))
    for w in works:
        w.wait()
    if dev.type == "cuda":
        torch.cuda.synchronize()
    bad = 0
    for item in checks:
        if item is None:
            continue
        (src, dst, tag, seq, n), t = item
        if not torch.equal(t.cpu(), payload(src, dst, tag, seq, n)):
            bad += 1
            if bad <= 3:
                c.check(f"round {rnd} msg {src}->{dst} tag {tag} seq {seq} ({n} floats)", False)
    c.check(f"round {rnd}: {len(recvs)} receives intact", bad == 0, f"{bad} corrupted")
c.finish()
