"""Device barrier (every rank on its own GPU).

order:   each rank delays its stream (a sleep kernel, longer on higher
         ranks), then fills its own buffer with 100 + rank, then calls
         dist.barrier(). After the barrier every rank reads every peer's
         buffer through a CUDA-IPC mapping on its own stream and must see the
         filled values: the barrier returns only once every rank's stream has
         run everything enqueued before it. (A host-only barrier returns as
         soon as the peers' hosts arrive, long before their fills run.)
timeout: rank 0 calls the barrier alone with a short device timeout; its
         wait runs out, the kernel records the timeout and returns, and the
         call raises. Rank 1 never launches the barrier; it waits on the host
         until rank 0 reports, so no kernel is in flight when either exits.
"""
import ctypes
import os
import time

from common import Checker, init, torch, dist

import commux_b200 as commux

rank, world, dev = init(timeout_s=120)
c = Checker(rank)
mode = os.environ.get("CMX_BARRIER_MODE", "order")
store = dist.distributed_c10d._get_default_store()

# the device collectives are set up by the first CUDA collective (collective)
t = torch.ones(4, device=dev)
dist.all_reduce(t)
c.check("set-up all_reduce", float(t[0]) == world)

class IpcHandle(ctypes.Structure):  # CUipcMemHandle, passed by value
    _fields_ = [("reserved", ctypes.c_char * 64)]


if mode == "order":
    cuda = ctypes.CDLL("libcuda.so.1")
    n = 1 << 20
    x = torch.zeros(n, device=dev)
    torch.cuda.synchronize()
    # export this rank's allocation (base + offset) through CUDA IPC
    base, size = ctypes.c_uint64(), ctypes.c_size_t()
    assert cuda.cuMemGetAddressRange_v2(ctypes.byref(base), ctypes.byref(size), ctypes.c_uint64(x.data_ptr())) == 0
    handle = IpcHandle()
    assert cuda.cuIpcGetMemHandle(ctypes.byref(handle), base) == 0
    store.set(f"barrier/ipc/{rank}", bytes(handle) + (x.data_ptr() - base.value).to_bytes(8, "little"))
    peers, mapped = {}, []
    for p in range(world):
        if p == rank:
            continue
        blob = store.get(f"barrier/ipc/{p}")
        h = IpcHandle.from_buffer_copy(blob[:64])
        ptr = ctypes.c_uint64()
        # CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS
        rc = cuda.cuIpcOpenMemHandle_v2(ctypes.byref(ptr), h, ctypes.c_uint(1))
        assert rc == 0, f"cuIpcOpenMemHandle: {rc}"
        mapped.append(ptr.value)
        peers[p] = ptr.value + int.from_bytes(blob[64:72], "little")
    dist.barrier()  # every mapping is open
    for rnd in range(3):
        torch.cuda._sleep(int(2e8) * (rank + 1))  # ~0.1 s per rank index at 2 GHz
        x.fill_(100.0 * (rnd + 1) + rank)
        t0 = time.time()
        dist.barrier()
        waited = time.time() - t0
        for p, addr in peers.items():
            got = torch.empty(n, device=dev)
            # a copy on this rank's stream out of the peer's memory (NVLink)
            rc = cuda.cuMemcpyDtoDAsync_v2(ctypes.c_uint64(got.data_ptr()), ctypes.c_uint64(addr),
                                           ctypes.c_size_t(4 * n),
                                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            c.check("peer copy issued", rc == 0, f"cuMemcpyDtoDAsync {rc}")
            torch.cuda.synchronize()
            want = 100.0 * (rnd + 1) + p
            c.check(f"round {rnd}: rank {p}'s fill seen after the barrier", bool((got == want).all()),
                    f"got {got[:4].tolist()} want {want} (barrier took {waited:.3f} s)")
        dist.barrier()  # every read is done before the next fill
    peers.clear()
    torch.cuda.synchronize()
    for m in mapped:
        cuda.cuIpcCloseMemHandle(ctypes.c_uint64(m))
elif mode == "timeout":
    if rank == 0:
        t0 = time.time()
        try:
            dist.barrier()
            c.check("a barrier no peer joins raises", False, "it returned")
        except Exception as e:  # DistBackendError
            took = time.time() - t0
            c.check("the error names the timeout", "time" in str(e).lower(), str(e)[:300])
            c.check("the wait gave up within the device timeout", took < 30, f"{took:.1f} s")
        # the context still works
        y = torch.arange(8.0, device=dev) * 2
        c.check("context usable after the timeout", float(y.sum()) == 56.0)
        c.check("the device barrier ran", commux.stats().get("coll_barriers", 0) > 0, str(commux.stats()))
        store.set("barrier/timeout/done", b"1")
    else:
        store.wait(["barrier/timeout/done"])
c.finish()
