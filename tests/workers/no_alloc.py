"""commux_strided_copy_noalloc, called through ctypes, against the existing
entry point that runs the same pull kernel (a CUDA self send/recv through the
backend) and against a torch copy, on calls made back to back on one stream.
Also checks that the calls leave the device memory in use unchanged and that
oversize, unsupported and out-of-range inputs are rejected before launch."""
import ctypes
import os
import zlib

from common import Checker, init, torch, dist

import commux_b200

rank, world, dev = init(timeout_s=90)
c = Checker(rank)
lib = ctypes.CDLL(os.path.join(os.path.dirname(commux_b200.__file__), "lib", "libcommux_cuda.so"))
fn = lib.commux_strided_copy_noalloc
I64P = ctypes.POINTER(ctypes.c_int64)
fn.restype = ctypes.c_int
fn.argtypes = [ctypes.c_void_p, I64P, ctypes.c_void_p, I64P, I64P, ctypes.c_int, ctypes.c_int,
               ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
ERR = ctypes.create_string_buffer(512)


def arr(v):
    return (ctypes.c_int64 * max(1, len(v)))(*v)


def raw(dst_ptr, dst_strides, src_ptr, src_strides, sizes, elem):
    ERR.value = b""
    rc = fn(dst_ptr, arr(dst_strides), src_ptr, arr(src_strides), arr(sizes), len(sizes), elem,
            torch.cuda.current_stream().cuda_stream, ERR, len(ERR))
    return rc, ERR.value.decode()


def noalloc(dst, src):
    assert dst.shape == src.shape and dst.dtype == src.dtype
    return raw(dst.data_ptr(), dst.stride(), src.data_ptr(), src.stride(), list(src.shape), src.element_size())


def data(shape, dtype, salt):
    g = torch.Generator().manual_seed(zlib.crc32(repr((shape, str(dtype), salt)).encode()))
    if dtype.is_floating_point:
        return torch.randn(shape, generator=g).to(dtype)
    return torch.randint(-100, 100, shape, generator=g).to(dtype)


# (name, full shape, dtype, source view, destination view of a same-shaped buffer)
cases = [
    ("strided rows f64", (64, 48), torch.float64, lambda t: t[:, 5:40:3], None),
    ("x-face into ghost f32", (40, 36, 36), torch.float32, lambda t: t[2:38, 2:34, 2:4],
     lambda t: t[2:38, 2:34, 34:36]),
    ("transpose f16", (33, 17), torch.float16, lambda t: t.t(), None),
    ("contig bf16", (3, 1 << 20), torch.bfloat16, lambda t: t, None),
    ("odd bytes u8", (1001,), torch.uint8, lambda t: t, None),
]


def buffers(shape, dtype, sview, dview, salt):
    s = data(shape, dtype, salt).to(dev)
    sv = sview(s)
    if dview is None:
        return sv, torch.zeros(sv.shape, dtype=dtype, device=dev), torch.zeros(sv.shape, dtype=dtype, device=dev)
    a, b = torch.zeros(shape, dtype=dtype, device=dev), torch.zeros(shape, dtype=dtype, device=dev)
    return sv, dview(a), dview(b)


tag = 300
for i in range(0, len(cases), 2):
    pair = cases[i:i + 2]
    for rep in range(2):
        bufs = [buffers(shape, dt, sv, dv, (rep, k)) for k, (_, shape, dt, sv, dv) in enumerate(pair)]
        # the existing entry point: a CUDA self send/recv (pull kernel, per-stream scratch)
        for sv, ref, _ in bufs:
            r = dist.irecv(ref, rank, tag=tag)
            s = dist.isend(sv, rank, tag=tag)
            r.wait()
            s.wait()
            tag += 1
        # the no-alloc entry point, two calls back to back on the current stream
        for (name, *_), (sv, _, out) in zip(pair, bufs):
            rc, msg = noalloc(out, sv)
            c.check(f"{name} rc", rc == 0, msg)
        torch.cuda.synchronize()
        for (name, *_), (sv, ref, out) in zip(pair, bufs):
            want = sv.contiguous().cpu()
            c.equal(f"{name} rep{rep} existing path", ref.cpu(), want)
            c.equal(f"{name} rep{rep} noalloc", out.cpu(), want)
            c.check(f"{name} rep{rep} bit-identical", torch.equal(out.cpu(), ref.cpu()))

# device memory in use does not change across calls made after the set-up call
src = data((4096, 257), torch.float32, "mem").to(dev)
dst = torch.zeros(257, 4096, device=dev)
torch.cuda.synchronize()
before = (torch.cuda.memory_allocated(), torch.cuda.memory_reserved(), torch.cuda.mem_get_info()[0])
for _ in range(3):
    rc, msg = noalloc(dst, src.t())
    c.check("mem rc", rc == 0, msg)
torch.cuda.synchronize()
after = (torch.cuda.memory_allocated(), torch.cuda.memory_reserved(), torch.cuda.mem_get_info()[0])
c.check("no device allocation", before == after, f"before {before} after {after}")
c.equal("mem copy", dst.cpu(), src.t().cpu())

# rejections happen on the host, before anything is launched
small = torch.zeros(64, device=dev)
p = small.data_ptr()
rc, msg = raw(p, [1 << 31, 1], p, [1 << 30, 1], [2000, 1 << 30], 1)
c.check("oversize rejected", rc == 2 and "too large" in msg, f"rc {rc} {msg!r}")
rc, msg = raw(p, [1, 1 << 31], p, [1 << 31, 1], [1 << 31, 1 << 31], 1)
c.check("oversize inner rejected", rc == 2 and "too large" in msg, f"rc {rc} {msg!r}")
rc, msg = raw(p, [16, 8, 4, 2, 1], p, [1, 2, 4, 8, 16], [2, 2, 2, 2, 2], 4)
c.check("5 dims rejected", rc == 3, f"rc {rc} {msg!r}")
rc, msg = raw(p, [1], p, [1], [1 << 28], 4)
c.check("out of allocation rejected", rc == 4 and "leaves its allocation" in msg, f"rc {rc} {msg!r}")
rc, msg = raw(p, [1], p, [1], [8], 3)
c.check("bad elem size rejected", rc == 1, f"rc {rc} {msg!r}")
host = torch.zeros(64)
rc, msg = raw(p, [1], host.data_ptr(), [1], [64], 4)
c.check("host memory rejected", rc == 4, f"rc {rc} {msg!r}")
c.equal("untouched", small.cpu(), torch.zeros(64))
c.finish()
