"""commux_strided_copy_noalloc, called through ctypes, against the existing
entry point that runs the same pull kernel (a CUDA self send/recv through the
backend) and against a torch copy, on calls made back to back on one stream.
Also checks that the calls leave the device memory in use unchanged -- first
in this fresh process, where the set-up call loads the kernels and every
later call's kernel build (16/8/4/2/1-byte units and the 64-bit-stride walk)
is launched for the first time -- and that oversize, unsupported and
out-of-range inputs are rejected before launch."""
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


def free_bytes():
    torch.cuda.synchronize()
    return torch.cuda.mem_get_info()[0], torch.cuda.memory_reserved()


# -- fresh process: no pull kernel has run yet. Buffers first (torch's own
# kernels load here), then the set-up call, then the first call of every
# other kernel build, with the free device memory compared around them.
f32 = data((64, 1024), torch.float32, "fresh").to(dev)
f32_out = torch.zeros_like(f32)
firsts = []  # (name, dst view, src view, elem bytes or None for dst.element_size())
for name, dtype, step in (("8-byte units", torch.float64, 2), ("4-byte units", torch.float32, 2),
                          ("2-byte units", torch.float16, 2), ("1-byte units", torch.uint8, 2)):
    src_t = data((4096,), dtype, name).to(dev)
    firsts.append((name, torch.zeros(2048, dtype=dtype, device=dev), src_t[::step]))
# strides of 2^31 bytes and more (the 64-bit walk): two rows 2 GiB + 64 B apart
wide_pitch = (1 << 28) + 8
wide_src = torch.zeros(wide_pitch + 64, dtype=torch.float64, device=dev)
wide_src[:64] = torch.arange(64, dtype=torch.float64, device=dev)
wide_src[wide_pitch:wide_pitch + 64] = -torch.arange(64, dtype=torch.float64, device=dev)
wide_out = torch.zeros(2, 64, dtype=torch.float64, device=dev)
torch.cuda.synchronize()
rc, msg = noalloc(f32_out, f32)  # the set-up call
c.check("set-up call rc", rc == 0, msg)
before = free_bytes()
for name, out, sv in firsts:
    rc, msg = noalloc(out, sv)
    c.check(f"first call, {name}: rc", rc == 0, msg)
rc, msg = raw(wide_out.data_ptr(), [64, 1], wide_src.data_ptr(), [wide_pitch, 1], [2, 64], 8)
c.check("first call, 2 GiB stride: rc", rc == 0, msg)
after = free_bytes()
c.check("first calls of every kernel build allocate nothing", before == after, f"before {before} after {after}")
c.equal("set-up call copy", f32_out.cpu(), f32.cpu())
for name, out, sv in firsts:
    c.equal(f"first call, {name}", out.cpu(), sv.cpu())
c.equal("2 GiB stride copy", wide_out.cpu(),
        torch.stack([torch.arange(64, dtype=torch.float64), -torch.arange(64, dtype=torch.float64)]))
del wide_src
torch.cuda.empty_cache()

# negative strides (the raw C API allows them): a reversed copy, pointer at
# the last element
rev = data((1000,), torch.float32, "rev").to(dev)
rev_out = torch.zeros_like(rev)
rc, msg = raw(rev_out.data_ptr(), [1], rev.data_ptr() + 999 * 4, [-1], [1000], 4)
c.check("reversed rc", rc == 0, msg)
c.equal("reversed copy", rev_out.cpu(), rev.cpu().flip(0))
rev2 = data((30, 40), torch.float64, "rev2").to(dev)
rev2_out = torch.zeros(30, 20, dtype=torch.float64, device=dev)
rc, msg = raw(rev2_out.data_ptr(), [20, 1], rev2.data_ptr() + (29 * 40 + 1) * 8, [-40, 2], [30, 20], 8)
c.check("reversed rows rc", rc == 0, msg)
c.equal("reversed rows copy", rev2_out.cpu(), rev2.cpu().flip(0)[:, 1::2])
# 16-byte elements: every other 16-byte pair of a float64 buffer
e16 = data((512,), torch.float64, "e16").to(dev)
e16_out = torch.zeros(256, dtype=torch.float64, device=dev)
rc, msg = raw(e16_out.data_ptr(), [1], e16.data_ptr(), [2], [128], 16)
c.check("16-byte elements rc", rc == 0, msg)
c.equal("16-byte elements", e16_out.cpu(), e16.cpu().view(128, 4)[:, :2].reshape(-1))

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
