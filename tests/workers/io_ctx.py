"""IOContext: collective open/write/sync/close with error agreement, and
broadcast/gather of byte strings (reference: src/io.cpp:64-180; the reference
has no test for it)."""
import os
import sys

from common import ROOT  # noqa: F401
import commux_b200 as commux

rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
io = commux.make_tcp_io_context("127.0.0.1", int(os.environ["MASTER_PORT"]), rank, world)
fail = []
path = os.environ["CMX_IO_PATH"]
fd = io.open_file(path, os.O_CREAT | os.O_WRONLY, 0o644)
io.write_at(fd, bytes([65 + rank]) * 4, rank * 4)
io.sync_file(fd)
io.close_file(fd)
io.barrier()
if open(path, "rb").read() != b"".join(bytes([65 + r]) * 4 for r in range(world)):
    fail.append("file contents")
got = io.broadcast_bytes(b"hello" if rank == 1 else b"", 1)
if got != b"hello":
    fail.append(f"broadcast_bytes {got!r}")
g = io.gather_bytes(bytes([rank]) * (rank + 1), 0)
if rank == 0 and g != b"".join(bytes([r]) * (r + 1) for r in range(world)):
    fail.append(f"gather_bytes {g!r}")
# an empty payload, a large one, and a root other than 0
g2 = io.gather_bytes(b"" if rank == 0 else bytes([rank]) * (70000 * rank), world - 1)
want2 = b"".join(b"" if r == 0 else bytes([r]) * (70000 * r) for r in range(world))
if rank == world - 1 and g2 != want2:
    fail.append(f"gather_bytes (root {world - 1}) {len(g2)} bytes, want {len(want2)}")
if rank != world - 1 and g2 != b"":
    fail.append("gather_bytes returned data on a non-root rank")
try:
    fd2 = os.open(path, os.O_RDONLY)
    try:
        io.write_at(fd2, b"x", 0)  # read-only descriptor: the write must fail with progress
        fail.append("write_at on a read-only descriptor did not raise")
    except RuntimeError as e:
        if "0 of 1 bytes written" not in str(e):
            fail.append(f"write_at error text: {e}")
    finally:
        os.close(fd2)
except OSError as e:
    fail.append(f"reopen: {e}")
try:
    io.open_file("/nonexistent/dir/x" if rank == world - 1 else path, os.O_RDONLY, 0)
    fail.append("open_file error was not agreed")
except RuntimeError as e:
    if "open_file failed" not in str(e):
        fail.append(f"open_file error text: {e}")
if world > 1:
    if rank == 0:
        io.send_bytes(b"xyz", 1, 5)
    elif rank == 1:
        if io.recv_bytes(3, 0, 5) != b"xyz":
            fail.append("send/recv bytes")
io.barrier()
print("FAIL" if fail else "ok", fail, flush=True)
sys.exit(1 if fail else 0)
