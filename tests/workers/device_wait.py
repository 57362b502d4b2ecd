"""Makes device-side waits run out on flags that nothing sets (a 300 ms limit)
and checks that each one records its status and returns, with the context
still usable afterwards. See commux_device_wait_selftest in
csrc/cuda/wait_selftest.cu for the cases. One process, one GPU."""
import ctypes
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
torch.cuda.init()
lib = ctypes.CDLL(os.path.join(ROOT, "commux_b200", "lib", "libcommux_cuda.so"))
fn = lib.commux_device_wait_selftest
fn.restype = ctypes.c_int
fn.argtypes = [ctypes.c_void_p, ctypes.c_uint, ctypes.c_char_p, ctypes.c_size_t]
err = ctypes.create_string_buffer(512)
rc = fn(torch.cuda.current_stream().cuda_stream, 300, err, len(err))
msg = err.value.decode()
if rc != 0:
    print(f"FAIL ({rc}): {msg}", flush=True)
    sys.exit(1)
# the process can still run CUDA work
x = torch.ones(1 << 20, device="cuda", dtype=torch.float32)  # every partial sum exact in fp32
assert float(x.sum()) == float(1 << 20)
print("PASS device waits give up, report and leave the context usable", flush=True)
