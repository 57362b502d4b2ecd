"""Runs the bounds-check self-test of a libcommux_cuda.so built with
COMMUX_DEVICE_CHECKS (path in argv[1]) and checks that the package's
production library reports the checks as compiled out (argv[2]).

Runs in its own process: the two libraries share a soname, so they are never
loaded side by side."""
import ctypes
import sys

import torch

which, path = sys.argv[1], sys.argv[2]
torch.cuda.init()
lib = ctypes.CDLL(path)
lib.commux_device_checks_enabled.restype = ctypes.c_int
lib.commux_device_check_selftest.restype = ctypes.c_int
lib.commux_device_check_selftest.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
err = ctypes.create_string_buffer(512)
enabled = lib.commux_device_checks_enabled()
rc = lib.commux_device_check_selftest(torch.cuda.current_stream().cuda_stream, err, len(err))
msg = err.value.decode()
if which == "checked":
    assert enabled == 1, "bounds-check library reports the checks compiled out"
    assert rc == 0, f"self-test failed ({rc}): {msg}"
else:
    assert enabled == 0, "production library reports bounds checks compiled in"
    assert rc == 1, f"production self-test returned {rc}: {msg}"
print(f"PASS {which}: {msg}")
