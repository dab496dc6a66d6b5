"""The device's glibc-compatible expf, checked exhaustively against the host libm.

The reference calls libm expf in two tails: the softmax of the last kv_len % 8 scores
(dpuf_engine.c:406-409), whose argument s - max is <= 0, and the scalar SwiGLU tail
(dpuf_engine.c:990-996), expf(-g) for |g| < 40.  The device reproduces glibc's expf with a
double-precision exp rounded to float plus an exception table built from the host libm
(expf_table.cu).  This test evaluates the device function for EVERY float in [-160, 0] (below
about -104 expf is 0) and in [0, 40], and requires bit-identical results everywhere."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (first bit pattern, last bit pattern) of each range, inclusive
RANGES = [(0x80000000, 0xC3200000),  # -0 .. -160.0
          (0x00000000, 0x42200000)]  # +0 .. 40.0
CHUNK = 1 << 26


def test_device_expf_equals_host_libm_on_every_reachable_input():
    import ctypes

    import torch

    from dpuf_b200 import engine
    from oracle import oracle as orc

    assert torch.cuda.is_available(), "GPU test needs a CUDA device"
    lib = engine.cuda_lib()
    lib.dpuf_cuda_expf_eval.restype = ctypes.c_int32
    lib.dpuf_cuda_expf_eval.argtypes = [ctypes.c_uint32, ctypes.c_int64, ctypes.c_void_p]
    buf = torch.empty(CHUNK, dtype=torch.float32, device="cuda")
    host = torch.empty(CHUNK, dtype=torch.float32, pin_memory=True)
    checked = 0
    for lo, hi in RANGES:
        for b0 in range(lo, hi + 1, CHUNK):
            n = min(CHUNK, hi + 1 - b0)
            assert lib.dpuf_cuda_expf_eval(b0, n, buf.data_ptr()) == 0, engine.last_error()
            host[:n].copy_(buf[:n])
            bad, first = orc.expf_mismatch(b0, host[:n].numpy())
            assert bad == 0, f"{bad} inputs differ from libm expf, first at bits {b0 + first:#010x}"
            checked += n
    assert checked == (0xC3200000 - 0x80000000 + 1) + (0x42200000 + 1)
