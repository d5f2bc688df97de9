"""A bounded device wait that runs out: the kernel gives up, sets the library's device error
word and returns, and the context stays usable.

The peer all-reduce kernel (tropnn_b200_peer_allreduce_f32) is launched as rank 0 of a
two-rank set whose second "rank" is a second peer buffer on the same GPU that no kernel ever
serves: rank 0 pushes its data into both buffers, raises its flags and then waits for rank 1's
flag, which nothing sets. Its wait is bounded (2 s, on %globaltimer); after the limit every
CTA sets the error word and leaves. The test reads the word through
tropnn_b200_device_error (which also clears it), checks that the tensor was left untouched
(the kernel returns before writing results) and that kernels still run afterwards. No GPU
fault, trap or hang is involved: every address is a valid local allocation and every wait
ends.
"""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

from tropnn_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _device_error() -> int:
    flag = ctypes.c_int(-1)
    nat.check(nat.load().tropnn_b200_device_error(ctypes.byref(flag)), "device_error")
    return flag.value


def test_peer_wait_runs_out_and_reports_the_error() -> None:
    lib = nat.load()
    torch.cuda.set_device(0)
    assert _device_error() == 0  # clean start (reading also clears)
    capacity = 4096
    locals_: list[int] = []
    try:
        for _ in range(2):
            local = ctypes.c_void_p()
            handle = (ctypes.c_ubyte * 64)()
            nat.check(lib.tropnn_b200_peer_buffer_create(capacity, ctypes.byref(local), handle), "peer_buffer_create")
            locals_.append(local.value)
        buffers = (ctypes.c_void_p * 2)(*locals_)
        t = torch.arange(1000, dtype=torch.float32, device="cuda")
        before = t.clone()
        segments = (ctypes.c_void_p * 1)(t.data_ptr())
        counts = (ctypes.c_int64 * 1)(t.numel())
        stream = nat.stream_handle(t.device)
        t0 = time.perf_counter()
        nat.check(lib.tropnn_b200_peer_allreduce_f32(buffers, 2, 0, capacity, segments, counts, 1, 1, stream),
                  "peer_allreduce")
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert waited >= 1.5, f"the wait ended after {waited:.2f} s, before its 2 s limit"
        assert waited < 30.0
        assert _device_error() == 1
        assert _device_error() == 0  # the read cleared it
        assert torch.equal(t, before)  # no result was written after the failed barrier
        # The context is still usable: ordinary kernels (ours and torch's) run and agree.
        y = (t * 2.0).sum()
        assert float(y) == pytest.approx(999.0 * 1000.0)
    finally:
        torch.cuda.synchronize()
        for ptr in locals_:
            nat.check(lib.tropnn_b200_peer_buffer_destroy(ctypes.c_void_p(ptr)), "peer_buffer_destroy")
    assert _device_error() == 0
