"""Failure detection on the GPU without a fault: a cross-GPU wait that runs
out.  The all-reduce of a simulated second rank that never runs (its areas
live on this GPU and nothing ever sets its flags) must end with the device
error word reading the peer time-out (6), within the configured bound, and
leave the context usable."""

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

K_DEV_TIMEOUT_PEER = 6


def test_peer_wait_times_out_and_context_survives(cuda):
    from mu_b200 import _lib

    lib = _lib.load()
    world, n = 2, 4096
    scratch = int(lib.muk_allreduce_scratch_elems(n, world))
    flag_words = int(lib.muk_allreduce_flag_bytes()) // 4 + 4
    data = [torch.ones(n, device=cuda) for _ in range(world)]
    scr = [torch.zeros(scratch, device=cuda) for _ in range(world)]
    flags = [torch.zeros(flag_words, dtype=torch.int32, device=cuda) for _ in range(world)]

    def arr(ts):
        return (ctypes.c_void_p * world)(*[t.data_ptr() for t in ts])

    b, s, f = arr(data), arr(scr), arr(flags)
    assert _lib.device_error() == 0
    _lib.call("muk_set_peer_timeout_ms", 200)
    try:
        t0 = time.time()
        _lib.call("muk_allreduce_f32", ctypes.addressof(b), ctypes.addressof(s),
                  ctypes.addressof(f), 0, world, n, 1, n, torch.cuda.current_stream().cuda_stream)
        code = _lib.device_error()  # synchronises
        elapsed = time.time() - t0
    finally:
        _lib.call("muk_set_peer_timeout_ms", 5000)
    assert code == K_DEV_TIMEOUT_PEER
    assert elapsed < 5.0  # two waits of 0.2 s each, not the 5 s default
    # the context is still usable and the error word was cleared
    x = torch.arange(10, device=cuda, dtype=torch.float32)
    assert float((x * 2).sum()) == 90.0
    assert _lib.device_error() == 0


def test_peer_timeout_bounds_checked(cuda):
    from mu_b200 import _lib

    lib = _lib.load()
    assert lib.muk_set_peer_timeout_ms(0) == _lib.MUK_ERR_INVALID_ARG
    assert lib.muk_set_peer_timeout_ms(5000) == 0
