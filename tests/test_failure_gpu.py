"""Failure detection without a GPU fault: a device-side bounded wait that runs
out sets the device error word and returns; the host reads it as
ACT_E_TIMEOUT and the context stays usable.  Nothing traps or hangs -- the wait
is cut to a few thousand polls, and the barrier it waits on simply never
completes."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from actcomp import _lib

    return _lib


def test_bounded_wait_times_out_and_reports():
    L = _lib()
    lib = L.load()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.actcomp_clear_device_error(s) == L.ACT_OK
    word = ctypes.c_uint32(0)
    # a wait that completes leaves the word alone
    assert lib.actcomp_selftest_bounded_wait(1024, 1, s) == L.ACT_OK
    assert lib.actcomp_last_device_error(s, ctypes.byref(word)) == L.ACT_OK and word.value == 0
    # a wait on a barrier nothing completes gives up after its polls and returns
    t0 = time.perf_counter()
    assert lib.actcomp_selftest_bounded_wait(4096, 0, s) == L.ACT_OK
    st = lib.actcomp_last_device_error(s, ctypes.byref(word))  # synchronises the stream
    assert time.perf_counter() - t0 < 10.0
    assert st == L.ACT_E_TIMEOUT and word.value & 1
    # the context is still usable, and the word clears
    assert lib.actcomp_clear_device_error(s) == L.ACT_OK
    assert lib.actcomp_last_device_error(s, ctypes.byref(word)) == L.ACT_OK and word.value == 0
    import actcomp

    x = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    c = actcomp.encode(x, None, None, bits=8, group=128)
    xh = actcomp.decode(c)
    torch.cuda.synchronize()
    assert (xh.float() - x.float()).norm() / x.float().norm() < 1e-2
