"""The bounded device-side wait, made to run out on purpose.

Every kernel of the library waits on mbarriers (bulk-copy landings, the
tensor-core pipeline) with a time limit; when a wait gives up, the kernel
records a flag, waits (bounded) for its own copies in flight and returns, and
qz_poll_device_error reports QZ_ERR_TIMEOUT.  qz_selftest_wait runs that same
wait on an mbarrier nothing arrives on, with a limit of a few microseconds, so
the failure path runs without faulting or hanging the GPU."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_survives():
    import qwantize_b200 as q
    from qwantize_b200 import _lib
    L = _lib.load()
    dev = torch.device("cuda", 0)
    torch.cuda.synchronize(dev)
    flags = ctypes.c_uint(0)
    assert L.qz_poll_device_error(1, ctypes.byref(flags)) == _lib.QZ_OK  # start clean
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    assert L.qz_selftest_wait(5000, stream) == _lib.QZ_OK
    torch.cuda.synchronize(dev)
    assert L.qz_poll_device_error(0, ctypes.byref(flags)) == _lib.QZ_ERR_TIMEOUT
    assert flags.value & 1
    # clearing resets the flag; the context still runs work correctly
    assert L.qz_poll_device_error(1, None) == _lib.QZ_ERR_TIMEOUT
    assert L.qz_poll_device_error(0, ctypes.byref(flags)) == _lib.QZ_OK and flags.value == 0
    from qwantize_b200.synthetic import make_weight
    W = make_weight(64, 512, seed=9)
    s_gpu, q_gpu = q.nvfp4_optimal(W.to(dev).reshape(64, 32, 16))
    s_ref, q_ref = q.nvfp4_optimal(W.to(dev).reshape(64, 32, 16))
    assert torch.equal(s_gpu, s_ref) and torch.equal(q_gpu, q_ref)
    assert L.qz_poll_device_error(0, None) == _lib.QZ_OK


def test_wait_limit_is_checked():
    from qwantize_b200 import _lib
    L = _lib.load()
    assert L.qz_selftest_wait(2_000_000_000, None) == _lib.QZ_ERR_INVALID
