"""The allocation-free full Gram entry point, qz_gram_full_noalloc.

Some callers cannot let a library allocate device memory mid-call: code that
runs inside another framework's memory pool or allocator hook, or a program
that has already handed the device's memory to another component.  For them
the full Gram keeps its per-tile counters in a fixed device array inside the
library instead of a per-call buffer.  This test calls it through the C ABI
twice in a row and checks each result against the regular qz_gram entry
point (and against a double-precision Gram within the fp32-accumulation bound
the other Gram tests use).  It lives in its own file, collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _x(T, K, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(T, K, generator=g) * torch.exp(torch.randn(K, generator=g))).to(torch.bfloat16)


def test_noalloc_gram_matches_qz_gram_twice():
    from qwantize_b200 import _lib
    L = _lib.load()
    dev = torch.device("cuda", 0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    # 600,000 tokens span three 262,144-row segments: a segment's add waits on
    # the tile's counter, so stale counters from the previous call would let a
    # later segment run before the first one's overwrite and drop its sum
    for T, K, seed in ((3000, 384, 1), (70000, 512, 2), (600000, 256, 3)):
        X = _x(T, K, seed).to(dev)
        ref = torch.empty(K, K, device=dev)
        _lib.check(L.qz_gram(ctypes.c_void_p(X.data_ptr()), T, K, _lib.GRAM_FULL, 16, 0,
                             ctypes.c_void_p(ref.data_ptr()), stream), "qz_gram")
        for _ in range(2):  # two calls in a row: the shared counters must be re-zeroed
            H = torch.full((K, K), float("nan"), device=dev)
            _lib.check(L.qz_gram_full_noalloc(ctypes.c_void_p(X.data_ptr()), T, K, 0,
                                              ctypes.c_void_p(H.data_ptr()), stream),
                       "qz_gram_full_noalloc")
            torch.cuda.synchronize()
            assert torch.equal(H, ref)
        Xd = X.double().cpu()
        err = (H.double().cpu() - Xd.T @ Xd).abs()
        assert bool((err <= T * 2.0 ** -24 * (Xd.abs().T @ Xd.abs()) + 1e-30).all())
    assert L.qz_poll_device_error(0, None) == _lib.QZ_OK


def test_noalloc_gram_rejects_too_large_k():
    from qwantize_b200 import _lib
    L = _lib.load()
    st = L.qz_gram_full_noalloc(ctypes.c_void_p(16), 64, 92424, 0, ctypes.c_void_p(16), None)
    assert st == _lib.QZ_ERR_INVALID
    assert b"92416" in L.qz_last_error()
