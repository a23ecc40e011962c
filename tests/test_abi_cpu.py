"""CPU-side checks of the boundary: the library builds, loads, exports every
symbol the header declares, and the host-side validation behaves like the
reference's asserts (no device call is made here)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "qwantize_b200.h")).read()
    return sorted(set(re.findall(r"^QZ_API\s+(?:int|const char\*)\s+(qz_\w+)\(", src, re.M)))


def test_library_exports_every_header_symbol():
    from qwantize_b200 import _lib
    L = _lib.load()
    syms = header_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(L, s), s
    assert set(syms) == set(_lib.EXPORTS)


def test_scale_tables_match_reference_definition():
    from qwantize_b200 import _lib
    t = _lib.scale_table(_lib.FMT_NVFP4)
    allb = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    assert torch.equal(t, allb[(allb > 0) & ~allb.isnan()].unique().sort().values)
    u = _lib.scale_table(_lib.FMT_MXFP4)
    assert torch.equal(u, torch.pow(2.0, torch.arange(1, 255).float() - 127.0))


def test_invalid_arguments_fail_before_any_device_call():
    from qwantize_b200 import _lib
    L = _lib.load()
    # bad block size -> QZ_ERR_INVALID with a message, no device touched
    st = L.qz_quantize(None, 1, 10, 8, 0, 0, None, 0, None, None, None, None, None, None, None)
    assert st == _lib.QZ_ERR_INVALID
    assert b"block_size" in L.qz_last_error()
    st = L.qz_fp4_unpack(None, 6, None, None)
    assert st == _lib.QZ_ERR_INVALID and b"multiple of 4" in L.qz_last_error()
    with pytest.raises(AssertionError):
        _lib.check(st)


def test_python_api_asserts_block_size():
    import qwantize_b200 as q
    with pytest.raises(AssertionError):
        q.nvfp4_naive(torch.zeros(4, 8))
    with pytest.raises(AssertionError):
        q.nvfp4_optimal_hessian(torch.zeros(4, 16))


def test_no_device_means_loud_failure():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import qwantize_b200 as q
    with pytest.raises(RuntimeError, match="CUDA"):
        q.nvfp4_optimal(torch.zeros(4, 16))


def test_division_free_rounding_is_exact_for_fp16_and_bf16():
    """The kernels replace bucketize(|x|/s) by counting thresholds B_k*s that
    |x| exceeds.  Exhaustive over every finite non-negative fp16 and bf16
    magnitude and every E4M3 / UE8M0 scale."""
    B = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
    from qwantize_b200 import _lib
    scales = torch.cat([_lib.scale_table(0), _lib.scale_table(1)])
    mags = [torch.arange(0, 0x7C00, dtype=torch.int32).to(torch.int16).view(torch.float16).float(),
            torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float()]
    for a in mags:
        for s in scales:
            ref = torch.bucketize(a / s, B)
            alt = (a[:, None] > (B * s)[None, :]).sum(-1)
            assert torch.equal(ref, alt), float(s)


def test_integer_formats_validation_and_tables():
    """NVINT4 / INT8 argument checks come before any device call; the INT8
    candidate table is the E4M3 values divided by 127 in fp32."""
    import ctypes

    from qwantize_b200 import _lib
    L = _lib.load()
    buf = ctypes.create_string_buffer(64)
    x = ctypes.addressof(buf) + (16 - ctypes.addressof(buf) % 16) % 16  # 16-byte aligned host address
    st = L.qz_quantize(x, 1, 4, 64, _lib.FMT_NVINT4, 0, None, 0, None, None, None, None, None, None, None)
    assert st == _lib.QZ_ERR_INVALID and b"expected one of (16, 32)" in L.qz_last_error()
    st = L.qz_quantize(x, 1, 4, 16, _lib.FMT_INT8, 0, None, 0, None, None, None, None, None, None, None)
    assert st == _lib.QZ_ERR_INVALID and b"expected one of (32, 64, 128, 256)" in L.qz_last_error()
    st = L.qz_quantize(x, 1, 4, 32, _lib.FMT_INT8, 4, None, 0, None, None, None, None, None, None, None)
    assert st == _lib.QZ_ERR_INVALID and b"naive, SSE and Hessian" in L.qz_last_error()
    st = L.qz_quantize(x, 1, 4, 32, _lib.FMT_INT8, 0, None, 0, None, x + 4, None, None, None, None, None)
    assert st == _lib.QZ_ERR_INVALID and b"16-byte aligned" in L.qz_last_error()
    st = L.qz_quantize(x, 1, 4, 32, _lib.FMT_NVINT4, 2, None, 0, None, None, None, None, None, None, None)
    assert st == _lib.QZ_ERR_INVALID and b"X or H_blocks" in L.qz_last_error()
    e4 = _lib.scale_table(_lib.FMT_NVINT4)
    assert torch.equal(e4, _lib.scale_table(_lib.FMT_NVFP4))
    assert torch.equal(_lib.scale_table(_lib.FMT_INT8), e4 / 127.0)
