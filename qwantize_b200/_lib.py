"""ctypes binding of libqwantize_b200.so (the C ABI in include/qwantize_b200.h).

The library is loaded from this package directory (built in-tree by
``python -m qwantize_b200.build``).  There is no fallback: if the library or a
sm_100 GPU is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwantize_b200.so")

QZ_OK, QZ_ERR_INVALID, QZ_ERR_CUDA, QZ_ERR_TIMEOUT, QZ_ERR_UNSUPPORTED = 0, 1, 2, 3, 4
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
FMT_NVFP4, FMT_MXFP4 = 0, 1
FMT_NVINT4, FMT_INT8 = 3, 4  # symmetric integer grids (nvint4/, int8/ of the reference)
METHOD_NAIVE, METHOD_SSE, METHOD_HESSIAN, METHOD_NAIVE_ARGMIN, METHOD_TWO_ARGMIN = 0, 1, 2, 3, 4
GRAM_FULL, GRAM_BLOCKDIAG, GRAM_FULL_UPPER_TILES = 0, 1, 2

# every symbol include/qwantize_b200.h declares
EXPORTS = [
    "qz_quantize", "qz_dequantize", "qz_dequantize_packed", "qz_fp4_unpack", "qz_gram",
    "qz_weight_error_sums", "qz_output_error_sums", "qz_scale_table", "qz_last_error",
    "qz_version", "qz_device_ok", "qz_poll_device_error", "qz_gram_full_noalloc", "qz_admm",
    "qz_quantize_table", "qz_selftest_wait", "qz_quantize_grouped", "qz_gptq", "qz_spd_inverse",
    "qz_gram_unpack",
]


class QzQuantItem(ctypes.Structure):
    """One input of qz_quantize_grouped (include/qwantize_b200.h)."""
    _fields_ = [("x", ctypes.c_void_p), ("n_blocks", ctypes.c_int64), ("scales", ctypes.c_void_p),
                ("quants", ctypes.c_void_p), ("dq", ctypes.c_void_p), ("scale_codes", ctypes.c_void_p),
                ("packed", ctypes.c_void_p), ("dq_bf16", ctypes.c_void_p)]

_lib = None


class QwantizeError(RuntimeError):
    pass


def load():
    """Load and type the library (CPU-safe: no device call happens here)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: run `python -m qwantize_b200.build` first")
    L = ctypes.CDLL(LIB_PATH)
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.qz_quantize.argtypes = [vp, i32, i64, i32, i32, i32, vp, i64, vp, vp, vp, vp, vp, vp, vp]
    L.qz_dequantize.argtypes = [vp, vp, i64, i32, vp, vp]
    L.qz_quantize_table.argtypes = [vp, i32, i64, i32, i32, vp, i32, vp, i64, vp, vp, vp, vp, vp, vp, vp]
    L.qz_admm.argtypes = [vp, i32, i64, i32, vp, vp, vp, i64, i32, i32, ctypes.c_float, vp, vp, vp, vp, vp,
                          vp, vp]
    L.qz_dequantize_packed.argtypes = [vp, vp, i64, i32, i32, vp, vp, vp]
    L.qz_fp4_unpack.argtypes = [vp, i64, vp, vp]
    L.qz_gram.argtypes = [vp, i64, i64, i32, i32, i32, vp, vp]
    L.qz_gram_full_noalloc.argtypes = [vp, i64, i64, i32, vp, vp]
    L.qz_weight_error_sums.argtypes = [vp, i32, vp, i32, i64, vp, vp]
    L.qz_output_error_sums.argtypes = [vp, i64, i64, vp, vp, i64, vp, vp]
    L.qz_scale_table.argtypes = [i32, vp, vp]
    L.qz_poll_device_error.argtypes = [i32, vp]
    L.qz_selftest_wait.argtypes = [ctypes.c_uint64, vp]
    L.qz_quantize_grouped.argtypes = [vp, i32, i32, i32, i32, i32, vp]
    L.qz_spd_inverse.argtypes = [vp, i64, vp, vp, vp]
    L.qz_gram_unpack.argtypes = [vp, i64, vp, vp]
    L.qz_gptq.argtypes = [vp, vp, vp, vp, vp, i64, i64, i32, i32, i32, i32, vp, vp, vp]
    L.qz_last_error.restype = ctypes.c_char_p
    for name in EXPORTS:
        if name not in ("qz_last_error",):
            getattr(L, name).restype = ctypes.c_int
    L.qz_last_error.restype = ctypes.c_char_p
    _lib = L
    return L


def check(status: int, what: str = "") -> None:
    if status == QZ_OK:
        return
    msg = load().qz_last_error().decode(errors="replace")
    if status == QZ_ERR_INVALID:
        raise AssertionError(msg)
    raise QwantizeError(f"{what}: {msg} (status {status})")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return DTYPE_BF16
    if dt == torch.float16:
        return DTYPE_F16
    if dt == torch.float32:
        return DTYPE_F32
    raise ValueError(f"unsupported dtype {dt}")


def scale_table(fmt: int) -> torch.Tensor:
    buf = (ctypes.c_float * 256)()
    n = ctypes.c_int(0)
    check(load().qz_scale_table(fmt, buf, ctypes.byref(n)), "qz_scale_table")
    return torch.tensor(list(buf)[: n.value], dtype=torch.float32)
