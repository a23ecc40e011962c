"""ctypes wrapper around liboracle.so, the CPU restatement of qwantize's scale search.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline legs of bench.py, as the checker.  The product package
(qwantize_b200) never imports it.

Every entry point takes/returns numpy arrays.  Work over many blocks is split
into ranges run on a thread pool (ctypes drops the GIL during the C call).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

DT_F32, DT_BF16, DT_F16 = 0, 1, 2
FMT_NVFP4, FMT_MXFP4 = 0, 1
M_NAIVE, M_SSE, M_HESSIAN, M_NAIVE_TORCH, M_TWO_TORCH = 0, 1, 2, 3, 4

_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (IEEE flags)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "qz_oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.qzo_quantize.argtypes = [vp, i32, i64, i32, i32, i32, vp, i64, vp, vp, vp]
        L.qzo_quantize.restype = i64
        L.qzo_e4m3_snap.argtypes = [ctypes.c_float]
        L.qzo_e4m3_snap.restype = ctypes.c_float
        L.qzo_e4m3_code.argtypes = [ctypes.c_float]
        L.qzo_e4m3_code.restype = ctypes.c_uint8
        L.qzo_ue8m0_code.argtypes = [ctypes.c_float]
        L.qzo_ue8m0_code.restype = ctypes.c_uint8
        L.qzo_e4m3_table.argtypes = [vp]
        L.qzo_ue8m0_table.argtypes = [vp]
        L.qzo_pack.argtypes = [vp, i64, vp]
        L.qzo_unpack.argtypes = [vp, i64, vp]
        L.qzo_dequantize.argtypes = [vp, vp, i64, i32, vp]
        L.qzo_block_gram.argtypes = [vp, i64, i64, i32, vp]
        L.qzo_gram.argtypes = [vp, i64, i64, vp]
        L.qzo_metrics.argtypes = [vp, vp, i64, i64, vp, i64, vp]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data


def _dtype_code(x: np.ndarray, bf16: bool) -> int:
    if bf16:
        assert x.dtype == np.uint16
        return DT_BF16
    if x.dtype == np.float16:
        return DT_F16
    assert x.dtype == np.float32
    return DT_F32


def quantize(x, bs, fmt, method, H=None, bf16=True, want_dq=True, threads=None, counts=False):
    """Quantize a flat array of n_blocks*bs elements.

    x: uint16 bf16 bit patterns (bf16=True), float16 or float32.
    Returns (scales, quants, dq, n_candidates_in_range); with counts=True the
    last item is (n_in_range, n_full_evaluations): candidates inside the
    search bounds, and those that passed the clipping fast-fail and had their
    full error evaluated (the reference's own loop, nvfp4/reference.py:191-228).
    """
    x = np.ascontiguousarray(x).reshape(-1)
    n_blocks = x.size // bs
    dt = _dtype_code(x, bf16)
    scales = np.empty(n_blocks, np.float32)
    quants = np.empty(n_blocks * bs, np.float32)
    dq = np.empty(n_blocks * bs, np.float32) if want_dq else None
    J = 0
    if method == M_HESSIAN:
        H = np.ascontiguousarray(H, dtype=np.float32)
        J = H.shape[0]
    threads = threads or os.cpu_count() or 1
    L = lib()
    esz = x.itemsize
    if method == M_HESSIAN:
        # ranges must keep the (block % J) mapping: split on multiples of J
        step = max(J, ((n_blocks // (threads * 8)) // J) * J or J)
    else:
        step = max(1024, n_blocks // (threads * 8) + 1)
    ranges = [(b, min(n_blocks, b + step)) for b in range(0, n_blocks, step)]

    def run(r):
        b0, b1 = r
        return L.qzo_quantize(
            x.ctypes.data + b0 * bs * esz, dt, b1 - b0, bs, fmt, method,
            _ptr(H), J,
            scales.ctypes.data + b0 * 4, quants.ctypes.data + b0 * bs * 4,
            None if dq is None else dq.ctypes.data + b0 * bs * 4)

    if len(ranges) == 1 or threads == 1:
        ncand = sum(run(r) for r in ranges)
    else:
        with ThreadPoolExecutor(threads) as ex:
            ncand = sum(ex.map(run, ranges))
    # the C side counts in-range candidates in the low 32 bits and full
    # evaluations in the high bits of each range's total
    n_in, n_full = ncand & 0xFFFFFFFF, ncand >> 32
    return scales, quants, dq, ((n_in, n_full) if counts else n_in)


def e4m3_snap(v: float) -> float:
    return lib().qzo_e4m3_snap(v)


def e4m3_table() -> np.ndarray:
    t = np.empty(126, np.float32)
    lib().qzo_e4m3_table(t.ctypes.data)
    return t


def ue8m0_table() -> np.ndarray:
    t = np.empty(254, np.float32)
    lib().qzo_ue8m0_table(t.ctypes.data)
    return t


def scale_codes(scales: np.ndarray, fmt: int) -> np.ndarray:
    f = lib().qzo_e4m3_code if fmt == FMT_NVFP4 else lib().qzo_ue8m0_code
    return np.array([f(float(s)) for s in scales.reshape(-1)], np.uint8)


def pack(quants: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(quants, np.float32).reshape(-1)
    out = np.empty(q.size // 2, np.uint8)
    lib().qzo_pack(q.ctypes.data, q.size, out.ctypes.data)
    return out


def unpack(packed: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(packed, np.uint8).reshape(-1)
    out = np.empty(p.size * 2, np.int8)
    lib().qzo_unpack(p.ctypes.data, p.size, out.ctypes.data)
    return out


def block_gram(X_bf16: np.ndarray, bs: int) -> np.ndarray:
    X = np.ascontiguousarray(X_bf16, np.uint16)
    T, K = X.shape
    H = np.empty((K // bs, bs, bs), np.float32)
    lib().qzo_block_gram(X.ctypes.data, T, K, bs, H.ctypes.data)
    return H


def gram(X_bf16: np.ndarray) -> np.ndarray:
    X = np.ascontiguousarray(X_bf16, np.uint16)
    T, K = X.shape
    H = np.empty((K, K), np.float32)
    lib().qzo_gram(X.ctypes.data, T, K, H.ctypes.data)
    return H


def metrics_sums(W_bf16, Wdq, X_bf16=None):
    W = np.ascontiguousarray(W_bf16, np.uint16)
    M, K = W.shape
    Wdq = np.ascontiguousarray(Wdq, np.float32)
    out = np.zeros(4, np.float64)
    T = 0 if X_bf16 is None else X_bf16.shape[0]
    Xc = None if X_bf16 is None else np.ascontiguousarray(X_bf16, np.uint16)
    lib().qzo_metrics(W.ctypes.data, Wdq.ctypes.data, M, K, _ptr(Xc), T, out.ctypes.data)
    return out


def admm(x_bf16, bs, H, Hn, Minv, n_outer=3, n_inner=10, rho=1.0):
    """nvfp4_admm's iteration given (J, bs, bs) H, H/lambda_max, M_inv."""
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1)
    n_blocks = x.size // bs
    H, Hn, Minv = (np.ascontiguousarray(t, np.float32) for t in (H, Hn, Minv))
    J = H.shape[0]
    L = lib()
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.qzo_admm.argtypes = [vp, i32, i64, i32, vp, vp, vp, i64, i32, i32, ctypes.c_float, vp, vp]
    scales = np.empty(n_blocks, np.float32)
    quants = np.empty(n_blocks * bs, np.float32)
    L.qzo_admm(x.ctypes.data, DT_BF16, n_blocks, bs, H.ctypes.data, Hn.ctypes.data, Minv.ctypes.data, J,
               n_outer, n_inner, rho, scales.ctypes.data, quants.ctypes.data)
    return scales, quants


def quantize_table(x, bs, method, table, H=None, bf16=True):
    """qzo_quantize with a caller-supplied ascending scale table."""
    x = np.ascontiguousarray(x).reshape(-1)
    n_blocks = x.size // bs
    dt = _dtype_code(x, bf16)
    t = np.ascontiguousarray(table, np.float32)
    scales = np.empty(n_blocks, np.float32)
    quants = np.empty(n_blocks * bs, np.float32)
    dq = np.empty(n_blocks * bs, np.float32)
    J = 0
    if method == M_HESSIAN:
        H = np.ascontiguousarray(H, np.float32)
        J = H.shape[0]
    L = lib()
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.qzo_quantize_table.argtypes = [vp, i32, i64, i32, i32, vp, i32, vp, i64, vp, vp, vp]
    L.qzo_quantize_table.restype = i64
    L.qzo_quantize_table(x.ctypes.data, dt, n_blocks, bs, method, t.ctypes.data, t.size, _ptr(H), J,
                         scales.ctypes.data, quants.ctypes.data, dq.ctypes.data)
    return scales, quants, dq


FMT_NVINT4, FMT_INT8 = 3, 4


def quantize_int(x, bs, fmt, method, H=None, bf16=True, threads=None):
    """qzo_quantize_int: NVINT4 (fmt 3, bs 16/32) or INT8 (fmt 4, bs 32..256),
    block ranges on a thread pool (ctypes releases the GIL)."""
    x = np.ascontiguousarray(x).reshape(-1)
    n_blocks = x.size // bs
    dt = _dtype_code(x, bf16)
    scales = np.empty(n_blocks, np.float32)
    quants = np.empty(n_blocks * bs, np.float32)
    dq = np.empty(n_blocks * bs, np.float32)
    J = 0
    if method == M_HESSIAN:
        H = np.ascontiguousarray(H, np.float32)
        J = H.shape[0]
    L = lib()
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.qzo_quantize_int.argtypes = [vp, i32, i64, i32, i32, i32, vp, i64, vp, vp, vp]
    L.qzo_quantize_int.restype = i64
    threads = threads or os.cpu_count() or 1
    esz = x.itemsize
    if method == M_HESSIAN:
        step = max(J, ((n_blocks // (threads * 8)) // J) * J or J)
    else:
        step = max(256, n_blocks // (threads * 8) + 1)
    ranges = [(b, min(n_blocks, b + step)) for b in range(0, n_blocks, step)]

    def run(r):
        b0, b1 = r
        return L.qzo_quantize_int(x.ctypes.data + b0 * bs * esz, dt, b1 - b0, bs, fmt, method, _ptr(H), J,
                                  scales.ctypes.data + b0 * 4, quants.ctypes.data + b0 * bs * 4,
                                  dq.ctypes.data + b0 * bs * 4)

    if len(ranges) == 1 or threads == 1:
        for r in ranges:
            run(r)
    else:
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(run, ranges))
    return scales, quants, dq
