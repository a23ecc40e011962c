"""NVINT4 (symmetric int codes in [-7, 7], FP8-E4M3 block scales): the names of
qwantize.nvint4 (nvint4/__init__.py of the reference) backed by the sm_100a
kernels of qz_int.cu.  Signatures, shapes, dtypes and AssertionErrors follow
nvint4/reference.py; results are bit-identical to it (H-optimal: >= 99.9%)."""
from __future__ import annotations

import torch

from .. import _lib as L
from ..core import dequantize as _dequantize
from ..core import quantize_fp32 as _q
from ..core import quantize_native as _qn
from ..hessian import resolve_h_blocks as _h

__all__ = [
    "nvint4_naive", "nvint4_optimal", "nvint4_optimal_hessian", "nvint4_dequantize", "nvint4_quantize_packed",
    "build_fp8_e4m3_scales", "int4_quantize", "int4_dequantize_block", "compute_block_sse",
    "Q_MAX", "D_0", "VALID_BLOCK_SIZES",
]

Q_MAX = 7      # nvint4/reference.py:4
D_0 = 0.5      # nvint4/reference.py:5
VALID_BLOCK_SIZES = (16, 32)


def build_fp8_e4m3_scales(device="cpu"):
    """The 126 positive finite E4M3 values, ascending (nvint4/reference.py:19-26)."""
    return L.scale_table(L.FMT_NVINT4).to(device)


def int4_quantize(x, s):
    """``clamp(round(x / s), -7, 7)`` (nvint4/reference.py:29-41)."""
    return torch.clamp(torch.round(x / s), -Q_MAX, Q_MAX)


def int4_dequantize_block(quants, s):
    """``quants * s`` (nvint4/reference.py:44-46)."""
    return quants * s


def compute_block_sse(x, s):
    """Per-block SSE of INT4 quantization (nvint4/reference.py:49-56)."""
    if s.dim() == 1:
        s = s.unsqueeze(-1)
    return (x - int4_dequantize_block(int4_quantize(x, s), s)).pow(2).sum(dim=-1)


def nvint4_naive(W, dim=-1, return_dequant=False):
    """``s = E4M3(max|x| / 7)`` per block (nvint4/reference.py:59-95)."""
    return _q(W, dim, return_dequant, L.FMT_NVINT4, L.METHOD_NAIVE, valid=VALID_BLOCK_SIZES)


def nvint4_optimal(W, dim=-1, return_dequant=False):
    """Bounded exhaustive search over E4M3 scales minimizing block SSE
    (nvint4/reference.py:97-183)."""
    return _q(W, dim, return_dequant, L.FMT_NVINT4, L.METHOD_SSE, valid=VALID_BLOCK_SIZES)


def nvint4_optimal_hessian(W, dim=-1, return_dequant=False, X=None, H_blocks=None):
    """Scale search minimizing (x - s q)^T H_j (x - s q) (nvint4/reference.py:194-306);
    H_j = X_j^T X_j on the tensor cores when only X is given."""
    H = _h(W, dim, X, H_blocks, valid=VALID_BLOCK_SIZES)
    return _q(W, dim, return_dequant, L.FMT_NVINT4, L.METHOD_HESSIAN, H, valid=VALID_BLOCK_SIZES)


def nvint4_dequantize(scales, quants, dim=-1):
    """``quants * scales.unsqueeze(dim)`` (nvint4/reference.py:309-311)."""
    return _dequantize(scales, quants, dim, valid=VALID_BLOCK_SIZES)


_METHODS = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE, "hessian": L.METHOD_HESSIAN}


def nvint4_quantize_packed(W, method="optimal", dim=-1, return_dequant=False, X=None, H_blocks=None):
    """Native storage: ``(scale_codes, packed[, dq_bf16])`` -- E4M3 scale bytes
    and two's complement int4 nibbles, element 2i in the low nibble of byte i
    (0x8 marks a NaN quant).  Same scale choice as the fp32 functions."""
    H = _h(W, dim, X, H_blocks, valid=VALID_BLOCK_SIZES) if method == "hessian" else None
    return _qn(W, dim, return_dequant, L.FMT_NVINT4, _METHODS[method], H, valid=VALID_BLOCK_SIZES)
