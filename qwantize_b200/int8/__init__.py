"""INT8 (symmetric int codes in [-127, 127], scale = E4M3 value / 127 per
block of 32, 64, 128 or 256): the names of qwantize.int8 (int8/__init__.py of
the reference) backed by the sm_100a kernels of qz_int.cu.  Signatures,
shapes, dtypes and AssertionErrors follow int8/reference.py; results are
bit-identical to it (H-optimal: >= 99.9%)."""
from __future__ import annotations

import torch

from .. import _lib as L
from ..core import dequantize as _dequantize
from ..core import quantize_fp32 as _q
from ..core import quantize_native as _qn
from ..hessian import resolve_h_blocks as _h

__all__ = [
    "int8_naive", "int8_optimal", "int8_optimal_hessian", "int8_dequantize", "int8_quantize_packed",
    "build_fp8_e4m3_scales", "int8_quantize", "int8_dequantize_block", "compute_block_sse",
    "Q_MAX", "D_0", "VALID_BLOCK_SIZES",
]

Q_MAX = 127    # int8/reference.py:3
D_0 = 0.5      # int8/reference.py:4
VALID_BLOCK_SIZES = (32, 64, 128, 256)


def build_fp8_e4m3_scales(device="cpu"):
    """The 126 positive finite E4M3 values, ascending (int8/reference.py:18-33)."""
    return L.scale_table(L.FMT_NVFP4).to(device)


def int8_quantize(x, s):
    """``clamp(round(x / s), -127, 127)`` (int8/reference.py:36-48)."""
    return torch.clamp(torch.round(x / s), -Q_MAX, Q_MAX)


def int8_dequantize_block(quants, s):
    """``quants * s`` (int8/reference.py:51-62)."""
    return quants * s


def compute_block_sse(x, s):
    """Per-block SSE of INT8 quantization (int8/reference.py:65-83)."""
    if s.dim() == 1:
        s = s.unsqueeze(-1)
    return (x - int8_dequantize_block(int8_quantize(x, s), s)).pow(2).sum(dim=-1)


def int8_naive(W, dim=-1, return_dequant=False):
    """``s = E4M3(max|x|) / 127`` per block (int8/reference.py:86-131)."""
    return _q(W, dim, return_dequant, L.FMT_INT8, L.METHOD_NAIVE, valid=VALID_BLOCK_SIZES)


def int8_optimal(W, dim=-1, return_dequant=False):
    """Bounded exhaustive search over the scales E4M3 / 127 minimizing block SSE
    (int8/reference.py:134-233)."""
    return _q(W, dim, return_dequant, L.FMT_INT8, L.METHOD_SSE, valid=VALID_BLOCK_SIZES)


def int8_optimal_hessian(W, dim=-1, return_dequant=False, X=None, H_blocks=None):
    """Scale search minimizing (x - s q)^T H_j (x - s q) (int8/reference.py:261-372);
    H_j = X_j^T X_j on the tensor cores when only X is given."""
    H = _h(W, dim, X, H_blocks, valid=VALID_BLOCK_SIZES)
    return _q(W, dim, return_dequant, L.FMT_INT8, L.METHOD_HESSIAN, H, valid=VALID_BLOCK_SIZES)


def int8_dequantize(scales, quants, dim=-1):
    """``quants * scales.unsqueeze(dim)`` (int8/reference.py:375-389)."""
    return _dequantize(scales, quants, dim, valid=VALID_BLOCK_SIZES)


_METHODS = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE, "hessian": L.METHOD_HESSIAN}


def int8_quantize_packed(W, method="optimal", dim=-1, return_dequant=False, X=None, H_blocks=None):
    """Native storage: ``(scale_codes, int8 codes as uint8[, dq_bf16])`` -- the
    E4M3 byte of 127 * scale and one int8 per element (0x80 marks a NaN quant).
    Same scale choice as the fp32 functions."""
    H = _h(W, dim, X, H_blocks, valid=VALID_BLOCK_SIZES) if method == "hessian" else None
    return _qn(W, dim, return_dequant, L.FMT_INT8, _METHODS[method], H, valid=VALID_BLOCK_SIZES)
