"""MXFP4 (E2M1 codes, UE8M0 power-of-two block scales): the names of
qwantize.mxfp4 (mxfp4/__init__.py:1-21 of the reference) backed by the sm_100a
kernels.  Signatures, shapes and dtypes follow mxfp4/reference.py and
mxfp4/kernels.py.

``mxfp4_optimal_hessian`` implements the algorithm the reference's function
describes; the shipped one raises NameError (``M_dim`` undefined,
mxfp4/reference.py:301) and writes only the last block Hessian (:284).
``mxfp4_optimal_triton`` returns the full bounded search's result (the
reference's ``mxfp4_optimal``); ``mxfp4_*_torch`` reproduce the reference's
argmin-over-codebook variants bit for bit (including their +0.0 for
negative values that round to zero)."""
from __future__ import annotations

import torch

from .. import _lib as L
from ..core import dequantize as _dequantize
from ..core import quantize_fp32 as _q
from ..core import quantize_native as _qn
from ..hessian import resolve_h_blocks as _h
from ..reference_helpers import (D_0, FP4_BOUNDARIES, FP4_CODEBOOK, Q_MAX, compute_block_sse,
                                 fp4_dequantize, fp4_quantize)

__all__ = [
    "mxfp4_naive", "mxfp4_optimal", "mxfp4_optimal_hessian", "mxfp4_dequantize",
    "mxfp4_naive_triton", "mxfp4_optimal_triton", "mxfp4_naive_torch", "mxfp4_optimal_torch",
    "mxfp4_quantize_packed", "mxfp4_dequantize_packed", "build_ue8m0_scales",
    "scales_to_ue8m0_exponent", "fp4_quantize", "fp4_dequantize", "compute_block_sse",
    "FP4_CODEBOOK", "FP4_BOUNDARIES", "Q_MAX", "D_0",
]


def build_ue8m0_scales(device="cpu"):
    """2^(e-127), e = 1..254 (mxfp4/reference.py:21-34)."""
    return L.scale_table(L.FMT_MXFP4).to(device)


def scales_to_ue8m0_exponent(scales_f32):
    """round(log2(scale) + 127) as int32 (mxfp4/reference.py:392-403)."""
    safe = scales_f32.clamp(min=1e-30)
    return (safe.log2() + 127.0).round().to(torch.int32)


def mxfp4_naive(W, dim=-1, return_dequant=False):
    """``s = 2^(floor(log2 amax) - 2)`` per block (mxfp4/reference.py:89-129)."""
    return _q(W, dim, return_dequant, L.FMT_MXFP4, L.METHOD_NAIVE)


def mxfp4_optimal(W, dim=-1, return_dequant=False):
    """Bounded search over the 254 UE8M0 scales (mxfp4/reference.py:132-238)."""
    return _q(W, dim, return_dequant, L.FMT_MXFP4, L.METHOD_SSE)


def mxfp4_optimal_hessian(W, dim=-1, return_dequant=False, X=None, H_blocks=None):
    """Hessian-weighted UE8M0 search (mxfp4/reference.py:241-374, repaired)."""
    H = _h(W, dim, X, H_blocks)
    return _q(W, dim, return_dequant, L.FMT_MXFP4, L.METHOD_HESSIAN, H)


def mxfp4_dequantize(scales, quants, dim=-1):
    """``quants * scales.unsqueeze(dim)`` (mxfp4/reference.py:377-389)."""
    return _dequantize(scales, quants, dim)


def mxfp4_naive_triton(W, dim=-1, return_dequant=False):
    """Drop-in for mxfp4/kernels.py:164-208."""
    return mxfp4_naive(W, dim, return_dequant)


def mxfp4_optimal_triton(W, dim=-1, return_dequant=False):
    """Drop-in for mxfp4/kernels.py:211-259 (returns the full bounded search)."""
    return mxfp4_optimal(W, dim, return_dequant)


def mxfp4_naive_torch(W, dim=-1, return_dequant=False):
    """mxfp4/kernels.py:267-314: naive scale, nearest signed-codebook entry."""
    return _q(W, dim, return_dequant, L.FMT_MXFP4, L.METHOD_NAIVE_ARGMIN)


def mxfp4_optimal_torch(W, dim=-1, return_dequant=False):
    """mxfp4/kernels.py:317-377: the better of s0 and 2*s0 (strict '<')."""
    return _q(W, dim, return_dequant, L.FMT_MXFP4, L.METHOD_TWO_ARGMIN)


_METHODS = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE, "hessian": L.METHOD_HESSIAN}


def mxfp4_quantize_packed(W, method="optimal", dim=-1, return_dequant=False, X=None,
                          H_blocks=None):
    """Native storage in one pass: ``(ue8m0_exponents, packed[, dq_bf16])``."""
    H = _h(W, dim, X, H_blocks) if method == "hessian" else None
    return _qn(W, dim, return_dequant, L.FMT_MXFP4, _METHODS[method], H)


def mxfp4_dequantize_packed(scale_codes, packed, dtype=torch.bfloat16):
    from ..core import dequantize_native
    return dequantize_native(scale_codes, packed, L.FMT_MXFP4, dtype)
