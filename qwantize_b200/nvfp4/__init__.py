"""NVFP4 (E2M1 codes, FP8-E4M3 block scales): the names of qwantize.nvfp4
(nvfp4/__init__.py:1-16 of the reference) backed by the sm_100a kernels.

Signatures, shapes, dtypes and AssertionErrors follow nvfp4/reference.py.
The ``*_triton`` names return the same bit-exact results as the reference's
pure-PyTorch functions (the reference's own Triton kernels deviate from them
at E2M1 rounding ties and use a different Hessian fast-fail rule)."""
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
    "nvfp4_naive", "nvfp4_optimal", "nvfp4_optimal_hessian", "nvfp4_admm", "nvfp4_dequantize",
    "nvfp4_naive_triton", "nvfp4_optimal_triton", "nvfp4_optimal_hessian_triton",
    "nvfp4_quantize_packed", "nvfp4_dequantize_packed", "build_fp8_e4m3_scales",
    "fp4_quantize", "fp4_dequantize", "compute_block_sse",
    "FP4_CODEBOOK", "FP4_BOUNDARIES", "Q_MAX", "D_0",
]


def build_fp8_e4m3_scales(device="cpu"):
    """The 126 positive finite E4M3 values, ascending (nvfp4/reference.py:21-34)."""
    return L.scale_table(L.FMT_NVFP4).to(device)


def nvfp4_naive(W, dim=-1, return_dequant=False):
    """``s = E4M3(max|x| / 6)`` per block (nvfp4/reference.py:89-126)."""
    return _q(W, dim, return_dequant, L.FMT_NVFP4, L.METHOD_NAIVE)


def nvfp4_optimal(W, dim=-1, return_dequant=False):
    """Bounded exhaustive search for the E4M3 scale minimizing block SSE
    (nvfp4/reference.py:129-239)."""
    return _q(W, dim, return_dequant, L.FMT_NVFP4, L.METHOD_SSE)


def nvfp4_optimal_hessian(W, dim=-1, return_dequant=False, X=None, H_blocks=None):
    """Scale search minimizing (x - sq)^T H_j (x - sq) (nvfp4/reference.py:266-407).
    H_j = X_j^T X_j is built on the tensor cores when only X is given."""
    H = _h(W, dim, X, H_blocks)
    return _q(W, dim, return_dequant, L.FMT_NVFP4, L.METHOD_HESSIAN, H)


def nvfp4_admm(W, dim=-1, return_dequant=False, X=None, n_outer=3, n_inner=10, H_blocks=None):
    """ADMM-refined NVFP4 quantization under the block Hessians of X
    (nvfp4/reference.py:410-534): from the naive scale, n_outer rounds of
    n_inner ADMM steps that project onto the E2M1 codebook, then a closed-form
    E4M3 scale update.  H_j = X_j^T X_j is built on the tensor cores
    (``H_blocks`` may be passed instead, an extension of the reference's
    signature); the iteration runs in the qz_admm kernel."""
    assert X is not None or H_blocks is not None, "X (activations) required for ADMM quantization"
    from ..core import admm_fp32
    from ..hessian import admm_setup, block_hessians
    dim_ = dim % W.ndim
    bs = W.shape[dim_]
    assert bs in (16, 32)
    if H_blocks is None:
        H = block_hessians(X, bs)
    else:
        from ..core import cuda_device
        H = H_blocks.to(cuda_device(W), torch.float32).contiguous()
    Hn, Minv = admm_setup(H, 1.0)
    return admm_fp32(W, dim, return_dequant, H, Hn, Minv, n_outer, n_inner, 1.0)


def nvfp4_dequantize(scales, quants, dim=-1):
    """``quants * scales.unsqueeze(dim)`` (nvfp4/reference.py:537-549)."""
    return _dequantize(scales, quants, dim)


def nvfp4_naive_triton(W, dim=-1, return_dequant=False):
    """Drop-in for nvfp4/kernels.py:248-293."""
    return nvfp4_naive(W, dim, return_dequant)


def nvfp4_optimal_triton(W, dim=-1, return_dequant=False):
    """Drop-in for nvfp4/kernels.py:296-351."""
    return nvfp4_optimal(W, dim, return_dequant)


def nvfp4_optimal_hessian_triton(W, dim=-1, return_dequant=False, X=None):
    """Drop-in for nvfp4/kernels.py:354-427 (X required, as there)."""
    assert X is not None, "X (activations) required for Hessian-aware scale search"
    return nvfp4_optimal_hessian(W, dim, return_dequant, X=X)


_METHODS = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE, "hessian": L.METHOD_HESSIAN}


def nvfp4_quantize_packed(W, method="optimal", dim=-1, return_dequant=False, X=None,
                          H_blocks=None):
    """Native storage in one pass: ``(scale_codes, packed[, dq_bf16])`` --
    E4M3 scale bytes, two E2M1 nibbles per byte (element 2i in the low nibble,
    bit 3 = sign: the layout ``fp4_unpack`` decodes) and an optional bf16
    dequant.  Same scale choice as the fp32 functions."""
    H = _h(W, dim, X, H_blocks) if method == "hessian" else None
    return _qn(W, dim, return_dequant, L.FMT_NVFP4, _METHODS[method], H)


def nvfp4_dequantize_packed(scale_codes, packed, dtype=torch.bfloat16):
    from ..core import dequantize_native
    return dequantize_native(scale_codes, packed, L.FMT_NVFP4, dtype)
