"""Block FP4 quantization on other 8-bit scale grids (exotic_scales.py and
experiments/quant_exotic_scales.py of the reference): the unsigned UE4M4 and
UE5M3 grids, or any ascending table of up to 256 positive scales.

The search runs in the qz_quantize_table kernel: naive scale
snap_to_table(max|x| / 6), SSE-optimal and Hessian-optimal bounded searches
over the table with the NVFP4 rules.  Results equal the reference's torch
implementation bit for bit for the naive and SSE methods."""
from __future__ import annotations

import torch

from . import _lib as L
from .core import _blocks, to_host_like

_METHOD = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE, "hoptimal": L.METHOD_HESSIAN}


def _unsigned_fp8_values(exp_bits: int, mant_bits: int) -> torch.Tensor:
    """Every positive value of an unsigned (E, M) 8-bit float, IEEE-style
    (bias 2^(E-1) - 1, subnormals at e = 0, no code reserved), ascending."""
    assert exp_bits + mant_bits == 8
    bias = 2 ** (exp_bits - 1) - 1
    vals = set()
    for e in range(2 ** exp_bits):
        for m in range(2 ** mant_bits):
            f = m / 2 ** mant_bits
            v = f * 2.0 ** (1 - bias) if e == 0 else (1.0 + f) * 2.0 ** (e - bias)
            if v > 0:
                vals.add(v)
    return torch.tensor(sorted(vals), dtype=torch.float64).float()


def build_ue4m4_scales(device="cpu"):
    """Sorted positive UE4M4 values (4 exponent, 4 mantissa bits, unsigned)."""
    return _unsigned_fp8_values(4, 4).to(device)


def build_ue5m3_scales(device="cpu"):
    """Sorted positive UE5M3 values (5 exponent, 3 mantissa bits, unsigned)."""
    return _unsigned_fp8_values(5, 3).to(device)


def snap_to_table(x, sorted_table):
    """Nearest table entry (ties to the lower one): bucketize over the
    midpoints of consecutive entries (exotic_scales.py:60-74)."""
    table = sorted_table.to(x.device).to(x.dtype)
    boundaries = (table[:-1] + table[1:]) * 0.5
    return table[torch.bucketize(x.contiguous(), boundaries)]


def quantize_table(W, table, method="optimal", dim=-1, return_dequant=False, X=None, H_blocks=None):
    """(scales, quants[, dq]) of W on the scale grid ``table`` (ascending, 2..256
    positive values), the reference's return convention."""
    meth = _METHOD[method]
    dim_, bs, batch_shape, x, dev = _blocks(W, dim)
    t = table.to(dev, torch.float32).contiguous()
    assert 2 <= t.numel() <= 256 and bool((t[1:] > t[:-1]).all()) and bool((t > 0).all())
    H = None
    J = 0
    if meth == L.METHOD_HESSIAN:
        from .hessian import resolve_h_blocks
        H = resolve_h_blocks(W, dim, X, H_blocks)
        J = H.shape[0]
    N = x.shape[0]
    scales = torch.empty(N, dtype=torch.float32, device=dev)
    quants = torch.empty(N, bs, dtype=torch.float32, device=dev)
    dq = torch.empty(N, bs, dtype=torch.float32, device=dev) if return_dequant else None
    L.check(L.load().qz_quantize_table(L.ptr(x), L.dtype_code(x.dtype), N, bs, meth, L.ptr(t), t.numel(),
                                       L.ptr(H), J, L.ptr(scales), L.ptr(quants), L.ptr(dq), None, None, None,
                                       L.stream_ptr(dev)), "qz_quantize_table")
    res = (scales.reshape(*batch_shape), quants.reshape(*batch_shape, bs).movedim(-1, dim_))
    if return_dequant:
        res = res + (dq.reshape(*batch_shape, bs).movedim(-1, dim_),)
    return to_host_like(res, W.device, dev)


# The experiment's entry points (experiments/quant_exotic_scales.py:48-182):
# W (M, K), blocks along K, returning the (M, K) dequantized weight.
def fp4_naive(W, table, block_size):
    M, K = W.shape
    return quantize_table(W.reshape(M, K // block_size, block_size), table, "naive", return_dequant=True)[2].reshape(M, K)


def fp4_optimal(W, table, block_size):
    M, K = W.shape
    return quantize_table(W.reshape(M, K // block_size, block_size), table, "optimal", return_dequant=True)[2].reshape(M, K)


def fp4_hoptimal(W, X, table, block_size):
    M, K = W.shape
    return quantize_table(W.reshape(M, K // block_size, block_size), table, "hoptimal", return_dequant=True,
                          X=X)[2].reshape(M, K)
