"""compute_metrics (metrics.py:4-52 of the reference).

Weight error: one HBM pass with double accumulation.  Output error: the
tcgen05 GEMM of X against W and W_dq with the squared-difference reduction
fused into its epilogue (the T x M products are never stored)."""
from __future__ import annotations

import torch

from . import _lib as L
from .core import cuda_device


def _dev(t, dev, dtype=None):
    t = t.to(dev) if dtype is None else t.to(dev, dtype)
    return t.contiguous()


def weight_error_sums(W, W_dq) -> torch.Tensor:
    dev = cuda_device(W)
    Wd, Qd = _dev(W, dev), _dev(W_dq, dev)
    if Wd.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        Wd = Wd.float()
    if Qd.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        Qd = Qd.float()
    assert Wd.numel() == Qd.numel()
    sums = torch.zeros(2, dtype=torch.float64, device=dev)
    L.check(L.load().qz_weight_error_sums(L.ptr(Wd), L.dtype_code(Wd.dtype), L.ptr(Qd),
                                          L.dtype_code(Qd.dtype), Wd.numel(), L.ptr(sums),
                                          L.stream_ptr(dev)), "qz_weight_error_sums")
    return sums


def output_error_sums(W, W_dq, X) -> torch.Tensor:
    """[sum (X W_dq^T - X W^T)^2, sum (X W^T)^2] in double.  W and W_dq must be
    exactly representable in bf16 (true for any weight given in bf16 and for
    every dequant this library produces)."""
    dev = cuda_device(W)
    M, K = W.shape[0], W.shape[-1]
    Wb = _dev(W.reshape(M, K), dev, torch.bfloat16)
    Qb = _dev(W_dq.reshape(M, K), dev, torch.bfloat16)
    Xb = _dev(X, dev, torch.bfloat16)
    assert Xb.shape[1] == K
    sums = torch.zeros(2, dtype=torch.float64, device=dev)
    L.check(L.load().qz_output_error_sums(L.ptr(Xb), Xb.shape[0], K, L.ptr(Wb), L.ptr(Qb), M,
                                          L.ptr(sums), L.stream_ptr(dev)), "qz_output_error_sums")
    return sums


def compute_metrics(W, W_dq, X=None):
    """Weight and output quantization error (metrics.py:4-52):
    weight_error = ||W_dq - W||_F, weight_error_pct = 100 ||W_dq - W|| / ||W||,
    and with X: output_error = ||X W_dq^T - X W^T||_F, output_error_pct."""
    metrics = {}
    ws = weight_error_sums(W, W_dq).cpu()
    w_err, w_norm = float(ws[0]) ** 0.5, float(ws[1]) ** 0.5
    metrics["weight_error"] = w_err
    metrics["weight_error_pct"] = w_err / w_norm * 100
    if X is not None:
        os_ = output_error_sums(W, W_dq, X).cpu()
        out_err, out_norm = float(os_[0]) ** 0.5, float(os_[1]) ** 0.5
        metrics["output_error"] = out_err
        metrics["output_error_pct"] = out_err / out_norm * 100
    return metrics
