"""GPTQ error compensation on the full Hessian, with the block quantizers of
this library (the caller of the full Gram).

Follows experiments/quant_gptq_strided.py:49-135 (``gptq_strided``) and
:137-222 (``gptq_strided_ordered``) of the reference: damp the Hessian, take
the inverse through its Cholesky factor, then quantize column blocks left to
right, each block's scaled error propagated to all later columns.

B200 layout: the working weight is kept column-block-major, (K/bs, M, bs).
Rows are independent in GPTQ, so one kernel per group of ``group`` columns
carries every row through the group's blocks in shared memory (scale search --
naive, SSE-optimal or Hessian-optimal with the same arithmetic as the fp32
quantization kernels -- error, in-group update), and one tcgen05 GEMM per
group applies the group's scaled errors to every later column at fp32
accuracy (tf32 high / low operand pairs).  This is the standard lazy-batch
reordering of GPTQ's sums; results agree with the reference to floating-point
reassociation.
"""
from __future__ import annotations

import torch

from . import _lib as L
from .core import cuda_device

_FMT = {"nvfp4": L.FMT_NVFP4, "mxfp4": L.FMT_MXFP4}
_METHOD = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE, "hoptimal": L.METHOD_HESSIAN}


def spd_inverse(A: torch.Tensor) -> torch.Tensor:
    """Inverse of a symmetric positive definite fp32 matrix on the tensor cores
    (qz_spd_inverse; n a multiple of 32).  Raises torch.linalg.LinAlgError if
    a pivot is not positive, as torch.linalg.cholesky does."""
    n = A.shape[0]
    X = A.to(torch.float32).contiguous().clone()
    work = torch.empty(11 * n * n, dtype=torch.float32, device=X.device)
    status = torch.zeros(1, dtype=torch.int32, device=X.device)
    L.check(L.load().qz_spd_inverse(L.ptr(X), n, L.ptr(work), L.ptr(status), L.stream_ptr(X.device)),
            "qz_spd_inverse")
    if int(status.item()):
        raise torch.linalg.LinAlgError("the matrix is not positive definite")
    return X


def _inverse_hessian(H: torch.Tensor, damp: float) -> torch.Tensor:
    """Damped H^-1 (experiments/quant_gptq_strided.py:72-85): H + damp * mean(diag)
    I, inverted on the tensor cores when K is a multiple of 32 (through the
    Cholesky factor otherwise); a matrix that is not positive definite gets
    the reference's extra 1e-5 * dmu on the diagonal and a second attempt."""
    Hi = H.clone().float()
    dmu = damp * Hi.diagonal().mean()
    Hi.diagonal().add_(dmu)
    inv = spd_inverse if Hi.shape[0] % 32 == 0 else (lambda A: torch.cholesky_inverse(torch.linalg.cholesky(A)))
    try:
        return inv(Hi).contiguous()
    except torch.linalg.LinAlgError:
        Hi.diagonal().add_(1e-5 * dmu)
        return inv(Hi).contiguous()


def _quant_block(x: torch.Tensor, bs: int, fmt: int, method: int, H_blk, out_dq: torch.Tensor):
    """Dequantized (M, bs) block of fp32 weights through qz_quantize."""
    M = x.shape[0]
    Hp = None
    J = 0
    if method == L.METHOD_HESSIAN:
        Hp = H_blk.contiguous()
        J = 1
    L.check(L.load().qz_quantize(L.ptr(x), L.DTYPE_F32, M, bs, fmt, method, L.ptr(Hp), J, None, None,
                                 L.ptr(out_dq), None, None, None, L.stream_ptr(x.device)), "qz_quantize")
    return out_dq


def gptq(W: torch.Tensor, H: torch.Tensor, fmt: str = "nvfp4", method: str = "optimal",
         block_size: int = 16, damp: float = 0.01, group: int = 128, H_blocks: torch.Tensor = None):
    """Sequential GPTQ over column blocks (gptq_strided).

    W (M, K), H (K, K) -> (Q (M, K) fp32 dequantized, average per-row loss).
    ``H_blocks`` (K/bs, bs, bs) are the Hessians the H-optimal quantizer uses
    for each column block (default: the diagonal blocks of H).  ``group`` is
    the width in columns (32, 64 or 128) of the column groups one kernel
    carries through; the columns after a group are updated by one tensor-core
    GEMM per group (qz_gptq)."""
    bs = block_size
    assert bs in (16, 32)
    dev = cuda_device(W)
    W = W.to(dev)
    M, K = W.shape
    assert K % bs == 0 and H.shape == (K, K)
    nblk = K // bs
    group = max(bs, min(128, group))
    assert group in (32, 64, 128) and group % bs == 0, "group must be 32, 64 or 128 columns"
    fmt_c, meth_c = _FMT[fmt], _METHOD[method]
    Hd = H.to(dev, torch.float32)
    Hi = _inverse_hessian(Hd, damp)
    if meth_c == L.METHOD_HESSIAN and H_blocks is None:
        H_blocks = Hd.reshape(nblk, bs, nblk, bs).diagonal(dim1=0, dim2=2).permute(2, 0, 1)
    if H_blocks is not None:
        H_blocks = H_blocks.to(dev, torch.float32).contiguous()
    # column-block-major working copy: Wb[j] is W[:, j*bs:(j+1)*bs]
    Wb = W.float().reshape(M, nblk, bs).permute(1, 0, 2).contiguous()
    Qb = torch.empty_like(Wb)
    Hs = torch.empty(2, K, K, dtype=torch.float32, device=dev)
    E = torch.empty(M, 2 * group, dtype=torch.float32, device=dev)
    n_groups = (K + group - 1) // group
    parts = torch.zeros(n_groups * ((M + 7) // 8), dtype=torch.float64, device=dev)
    L.check(L.load().qz_gptq(L.ptr(Wb), L.ptr(Qb), L.ptr(Hi), L.ptr(Hs), L.ptr(H_blocks), M, K, bs, fmt_c,
                             meth_c, group, L.ptr(E), L.ptr(parts), L.stream_ptr(dev)), "qz_gptq")
    Q = Qb.permute(1, 0, 2).reshape(M, K)
    return Q, float(parts.sum().item()) / M


def gptq_ordered(W: torch.Tensor, H: torch.Tensor, fmt: str = "nvfp4", method: str = "optimal",
                 block_size: int = 16, damp: float = 0.01, group: int = 128):
    """GPTQ with column blocks taken in descending order of their stand-alone
    Hessian-weighted loss (gptq_strided_ordered): quantize each block alone,
    score r^T H_j r, permute W and H by blocks, run gptq, permute back."""
    bs = block_size
    dev = cuda_device(W)
    W = W.to(dev).float()
    M, K = W.shape
    nblk = K // bs
    Hd = H.to(dev, torch.float32)
    H_blocks = torch.stack([Hd[j * bs:(j + 1) * bs, j * bs:(j + 1) * bs] for j in range(nblk)]).contiguous()
    fmt_c, meth_c = _FMT[fmt], _METHOD[method]
    Wb = W.reshape(M, nblk, bs).permute(1, 0, 2).contiguous()
    losses = torch.empty(nblk, device=dev)
    tmp = torch.empty(M, bs, device=dev)
    for j in range(nblk):
        q = _quant_block(Wb[j], bs, fmt_c, meth_c, H_blocks[j], tmp)
        r = Wb[j] - q
        losses[j] = (r * (r @ H_blocks[j])).sum()
    _, blk_perm = losses.sort(descending=True)
    col_perm = (blk_perm.unsqueeze(1) * bs + torch.arange(bs, device=dev).unsqueeze(0)).reshape(-1)
    W_perm = W[:, col_perm].contiguous()
    H_perm = Hd[col_perm][:, col_perm].contiguous()
    Hb_perm = H_blocks[blk_perm].contiguous()
    Q_perm, avg_loss = gptq(W_perm, H_perm, fmt, method, bs, damp, group, H_blocks=Hb_perm)
    inv = torch.empty_like(col_perm)
    inv[col_perm] = torch.arange(K, device=dev)
    return Q_perm[:, inv], avg_loss
