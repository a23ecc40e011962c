"""Block Hessians H_j = X_j^T X_j for the Hessian-weighted scale search.

Replaces the reference's Python double loop of fp32 ``addmm_`` calls
(nvfp4/reference.py:304-317) with the tcgen05 Gram kernel (qz_gram)."""
from __future__ import annotations

import torch

from . import _lib as L
from .core import cuda_device


def gram(X: torch.Tensor, mode: str = "full", block_size: int = 16, out: torch.Tensor = None,
         accumulate: bool = False) -> torch.Tensor:
    """H = X^T X in fp32 for bf16 X (T, K).  mode "full" -> (K, K);
    "blockdiag" -> (K/bs, bs, bs); "upper_tiles" -> the 256 x 256 tiles on and
    above the diagonal, packed (t(t+1)/2, 256, 256), t = ceil(K / 256), each
    tile column-major (expand with unpack_upper_tiles)."""
    assert X.ndim == 2
    dev = cuda_device(X)
    Xd = X.to(dev, torch.bfloat16).contiguous()
    T, K = Xd.shape
    m = {"full": L.GRAM_FULL, "blockdiag": L.GRAM_BLOCKDIAG, "upper_tiles": L.GRAM_FULL_UPPER_TILES}[mode]
    if m == L.GRAM_BLOCKDIAG and block_size > 128:
        # blocks wider than one 128-column diagonal tile: the full Gram of each
        # contiguous column slice
        assert K % block_size == 0
        J = K // block_size
        if out is None:
            out = torch.empty((J, block_size, block_size), dtype=torch.float32, device=dev)
            accumulate = False
        for j in range(J):
            xs = Xd[:, j * block_size:(j + 1) * block_size].contiguous()
            L.check(L.load().qz_gram(L.ptr(xs), T, block_size, L.GRAM_FULL, block_size, int(accumulate),
                                     L.ptr(out[j]), L.stream_ptr(dev)), "qz_gram")
        return out
    if m == L.GRAM_BLOCKDIAG:
        assert K % block_size == 0
        shape = (K // block_size, block_size, block_size)
    elif m == L.GRAM_FULL_UPPER_TILES:
        t = (K + 255) // 256
        shape = (t * (t + 1) // 2, 256, 256)
    else:
        shape = (K, K)
    if out is None:
        out = torch.empty(shape, dtype=torch.float32, device=dev)
        accumulate = False
    assert tuple(out.shape) == shape and out.dtype == torch.float32 and out.is_contiguous()
    L.check(L.load().qz_gram(L.ptr(Xd), T, K, m, block_size, int(accumulate), L.ptr(out),
                             L.stream_ptr(dev)), "qz_gram")
    return out


def unpack_upper_tiles(packed: torch.Tensor, K: int, out: torch.Tensor = None) -> torch.Tensor:
    """The symmetric (K, K) H from gram(X, "upper_tiles") (qz_gram_unpack)."""
    dev = cuda_device(packed)
    t = (K + 255) // 256
    assert tuple(packed.shape) == (t * (t + 1) // 2, 256, 256) and packed.is_contiguous()
    if out is None:
        out = torch.empty((K, K), dtype=torch.float32, device=dev)
    assert tuple(out.shape) == (K, K) and out.dtype == torch.float32 and out.is_contiguous()
    L.check(L.load().qz_gram_unpack(L.ptr(packed), K, L.ptr(out), L.stream_ptr(dev)), "qz_gram_unpack")
    return out


def block_hessians(X: torch.Tensor, block_size: int) -> torch.Tensor:
    return gram(X, "blockdiag", block_size)


def resolve_h_blocks(W: torch.Tensor, dim: int, X, H_blocks, valid=(16, 32)) -> torch.Tensor:
    """The (J, bs, bs) fp32 device tensor the search uses: H_blocks if given
    (X is then ignored, as in the reference), else built from X."""
    assert X is not None or H_blocks is not None, "X or H_blocks required"
    bs = W.shape[dim % W.ndim]
    assert bs in valid, f"block_size={bs}, expected one of {tuple(valid)}"
    dev = cuda_device(W)
    if H_blocks is not None:
        return H_blocks.to(dev, torch.float32).contiguous()
    return block_hessians(X, bs)


def admm_setup(H: torch.Tensor, rho: float = 1.0):
    """The per-column-block matrices of nvfp4_admm (nvfp4/reference.py:466-475):
    H_norm = H / max(lambda_max(H), 1e-6) and M_inv = inv(H_norm + rho I), from
    batched bs x bs symmetric eigenvalue and inverse routines on the device."""
    bs = H.shape[-1]
    ev = torch.linalg.eigvalsh(H)
    max_eig = ev[:, -1].clamp(min=1e-6)
    Hn = H / max_eig.reshape(-1, 1, 1)
    eye = torch.eye(bs, device=H.device, dtype=H.dtype).unsqueeze(0)
    Minv = torch.linalg.inv(Hn + rho * eye)
    return Hn.contiguous(), Minv.contiguous()
