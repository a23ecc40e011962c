"""Multi-GPU execution of the quantization path, one process per GPU.

* Weight quantization shards **rows**: blocks are independent, so every rank
  quantizes a contiguous share of the rows of W (the leading axis that is not
  the block axis) and no collective is needed on the data path.  Gathering the
  shards onto every rank is optional and separate.
* The Hessian shards **tokens**: each rank builds the Gram of its own rows of X
  (whole 65,536-token chunks of the seeded stream, so the split does not change
  the data), then one all-reduce (sum, fp32) over the full H or only its block
  diagonal.
* compute_metrics shards tokens the same way and all-reduces four doubles.

The compute steps are the sm_100a kernels by default; the ``compute`` /
``gram_fn`` arguments let the host logic run under a CPU process group in tests.
"""
from __future__ import annotations

import datetime
import os
from typing import Callable, Optional

import torch
import torch.distributed as dist


def init(backend: str = "nccl", timeout_s: float = 120.0):
    """Join the process group described by the torchrun environment (RANK,
    WORLD_SIZE, MASTER_ADDR, MASTER_PORT, LOCAL_RANK) with a bounded timeout, so
    a rank that dies or never arrives turns into an error on the others instead
    of a hang.  Returns (rank, world_size, local_rank)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local


def _group_info(group):
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_range(n: int, world: int, rank: int):
    """Contiguous, balanced [start, stop) of n items for `rank` of `world`
    (the first n % world ranks take one more)."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def token_chunks(T: int, world: int, rank: int, chunk: int = 65536):
    """Token range [start, stop) of `rank`: whole `chunk`-token chunks dealt
    out contiguously (the last chunk may be short)."""
    n_chunks = (T + chunk - 1) // chunk
    c0, c1 = shard_range(n_chunks, world, rank)
    return min(T, c0 * chunk), min(T, c1 * chunk)


def _row_axis(W: torch.Tensor, dim: int) -> int:
    dim = dim % W.ndim
    return 1 if dim == 0 else 0


def quantize_sharded(fn: Callable, W: torch.Tensor, dim: int = -1, return_dequant: bool = False,
                     group=None, gather: bool = False, **kw):
    """Quantize this rank's share of the rows of W with ``fn`` (any of the
    drop-in functions, e.g. ``nvfp4_optimal``).  Returns ``(row_range, result)``
    where result is fn's tuple for the local rows; with ``gather=True`` the
    tuple is all-gathered into full-size tensors on every rank instead."""
    rank, world = _group_info(group)
    ax = _row_axis(W, dim)
    r0, r1 = shard_range(W.shape[ax], world, rank)
    local = W.narrow(ax, r0, r1 - r0)
    res = fn(local, dim=dim, return_dequant=return_dequant, **kw)
    if not gather or world == 1:
        return (r0, r1), res
    full = []
    counts = [shard_range(W.shape[ax], world, r) for r in range(world)]
    max_rows = max(b - a for a, b in counts)
    bdim = dim % W.ndim
    for t in res:
        # quants / dequant keep W's axes; scales drop the block axis
        t_ax = ax if t.ndim == W.ndim else (ax if ax < bdim else ax - 1)
        pad_shape = list(t.shape)
        pad_shape[t_ax] = max_rows
        padded = torch.zeros(pad_shape, dtype=t.dtype, device=t.device)
        padded.narrow(t_ax, 0, t.shape[t_ax]).copy_(t)
        bufs = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(bufs, padded, group=group)
        full.append(torch.cat([b.narrow(t_ax, 0, c1 - c0) for b, (c0, c1) in zip(bufs, counts)], dim=t_ax))
    return (0, W.shape[ax]), tuple(full)


def gram_sharded(X_local: torch.Tensor, mode: str = "full", block_size: int = 16, group=None,
                 gram_fn: Optional[Callable] = None, unpack_fn: Optional[Callable] = None) -> torch.Tensor:
    """H = X^T X over the tokens of all ranks: the local Gram of this rank's
    rows, then one all-reduce (sum, fp32).  mode "full" -> (K, K),
    "blockdiag" -> (K/bs, bs, bs).  For "full" over several ranks the ranks
    reduce only the 256 x 256 tiles on and above the diagonal (gram mode
    "upper_tiles", about half of H's bytes over NVLink) and expand the sum
    with unpack_fn(packed, K); the sums are the same, bit for bit."""
    if gram_fn is None:
        from .hessian import gram as gram_fn, unpack_upper_tiles
        unpack_fn = unpack_fn or unpack_upper_tiles
    _, world = _group_info(group)
    if mode == "full" and world > 1 and unpack_fn is not None:
        P = gram_fn(X_local, "upper_tiles", block_size)
        dist.all_reduce(P, op=dist.ReduceOp.SUM, group=group)
        return unpack_fn(P, X_local.shape[1])
    H = gram_fn(X_local, mode, block_size)
    if world > 1:
        dist.all_reduce(H, op=dist.ReduceOp.SUM, group=group)
    return H


def hessian_search_sharded(fn: Callable, W: torch.Tensor, X_local: torch.Tensor, group=None,
                           return_dequant: bool = False, gram_fn: Optional[Callable] = None):
    """H-optimal quantization across ranks: each rank builds the block
    Hessians of its own tokens (block-diagonal Gram), one all-reduce (sum,
    fp32) gives every rank the full H_j, then each rank searches only its
    share of W's rows (no further collective).  ``fn`` is a drop-in Hessian
    function (``nvfp4_optimal_hessian`` ...) taking ``H_blocks=``; W is
    (M, K/bs, bs) with the block dimension last.  Returns ``(row_range,
    result)`` as ``quantize_sharded`` does."""
    bs = W.shape[-1]
    H = gram_sharded(X_local, "blockdiag", bs, group=group, gram_fn=gram_fn)
    return quantize_sharded(fn, W, dim=-1, return_dequant=return_dequant, group=group, H_blocks=H)


def compute_metrics_sharded(W, W_dq, X_local=None, group=None, sums_fn: Optional[Callable] = None):
    """compute_metrics with the tokens of X sharded over ranks: the output-error
    sums of the local rows are all-reduced (double); the weight error is
    computed on every rank (it does not depend on X)."""
    if sums_fn is None:
        from .metrics import output_error_sums, weight_error_sums

        def sums_fn(W, W_dq, X):
            w = weight_error_sums(W, W_dq)
            o = output_error_sums(W, W_dq, X) if X is not None and X.shape[0] else torch.zeros_like(w)
            return torch.cat([w, o])
    s = sums_fn(W, W_dq, X_local)
    _, world = _group_info(group)
    if world > 1:
        w_part = s[:2].clone()
        dist.all_reduce(s, op=dist.ReduceOp.SUM, group=group)
        s[:2] = w_part  # weight sums are identical on every rank
    s = s.double().cpu()
    m = {"weight_error": float(s[0]) ** 0.5,
         "weight_error_pct": (float(s[0]) ** 0.5) / (float(s[1]) ** 0.5) * 100}
    if X_local is not None:
        m["output_error"] = float(s[2]) ** 0.5
        m["output_error_pct"] = (float(s[2]) ** 0.5) / (float(s[3]) ** 0.5) * 100
    return m
