"""Host side of the drop-in API: layout plumbing around the C ABI.

Mirrors the reference's wrappers (qwantize v0.1.2, e.g. nvfp4/reference.py:106-126):
``dim`` is moved last and the tensor viewed as (N, bs) blocks; outputs are
reshaped back to the reference's shapes.  All arithmetic runs in the sm_100a
kernels; a CPU tensor is copied to the current CUDA device and the results
are copied back (there is no CPU implementation).
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import _staging


def cuda_device(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("qwantize_b200 needs a CUDA (sm_100a) device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def _blocks(W: torch.Tensor, dim: int, valid=(16, 32)):
    dim = dim % W.ndim
    block_size = W.shape[dim]
    assert block_size in valid, f"block_size={block_size}, expected one of {tuple(valid)}"
    dev = cuda_device(W)
    x = W.movedim(dim, -1)
    batch_shape = x.shape[:-1]
    if x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        x = x.float()  # W.float() in the reference: float64 etc. round once to fp32
    x = (_staging.to_device(x, dev) if x.device.type == "cpu" else x.to(dev)).reshape(-1, block_size)
    if not x.is_contiguous():
        x = x.contiguous()
    if x.data_ptr() % 16:  # a view at an odd offset: the kernels load 16-byte vectors
        x = x.clone()
    return dim, block_size, batch_shape, x, dev


def quantize_fp32(W, dim, return_dequant, fmt, method, H_blocks=None, valid=(16, 32)):
    """Reference-shaped result: fp32 (scales, quants[, dq])."""
    dim, bs, batch_shape, x, dev = _blocks(W, dim, valid)
    N = x.shape[0]
    scales = torch.empty(N, dtype=torch.float32, device=dev)
    quants = torch.empty(N, bs, dtype=torch.float32, device=dev)
    dq = torch.empty(N, bs, dtype=torch.float32, device=dev) if return_dequant else None
    J = 0
    if method == L.METHOD_HESSIAN:
        J = H_blocks.shape[0]
        M_dim = N // J if J else 0
        assert N == M_dim * J
    st = L.load().qz_quantize(
        L.ptr(x), L.dtype_code(x.dtype), N, bs, fmt, method, L.ptr(H_blocks), J,
        L.ptr(scales), L.ptr(quants), L.ptr(dq), None, None, None, L.stream_ptr(dev))
    L.check(st, "qz_quantize")
    res = (scales.reshape(*batch_shape), quants.reshape(*batch_shape, bs).movedim(-1, dim))
    if return_dequant:
        res = res + (dq.reshape(*batch_shape, bs).movedim(-1, dim),)
    return to_host_like(res, W.device, dev)


def to_host_like(res, want, dev):
    """Return device results on `want`: unchanged on the GPU; for a CPU caller
    ordinary CPU tensors, copied through the library's page-locked staging
    buffers (qwantize_b200._staging) in order after the call's kernels."""
    if want.type != "cpu":
        return tuple(t.to(want) for t in res)
    return _staging.to_host(res, dev)


def quantize_native(W, dim, return_dequant, fmt, method, H_blocks=None, valid=(16, 32)):
    """Native storage: (scale_codes uint8, packed uint8 (..., bs/2 or bs)[, dq bf16]).

    scale_codes are E4M3 bytes (NVFP4, NVINT4; INT8: of 127 * scale) or UE8M0
    biased exponents (MXFP4); packed holds two 4-bit codes per byte, element 2i
    in the low nibble (INT8: one int8 per element)."""
    dim, bs, batch_shape, x, dev = _blocks(W, dim, valid)
    N = x.shape[0]
    codes = torch.empty(N, dtype=torch.uint8, device=dev)
    pw = bs if fmt == L.FMT_INT8 else bs // 2
    packed = torch.empty(N, pw, dtype=torch.uint8, device=dev)
    dq = torch.empty(N, bs, dtype=torch.bfloat16, device=dev) if return_dequant else None
    J = 0
    if method == L.METHOD_HESSIAN:
        J = H_blocks.shape[0]
        assert N % J == 0
    st = L.load().qz_quantize(
        L.ptr(x), L.dtype_code(x.dtype), N, bs, fmt, method, L.ptr(H_blocks), J,
        None, None, None, L.ptr(codes), L.ptr(packed), L.ptr(dq), L.stream_ptr(dev))
    L.check(st, "qz_quantize")
    res = (codes.reshape(*batch_shape), packed.reshape(*batch_shape, pw))
    if return_dequant:
        res = res + (dq.reshape(*batch_shape, bs).movedim(-1, dim),)
    return to_host_like(res, W.device, dev)


def dequantize(scales, quants, dim=-1, valid=(16, 32)):
    """quants * scales.unsqueeze(dim) (nvfp4/reference.py:537-549)."""
    dim = dim % quants.ndim
    bs = quants.shape[dim]
    assert bs in valid, f"block_size={bs}, expected one of {tuple(valid)}"
    dev = cuda_device(quants)
    q = quants.movedim(dim, -1).to(dev, torch.float32).contiguous()
    batch_shape = q.shape[:-1]
    s = scales.to(dev, torch.float32).reshape(-1).contiguous()
    assert s.numel() * bs == q.numel()
    out = torch.empty_like(q)
    L.check(L.load().qz_dequantize(L.ptr(s), L.ptr(q), s.numel(), bs, L.ptr(out),
                                   L.stream_ptr(dev)), "qz_dequantize")
    return to_host_like((out.reshape(*batch_shape, bs).movedim(-1, dim),), quants.device, dev)[0]


def dequantize_native(scale_codes, packed, fmt, dtype=torch.bfloat16):
    """(scale_codes (...), packed (..., bs/2)) -> dequantized (..., bs)."""
    dev = cuda_device(packed)
    bs = packed.shape[-1] * 2
    assert bs in (16, 32)
    p = packed.to(dev).contiguous()
    c = scale_codes.to(dev).contiguous()
    n_blocks = c.numel()
    out = torch.empty(*packed.shape[:-1], bs, dtype=dtype, device=dev)
    f32 = out if dtype == torch.float32 else None
    b16 = out if dtype == torch.bfloat16 else None
    assert f32 is not None or b16 is not None, "dtype must be float32 or bfloat16"
    L.check(L.load().qz_dequantize_packed(L.ptr(p), L.ptr(c), n_blocks, bs, fmt, L.ptr(f32),
                                          L.ptr(b16), L.stream_ptr(dev)), "qz_dequantize_packed")
    return to_host_like((out,), packed.device, dev)[0]


def admm_fp32(W, dim, return_dequant, H, Hn, Minv, n_outer=3, n_inner=10, rho=1.0):
    """nvfp4_admm's iteration (qz_admm) on blocks of W given the per-column-block
    H, H / lambda_max and inv(H / lambda_max + rho I)."""
    dim, bs, batch_shape, x, dev = _blocks(W, dim)
    N = x.shape[0]
    J = H.shape[0]
    M_dim = N // J if J else 0
    assert N == M_dim * J, f"Weight blocks ({N}) must equal M * K//bs ({M_dim} * {J})"
    scales = torch.empty(N, dtype=torch.float32, device=dev)
    quants = torch.empty(N, bs, dtype=torch.float32, device=dev)
    dq = torch.empty(N, bs, dtype=torch.float32, device=dev) if return_dequant else None
    H, Hn, Minv = (t.to(dev, torch.float32).contiguous() for t in (H, Hn, Minv))
    st = L.load().qz_admm(L.ptr(x), L.dtype_code(x.dtype), N, bs, L.ptr(H), L.ptr(Hn), L.ptr(Minv), J,
                          int(n_outer), int(n_inner), float(rho), L.ptr(scales), L.ptr(quants), L.ptr(dq),
                          None, None, None, L.stream_ptr(dev))
    L.check(st, "qz_admm")
    res = (scales.reshape(*batch_shape), quants.reshape(*batch_shape, bs).movedim(-1, dim))
    if return_dequant:
        res = res + (dq.reshape(*batch_shape, bs).movedim(-1, dim),)
    return to_host_like(res, W.device, dev)


def quantize_many(weights, fmt, method, block_size=16, packed=True, return_dequant=False, outputs=None):
    """Quantize a list of weights (fmt "nvfp4" / "mxfp4", method "naive" /
    "optimal"; each (..., K) with K a multiple of
    block_size, blocks along the last dimension, all of one dtype and device)
    in one grouped launch per 256 weights (qz_quantize_grouped): the chunks
    of every weight share the GPU, so many small matrices (row shards of a
    layer stack) run as one wave-filling launch.  Results are bit-identical to
    one call per weight.

    packed=True returns, per weight, (scale_codes (..., K/bs) uint8, packed
    (..., K/bs, bs/2) uint8[, dq bf16]); packed=False returns the reference's
    fp32 (scales, quants[, dq]) shaped (..., K/bs[, bs]).  ``outputs`` may
    supply preallocated tuples of the same layout (device tensors)."""
    fmt = {"nvfp4": L.FMT_NVFP4, "mxfp4": L.FMT_MXFP4}.get(fmt, fmt)
    method = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE}.get(method, method)
    assert block_size in (16, 32), f"block_size={block_size}, expected one of (16, 32)"
    assert fmt in (L.FMT_NVFP4, L.FMT_MXFP4), "grouped launches run NVFP4 and MXFP4"
    assert method in (L.METHOD_NAIVE, L.METHOD_SSE), "grouped launches run the naive and SSE methods"
    if not weights:
        return []
    dev = cuda_device(weights[0])
    dt = weights[0].dtype
    items = (L.QzQuantItem * len(weights))()
    keep, results = [], []
    for i, W in enumerate(weights):
        assert W.dtype == dt, "all weights of a grouped call share one dtype"
        assert W.shape[-1] % block_size == 0, f"last dimension {W.shape[-1]} is not a multiple of {block_size}"
        x = (_staging.to_device(W, dev) if W.device.type == "cpu" else W.to(dev).contiguous()).reshape(
            -1, block_size)
        if x.data_ptr() % 16:
            x = x.clone()
        N = x.shape[0]
        bshape = (*W.shape[:-1], W.shape[-1] // block_size)
        if outputs is not None:
            out = tuple(outputs[i])
            # the kernel writes through these pointers: layout, dtype and device must match exactly
            want = ([(bshape, torch.uint8), ((*bshape, block_size // 2), torch.uint8),
                     ((*bshape, block_size), torch.bfloat16)] if packed else
                    [(bshape, torch.float32), ((*bshape, block_size), torch.float32),
                     ((*bshape, block_size), torch.float32)])
            assert len(out) == (3 if return_dequant else 2), f"outputs[{i}]: {len(out)} tensors"
            for t, (shape, dtype) in zip(out, want):
                assert (tuple(t.shape) == tuple(shape) and t.dtype == dtype and t.device == dev
                        and t.is_contiguous()), (f"outputs[{i}]: expected a contiguous {dtype} tensor of shape "
                                                 f"{tuple(shape)} on {dev}, got {t.dtype} {tuple(t.shape)} on {t.device}")
        elif packed:
            out = (torch.empty(bshape, dtype=torch.uint8, device=dev),
                   torch.empty(*bshape, block_size // 2, dtype=torch.uint8, device=dev))
            if return_dequant:
                out = out + (torch.empty(*bshape, block_size, dtype=torch.bfloat16, device=dev),)
        else:
            out = (torch.empty(bshape, dtype=torch.float32, device=dev),
                   torch.empty(*bshape, block_size, dtype=torch.float32, device=dev))
            if return_dequant:
                out = out + (torch.empty(*bshape, block_size, dtype=torch.float32, device=dev),)
        it = items[i]
        it.x, it.n_blocks = x.data_ptr(), N
        if packed:
            it.scale_codes, it.packed = out[0].data_ptr(), out[1].data_ptr()
            it.dq_bf16 = out[2].data_ptr() if len(out) > 2 else None
        else:
            it.scales, it.quants = out[0].data_ptr(), out[1].data_ptr()
            it.dq = out[2].data_ptr() if len(out) > 2 else None
        keep.append(x)
        results.append(out)
    L.check(L.load().qz_quantize_grouped(items, len(weights), L.dtype_code(x.dtype), block_size, fmt, method,
                                         L.stream_ptr(dev)), "qz_quantize_grouped")
    if weights[0].device.type == "cpu":
        results = [_staging.to_host(r, dev) for r in results]
    elif weights[0].device != dev:
        results = [tuple(t.to(weights[0].device) for t in r) for r in results]
    return results
