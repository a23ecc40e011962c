"""Host <-> device copies for callers that pass CPU tensors to the drop-in API.

A CPU caller gets ordinary (pageable) CPU tensors back, like the reference's
functions return.  Copying straight between pageable memory and the GPU runs
at a fraction of PCIe speed, and handing back freshly page-locked tensors makes
every call that keeps its results pay the page locking (about 150-200 ms for
the 205 MB of fp32 results of one 2560 x 9728 weight).  Instead each device has
two small page-locked staging buffers owned by this module: the data moves in
chunks, the DMA of one chunk overlapping the host-side copy of the other
(torch's multi-threaded memcpy).  The copies run on the device's current
stream, so they are ordered with the kernels of the same call.
"""
from __future__ import annotations

import threading

import torch

_CHUNK = 8 << 20  # bytes per staging buffer
_lock = threading.Lock()
_state = {}       # device index -> ([two pinned uint8 buffers], [their last events])


def _buffers(dev: torch.device):
    st = _state.get(dev.index)
    if st is None:
        st = ([torch.empty(_CHUNK, dtype=torch.uint8, pin_memory=True) for _ in range(2)], [None, None])
        _state[dev.index] = st
    return st


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1).view(torch.uint8)


def to_device(x: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """Contiguous copy of the CPU tensor x on dev, issued on dev's current
    stream.  x is fully read before the call returns, so the caller may modify
    it afterwards; the device copy completes in stream order."""
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=dev)
    if x.numel() == 0:
        return out
    src, dst = _bytes(x), _bytes(out)
    stream = torch.cuda.current_stream(dev)
    with _lock:
        bufs, evs = _buffers(dev)
        for k, off in enumerate(range(0, src.numel(), _CHUNK)):
            m = min(_CHUNK, src.numel() - off)
            b = k & 1
            if evs[b] is not None:
                evs[b].synchronize()  # the buffer's previous DMA is done
            bufs[b][:m].copy_(src[off:off + m])
            dst[off:off + m].copy_(bufs[b][:m], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            evs[b] = ev
    return out


def to_host(ts, dev: torch.device):
    """Pageable, contiguous CPU copies of the device tensors ts (same shapes
    and dtypes), after all work queued on dev's current stream; returns when
    every copy is complete."""
    stream = torch.cuda.current_stream(dev)
    outs = []
    with _lock:
        bufs, evs = _buffers(dev)
        pend = [None, None]  # per buffer: (destination bytes, length) still to copy out
        k = 0

        def drain(b):
            evs[b].synchronize()
            if pend[b] is not None:
                d, m = pend[b]
                d.copy_(bufs[b][:m])
                pend[b] = None

        for t in ts:
            tc = t.contiguous()
            o = torch.empty(t.shape, dtype=t.dtype)
            if tc.numel():
                src, dst = _bytes(tc), _bytes(o)
                for off in range(0, src.numel(), _CHUNK):
                    m = min(_CHUNK, src.numel() - off)
                    b = k & 1
                    if evs[b] is not None:
                        drain(b)
                    bufs[b][:m].copy_(src[off:off + m], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(stream)
                    evs[b] = ev
                    pend[b] = (dst[off:off + m], m)
                    k += 1
            outs.append(o)
        for b in ((k & 1), (k + 1) & 1):  # the older chunk first
            if evs[b] is not None:
                drain(b)
    return tuple(outs)
