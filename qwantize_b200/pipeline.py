"""Quantize weights that live in host memory, overlapping the PCIe copies with
the kernels.

``quantize_host_batch`` takes host (ideally pinned) bf16 weights and returns
the native outputs -- scale bytes, packed E2M1 codes and optionally the bf16
dequant -- in host memory.  Items rotate over a few CUDA streams, each with its
own device buffers, so the host->device copy of one weight, the quantization
of another and the device->host copy of a third run at the same time.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import _lib as L

_FMT = {"nvfp4": L.FMT_NVFP4, "mxfp4": L.FMT_MXFP4}
_METHOD = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE}


class HostBatchQuantizer:
    """Reusable device buffers and streams for quantizing host weights of up to
    ``max_numel`` elements each."""

    def __init__(self, max_numel: int, device=None, slots: int = 3, with_dequant: bool = True):
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.slots = []
        for _ in range(slots):
            self.slots.append({
                "stream": torch.cuda.Stream(self.device),
                "x": torch.empty(max_numel, dtype=torch.bfloat16, device=self.device),
                "codes": torch.empty(max_numel // 16, dtype=torch.uint8, device=self.device),
                "packed": torch.empty(max_numel // 2, dtype=torch.uint8, device=self.device),
                "dq": torch.empty(max_numel, dtype=torch.bfloat16, device=self.device) if with_dequant else None,
                "done": None,
            })
        self.max_numel = max_numel

    def run(self, weights: Sequence[torch.Tensor], fmt: str = "nvfp4", method: str = "optimal",
            block_size: int = 16, outputs: Optional[List[tuple]] = None, return_dequant: bool = True):
        """Quantize every host tensor in ``weights`` (bf16, numel divisible by
        block_size, blocks along the last axis).  Returns a list of host tuples
        (scale_codes, packed[, dq_bf16]); pass ``outputs`` (pinned tensors of
        the right sizes) to reuse buffers."""
        return self.run_items([(w, fmt, method, block_size) for w in weights], outputs, return_dequant)

    def run_items(self, items, outputs: Optional[List[tuple]] = None, return_dequant: bool = True):
        """Like run(), with a (weight, fmt, method, block_size) spec per item."""
        lib = L.load()
        if return_dequant and self.slots[0]["dq"] is None:
            raise ValueError("return_dequant=True needs a HostBatchQuantizer built with with_dequant=True")
        res = []
        for i, (w, fmt, method, block_size) in enumerate(items):
            assert block_size in (16, 32)
            assert w.dtype == torch.bfloat16 and w.numel() % block_size == 0
            n = w.numel()
            assert n <= self.max_numel
            slot = self.slots[i % len(self.slots)]
            st = slot["stream"]
            if outputs is not None:
                out = outputs[i]
            else:
                out = (torch.empty(n // block_size, dtype=torch.uint8, pin_memory=True),
                       torch.empty(n // 2, dtype=torch.uint8, pin_memory=True))
                if return_dequant:
                    out = out + (torch.empty(n, dtype=torch.bfloat16, pin_memory=True),)
            with torch.cuda.stream(st):
                if slot["done"] is not None:
                    st.wait_event(slot["done"])  # the previous item of this slot is done
                x = slot["x"][:n]
                x.copy_(w.reshape(-1), non_blocking=True)
                dq = slot["dq"][:n] if return_dequant else None
                L.check(lib.qz_quantize(
                    L.ptr(x), L.DTYPE_BF16, n // block_size, block_size, _FMT[fmt], _METHOD[method],
                    None, 0, None, None, None, L.ptr(slot["codes"]), L.ptr(slot["packed"]), L.ptr(dq),
                    L.ctypes.c_void_p(st.cuda_stream)), "qz_quantize")
                out[0].copy_(slot["codes"][: n // block_size], non_blocking=True)
                out[1].copy_(slot["packed"][: n // 2], non_blocking=True)
                if dq is not None:
                    out[2].copy_(dq, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(st)
                slot["done"] = ev
            res.append(out)
        for s in self.slots:
            if s["done"] is not None:
                s["done"].synchronize()
        return res


def quantize_host_batch(weights, fmt="nvfp4", method="optimal", block_size=16, return_dequant=True):
    """One-shot helper around HostBatchQuantizer."""
    q = HostBatchQuantizer(max(w.numel() for w in weights), with_dequant=return_dequant)
    return q.run(weights, fmt, method, block_size, return_dequant=return_dequant)
