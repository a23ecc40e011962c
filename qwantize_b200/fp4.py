"""Packed E2M1 storage (fp4.py:117-282 of the reference)."""
from __future__ import annotations

import torch

from . import _lib as L


def fp4_unpack(input_data: torch.Tensor) -> torch.Tensor:
    """Unpack FP4 nibbles from a uint8 CUDA tensor to int8 values of the doubled
    codebook {0, 1, 2, 3, 4, 6, 8, 12} with sign (fp4.py:257-282): byte i gives
    output 2i (low nibble) and 2i+1 (high nibble)."""
    assert input_data.dtype == torch.uint8
    assert input_data.is_cuda
    n_bytes = input_data.numel()
    assert n_bytes % 4 == 0, "Input size must be a multiple of 4 bytes"
    inp = input_data.contiguous()
    out = torch.empty(n_bytes * 2, dtype=torch.int8, device=inp.device)
    L.check(L.load().qz_fp4_unpack(L.ptr(inp), n_bytes, L.ptr(out), L.stream_ptr(inp.device)),
            "qz_fp4_unpack")
    return out
