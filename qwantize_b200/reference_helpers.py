"""Small element helpers exported by the reference's subpackages
(nvfp4/reference.py:13-86, mxfp4/reference.py:13-86): the E2M1 constants and
``fp4_quantize`` / ``fp4_dequantize`` / ``compute_block_sse`` with arbitrary
broadcast scales.  They are conveniences for callers that use them directly;
the library's own quantization never calls them (the kernels fuse the same
arithmetic).  They use the reference's exact formulas on whatever device the
inputs live on."""
from __future__ import annotations

import torch

FP4_CODEBOOK = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
FP4_BOUNDARIES = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])
Q_MAX = 6.0
D_0 = 0.25


def fp4_quantize(x, s):
    """sign(x) * codebook[bucketize(|x| / s)] (ties to the smaller entry)."""
    b = FP4_BOUNDARIES.to(x.device)
    cb = FP4_CODEBOOK.to(x.device)
    return x.sign() * cb[torch.bucketize(x.abs() / s, b)]


def fp4_dequantize(quants, s):
    return quants * s


def compute_block_sse(x, s):
    if s.dim() == 1:
        s = s.unsqueeze(-1)
    dq = fp4_dequantize(fp4_quantize(x, s), s)
    return (x - dq).pow(2).sum(dim=-1)
