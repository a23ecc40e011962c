"""qwantize_b200: B200-native (sm_100a) NVFP4 / MXFP4 / NVINT4 / INT8 block-scale quantization.

Drop-in for the public API of qwantize v0.1.2 (qwantize/__init__.py:1-13):
the same function names, keyword arguments, (..., block_size) blocked layout
and (scales, quants[, W_dq]) returns, computed by hand-written CUDA kernels
behind the C ABI in include/qwantize_b200.h.  Naive and SSE results are
bit-identical to the reference's pure-PyTorch path."""
from .core import quantize_many
from .fp4 import fp4_unpack
from .int8 import int8_dequantize, int8_naive, int8_optimal, int8_optimal_hessian, int8_quantize_packed
from .metrics import compute_metrics
from .mxfp4 import (mxfp4_dequantize, mxfp4_dequantize_packed, mxfp4_naive, mxfp4_naive_torch,
                    mxfp4_naive_triton, mxfp4_optimal, mxfp4_optimal_hessian, mxfp4_optimal_torch,
                    mxfp4_optimal_triton, mxfp4_quantize_packed)
from .nvfp4 import (nvfp4_admm, nvfp4_dequantize, nvfp4_dequantize_packed, nvfp4_naive, nvfp4_naive_triton,
                    nvfp4_optimal, nvfp4_optimal_hessian, nvfp4_optimal_hessian_triton,
                    nvfp4_optimal_triton, nvfp4_quantize_packed)
from .nvint4 import (nvint4_dequantize, nvint4_naive, nvint4_optimal, nvint4_optimal_hessian,
                     nvint4_quantize_packed)

__version__ = "0.1.0"
