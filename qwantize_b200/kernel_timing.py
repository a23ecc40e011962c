"""Time one quantization launch on the synthetic 2560 x 9728 config-1 weight.

    python -m qwantize_b200.kernel_timing --fmt nvint4 --bs 16 --method optimal [--reps 20]

Calls qz_quantize through the C ABI with native outputs (scale bytes, packed
codes, bf16 dequant), inputs resident on the device, CUDA-event timed after
two warm-up launches; prints one line.  With --reps 1 it makes exactly three
launches (two warm-up, one timed), which keeps profiler captures small."""
from __future__ import annotations

import argparse

import torch

from . import _lib as L
from .synthetic import make_weight_device

FORMATS = {"nvfp4": L.FMT_NVFP4, "mxfp4": L.FMT_MXFP4, "nvint4": L.FMT_NVINT4, "int8": L.FMT_INT8}
METHODS = {"naive": L.METHOD_NAIVE, "optimal": L.METHOD_SSE}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--fmt", choices=sorted(FORMATS), default="nvfp4")
    ap.add_argument("--bs", type=int, default=16)
    ap.add_argument("--method", choices=sorted(METHODS), default="optimal")
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    M, K = 2560, 9728
    n = M * K
    W = make_weight_device(M, K, 0, dev)
    codes = torch.empty(n // a.bs, dtype=torch.uint8, device=dev)
    packed = torch.empty(n, dtype=torch.uint8, device=dev)
    dq = torch.empty(n, dtype=torch.bfloat16, device=dev)
    lib = L.load()

    def run():
        L.check(lib.qz_quantize(L.ptr(W), L.DTYPE_BF16, n // a.bs, a.bs, FORMATS[a.fmt], METHODS[a.method], None, 0,
                                None, None, None, L.ptr(codes), L.ptr(packed), L.ptr(dq), L.stream_ptr(dev)),
                "qz_quantize")

    run()
    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.reps
    print(f"{a.fmt} bs{a.bs} {a.method}: {ms:.4f} ms per launch, {n / ms / 1e6:.1f} G weights/s")


if __name__ == "__main__":
    main()
