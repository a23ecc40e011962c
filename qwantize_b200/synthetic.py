"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the real Qwen3-4B checkpoint and WikiText-2
activations the reference measured on are not available).

* Weights: N(0, 0.02^2) fp32, a seeded random 0.1% of entries multiplied by 20
  (heavy-tail outliers), then one cast to bf16.
* Activations: Student-t(nu=4) per element, times a per-channel lognormal(0, 1)
  scale, with 1% of channels further multiplied by 10, cast to bf16.  Generated
  in 65,536-token chunks, chunk c seeded with ``seed + c``, so a token-sharded
  run over any number of GPUs sees exactly the same rows.
"""
from __future__ import annotations

import hashlib

import torch

CHUNK_TOKENS = 65536

# Qwen3-4B linear stack: 36 layers, hidden 2560, intermediate 9728,
# 32 query heads / 8 KV heads of dim 128.  (name, out_features, in_features)
QWEN3_4B_LAYER = [
    ("q_proj", 4096, 2560), ("k_proj", 1024, 2560), ("v_proj", 1024, 2560),
    ("o_proj", 2560, 4096), ("gate_proj", 9728, 2560), ("up_proj", 9728, 2560),
    ("down_proj", 2560, 9728),
]
QWEN3_4B_LAYERS = 36

# Llama-3-70B linear stack: 80 layers, hidden 8192, intermediate 28672.
LLAMA3_70B_LAYER = [
    ("q_proj", 8192, 8192), ("k_proj", 1024, 8192), ("v_proj", 1024, 8192),
    ("o_proj", 8192, 8192), ("gate_proj", 28672, 8192), ("up_proj", 28672, 8192),
    ("down_proj", 8192, 28672),
]
LLAMA3_70B_LAYERS = 80


def make_weight(M: int, K: int, seed: int = 0, device="cpu") -> torch.Tensor:
    """bf16 (M, K) weight; identical bits for a given seed on any machine
    running the same torch build (CPU generator; moved to ``device`` after)."""
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(M, K, generator=g) * 0.02
    idx = torch.randperm(M * K, generator=g)[: (M * K) // 1000]
    w.view(-1)[idx] *= 20
    return w.to(torch.bfloat16).to(device)


def make_weight_device(M: int, K: int, seed: int, device) -> torch.Tensor:
    """Same distribution generated directly on a CUDA device (for the large
    stacks, where a CPU generator would dominate set-up time)."""
    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(M, K, generator=g, device=device) * 0.02
    n_out = (M * K) // 1000
    idx = torch.randint(0, M * K, (n_out,), generator=g, device=device)
    w.view(-1)[idx] *= 20
    return w.to(torch.bfloat16)


def layer_seed(layer: int, proj: str, base: int = 0) -> int:
    h = hashlib.sha256(f"{base}:{layer}:{proj}".encode()).digest()
    return int.from_bytes(h[:4], "little")


def channel_scales(K: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    chs = torch.exp(torch.randn(K, generator=g))
    out = torch.randperm(K, generator=g)[: K // 100]
    chs[out] *= 10
    return chs


def _student_t4(shape, g, device):
    z = torch.randn(shape, generator=g, device=device)
    v = torch.zeros(shape, device=device)
    for _ in range(4):
        e = torch.randn(shape, generator=g, device=device)
        v += e * e
    return z / torch.sqrt(v / 4.0)


def make_activations(T: int, K: int, seed: int = 1, device="cpu", t0: int = 0,
                     chunk_tokens: int = CHUNK_TOKENS) -> torch.Tensor:
    """bf16 (T, K) activation rows [t0, t0+T) of the seeded stream.  Whole
    chunks are always generated, so a row's value does not depend on the slice
    asked for (token shards of any size agree)."""
    chs = channel_scales(K, seed).to(device)
    out = torch.empty(T, K, dtype=torch.bfloat16, device=device)
    t = t0
    while t < t0 + T:
        c = t // chunk_tokens
        c0 = c * chunk_tokens
        lo, hi = t - c0, min(t0 + T - c0, chunk_tokens)
        g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + c)
        rows = _student_t4((chunk_tokens, K), g, device)[lo:hi]
        out[t - t0: t - t0 + (hi - lo)] = (rows * chs).to(torch.bfloat16)
        t += hi - lo
    return out
