"""Helpers for loading the committed golden fixtures (tests/golden)."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

QUANT_FUNCS = [
    ("nvfp4_naive", 0, 0), ("nvfp4_optimal", 0, 1),
    ("mxfp4_naive", 1, 0), ("mxfp4_optimal", 1, 1),
    ("mxfp4_naive_torch", 1, 3), ("mxfp4_optimal_torch", 1, 4),
]


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def digests():
    with open(os.path.join(GOLDEN, "digests.json")) as f:
        return json.load(f)


def same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32).reshape(-1).view(np.uint32)
    b = np.ascontiguousarray(b, np.float32).reshape(-1).view(np.uint32)
    return a.shape == b.shape and bool((a == b).all())


def n_diff_bits(a, b):
    a = np.ascontiguousarray(a, np.float32).reshape(-1).view(np.uint32)
    b = np.ascontiguousarray(b, np.float32).reshape(-1).view(np.uint32)
    return int((a != b).sum())


def ref_admm_matrices(X, bs):
    """H (the reference's fp32 addmm build, nvfp4/reference.py:456-464), H/lambda_max
    and inv(H/lambda_max + I) as the reference computes them on the CPU (:466-475)."""
    import torch
    K = X.shape[1]
    J = K // bs
    H = torch.empty(J, bs, bs)
    for j in range(J):
        acc = torch.zeros(bs, bs)
        for t0 in range(0, X.shape[0], 8192):
            Xj = X[t0:t0 + 8192, j * bs:(j + 1) * bs].float()
            acc.addmm_(Xj.T, Xj)
        H[j] = acc
    ev = torch.linalg.eigvalsh(H)
    Hn = H / ev[:, -1].clamp(min=1e-6).reshape(-1, 1, 1)
    Minv = torch.linalg.inv(Hn + torch.eye(bs).unsqueeze(0))
    return H, Hn, Minv
