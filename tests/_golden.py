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


E2M1_BOUNDARIES = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
E2M1_CODEBOOK = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)


def scales_from_codes(codes, fmt):
    """fp32 scales from one byte per block: E4M3 bytes (NVFP4) or UE8M0 biased
    exponents (MXFP4)."""
    import torch
    codes = np.ascontiguousarray(codes, np.uint8).reshape(-1)
    if fmt == 0:
        return torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    e = codes.astype(np.int64)
    return np.where(e == 0xFF, np.nan, np.ldexp(1.0, e - 127)).astype(np.float32)


def dq_e2m1(x, scales):
    """The reference's fp4_quantize * s (nvfp4/reference.py:37-69) per block:
    |x| / s in fp32, bucketize with ties to the smaller entry (NaN to the last
    bucket), sign(x) times the codebook value, times s (exact)."""
    x = np.ascontiguousarray(x, np.float32)
    s = np.asarray(scales, np.float32).reshape(x.shape[0], 1)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = np.abs(x) / s
    idx = np.where(np.isnan(y), 7, np.searchsorted(E2M1_BOUNDARIES, y, side="left"))
    return np.sign(x) * E2M1_CODEBOOK[idx] * s


def dq_int(x, scales, qmax):
    """clamp(round(x / s), -Q, Q) * s with round half to even (the integer
    grids: nvint4/reference.py:29-46, int8/reference.py:36-62)."""
    x = np.ascontiguousarray(x, np.float32)
    s = np.asarray(scales, np.float32).reshape(x.shape[0], 1)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.clip(np.rint(x / s), -qmax, qmax)
    return (q * s).astype(np.float32)


def hessian_objective(x, dq, H):
    """r^T H_b r in float64 per block, r = x - dq, with H_b = H[b] (one matrix
    per row of x).  The objective the Hessian search minimises
    (nvfp4/reference.py:242-263), evaluated exactly enough to compare two
    choices for one block."""
    r = np.asarray(x, np.float64) - np.asarray(dq, np.float64)
    return np.einsum("na,nab,nb->n", r, np.asarray(H, np.float64), r)


def hessian_parity(x, got, ref, H, grid="e2m1", min_same=0.999, rel=1e-5):
    """The H-optimal parity bar: at least min_same of the blocks pick the
    reference's choice, and every block that picks another one has an
    objective within rel (relative) of the reference choice's objective.
    `got` / `ref` are per-block scales (grid "e2m1", or the integer Q 7 / 127)
    or, with grid "dq", the dequantized blocks themselves.  Block b uses
    H[b % J].  Returns (fraction identical, number differing, worst gap)."""
    xb = np.asarray(x, np.float32)
    xb = xb.reshape(-1, xb.shape[-1]) if grid != "dq" else xb
    if grid == "dq":
        bs = H.shape[-1]
        xb = xb.reshape(-1, bs)
        g = np.asarray(got, np.float32).reshape(-1, bs)
        r = np.asarray(ref, np.float32).reshape(-1, bs)
        diff = (g.view(np.uint32) != r.view(np.uint32)).any(axis=1)
    else:
        g = np.asarray(got, np.float32).reshape(-1)
        r = np.asarray(ref, np.float32).reshape(-1)
        xb = xb.reshape(g.size, -1)
        diff = g.view(np.uint32) != r.view(np.uint32)
    same = 1.0 - diff.mean()
    worst = 0.0
    if diff.any():
        rows = np.nonzero(diff)[0]
        Hs = np.asarray(H)[rows % H.shape[0]]
        xr = xb[rows]
        if grid == "dq":
            dg, dr = g[rows], r[rows]
        elif grid == "e2m1":
            dg, dr = dq_e2m1(xr, g[rows]), dq_e2m1(xr, r[rows])
        else:
            dg, dr = dq_int(xr, g[rows], grid), dq_int(xr, r[rows], grid)
        eg, er = hessian_objective(xr, dg, Hs), hessian_objective(xr, dr, Hs)
        gap = np.abs(eg - er) / np.maximum(np.abs(er), 1e-300)
        worst = float(gap.max())
        assert worst <= rel, (f"{int(diff.sum())} differing blocks, worst relative objective gap {worst:.3g} "
                              f"at block {int(rows[gap.argmax()])}")
    assert same >= min_same, (same, int(diff.sum()))
    return same, int(diff.sum()), worst
