"""Generate the golden fixtures under tests/golden by running the reference
package (qwantize v0.1.2, pure-PyTorch CPU path) on seeded inputs.

Run in a container that has the reference checked out:

    python tests/golden/make_golden.py /path/to/qwantize

Outputs (all small; large cases are stored as SHA-256 digests):
  quant_small.npz      small seeded weight + hand-made edge blocks, every
                       naive / optimal / *_torch function, bs 16 and 32
  digests.json         SHA-256 of scales/quants/dq bytes for the full
                       2560x9728 config-0/1 weight (seed 0), every function
  hessian_small.npz    H-optimal NVFP4 (X path and H_blocks path) and MXFP4
                       (the shipped function with its two bugs fixed, see
                       below) on a seeded weight and seeded activations
  metrics_small.npz    compute_metrics on seeded W / W_dq / X
  unpack_lut.npz       fp4_unpack's decode table read from fp4.py's source
                       (the Triton kernel needs a GPU, so it is read as text)
  int_small.npz        NVINT4 (bs 16/32) and INT8 (bs 32..256) naive / optimal
                       on the small weight, the edge blocks and exact INT4
                       round-half-even ties; H-optimal with X and with H_blocks

``--only int`` regenerates int_small.npz alone; ``--only int-digests`` writes
int_digests.json (SHA-256 of the NVINT4 / INT8 outputs on the full config-0/1
weight); ``--only tail`` writes tail_small.npz (ragged block counts, every
function); ``--only hessian-config2`` writes hessian_config2.npz: the reference's
H-optimal scale choices (NVFP4 and the repaired MXFP4, blocks of 16 and 32) on
the full 2560x9728 config weight, with the block Hessians they were given.

The reference checkout is a required argument (the script never guesses a
path).
"""
from __future__ import annotations

import hashlib
import inspect
import json
import os
import re
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))
from qwantize_b200.synthetic import make_activations, make_weight  # noqa: E402

QUANT_FUNCS = [  # (name, fmt, method code used by the oracle / library)
    ("nvfp4_naive", 0, 0), ("nvfp4_optimal", 0, 1),
    ("mxfp4_naive", 1, 0), ("mxfp4_optimal", 1, 1),
    ("mxfp4_naive_torch", 1, 3), ("mxfp4_optimal_torch", 1, 4),
]


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def edge_blocks() -> torch.Tensor:
    """(n, 32) fp32 rows (cast to bf16 by the caller) exercising the corners."""
    rows = []
    z = torch.zeros(32)
    rows.append(z.clone())                                   # all +0
    rows.append(-z.clone())                                  # all -0
    rows.append(torch.linspace(-1e-4, 1e-4, 32))             # NVFP4 scale snaps to 0
    r = torch.full((32,), 1e-3); r[5] = 6 * 2.0 ** -10; rows.append(r)  # at the s=0 edge
    r = torch.linspace(-3000, 3000, 32); rows.append(r)      # amax/6 > 464: NaN scale
    r = torch.full((32,), 1.0); r[0] = 2784.0; rows.append(r)  # amax/6 = 464: tie -> 448
    r = torch.full((32,), 1e-3); r[7] = 1.0; rows.append(r)  # single outlier
    s = 0.25                                                 # exact E2M1 boundary ties at s
    ties = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0]) * s
    r = torch.cat([ties, -ties, ties * 2, -ties * 0.5]); r[0] = 1.5; rows.append(r)
    r = torch.full((32,), 0.5); rows.append(r)               # constant block
    r = torch.full((32,), -0.01); r[3] = 0.0; r[4] = -0.0; rows.append(r)
    r = torch.randn(32, generator=torch.Generator().manual_seed(5)) * 1e-38; rows.append(r)  # subnormals
    r = torch.full((32,), 3.0e38); r[1] = -1e38; rows.append(r)  # near fp32/bf16 max
    r = torch.ones(32); r[2] = float("nan"); rows.append(r)
    r = torch.ones(32); r[9] = float("inf"); rows.append(r)
    r = torch.ones(32); r[9] = -float("inf"); rows.append(r)
    r = torch.full((32,), float("nan")); rows.append(r)
    g = torch.Generator().manual_seed(7)
    for _ in range(48):                                      # wide dynamic range
        rows.append(torch.randn(32, generator=g) * torch.exp(torch.randn(32, generator=g) * 4))
    for k in range(16):                                      # power-of-two-ish amax sweep
        rows.append(torch.randn(32, generator=g) * 2.0 ** (k - 12))
    return torch.stack(rows)


def fixed_mxfp4_hessian(q):
    """The shipped mxfp4_optimal_hessian raises NameError (M_dim undefined,
    mxfp4/reference.py:301) and writes only the last H block (the H[j] = acc
    line, mxfp4/reference.py:284, sits outside the j loop).  Apply exactly those
    two fixes to its source and return the repaired function."""
    mod = sys.modules["qwantize.mxfp4.reference"]
    src = inspect.getsource(mod.mxfp4_optimal_hessian)
    fixed = src.replace("                acc.addmm_(Xj.T, Xj)\n        H[j] = acc",
                        "                acc.addmm_(Xj.T, Xj)\n            H[j] = acc")
    fixed = fixed.replace("    all_scales = build_ue8m0_scales(device=x.device)",
                          "    M_dim = N // num_col_blocks\n"
                          "    all_scales = build_ue8m0_scales(device=x.device)")
    assert fixed != src and fixed.count("M_dim = N // num_col_blocks") == 1
    ns = dict(mod.__dict__)
    exec(compile(fixed, mod.__file__, "exec"), ns)
    return ns["mxfp4_optimal_hessian"]


def ref_block_hessians(X: torch.Tensor, bs: int) -> torch.Tensor:
    """The reference's own H build (nvfp4/reference.py:308-317), verbatim in
    behaviour: fp32 addmm over 8192-token slices."""
    K = X.shape[1]
    J = K // bs
    H = torch.empty(J, bs, bs)
    for j in range(J):
        acc = torch.zeros(bs, bs)
        for t0 in range(0, X.shape[0], 8192):
            Xj = X[t0:t0 + 8192, j * bs:(j + 1) * bs].float()
            acc.addmm_(Xj.T, Xj)
        H[j] = acc
    return H


def int_tie_blocks() -> torch.Tensor:
    """(n, 32) rows whose naive NVINT4 scale is 0.25 (amax 1.75) with elements
    on exact half-integer multiples of it, both signs (round half to even)."""
    rows = []
    half = (torch.arange(7) + 0.5) * 0.25
    for k in range(4):
        r = torch.cat([half, -half, half.flip(0), -half.flip(0), torch.tensor([1.75, -1.75, 0.0, -0.0])])
        rows.append(torch.roll(r, 5 * k))
    r = torch.full((32,), 0.125); r[0] = 1.75; rows.append(r)     # all at 0.5 * s: round to 0
    r = torch.full((32,), -0.375); r[0] = 1.75; rows.append(r)    # 1.5 * s: round to -2
    return torch.stack(rows)


def make_int(q, W, E, Wh, X):
    """NVINT4 / INT8 fixtures (nvint4/reference.py, int8/reference.py)."""
    T_ = int_tie_blocks().to(torch.bfloat16)
    E256 = E.reshape(-1, 256)
    out = {"W": bits(W), "E": bits(E), "T": bits(T_), "Wh": bits(Wh)}
    for name, bss in (("nvint4", (16, 32)), ("int8", (32, 64, 128, 256))):
        for bs in bss:
            for src_name, src in (("W", W), ("E", E256 if name == "int8" else E), ("T", T_)):
                if name == "int8" and src_name == "T":
                    continue
                Wb = src.reshape(src.shape[0], -1, bs)
                for fn in ("naive", "optimal"):
                    s, qq, dq = getattr(q, f"{name}_{fn}")(Wb, return_dequant=True)
                    key = f"{name}_{src_name}_{fn}_{bs}"
                    out[key + "_scales"], out[key + "_quants"], out[key + "_dq"] = s.numpy(), qq.numpy(), dq.numpy()
            M, K = Wh.shape
            H = ref_block_hessians(X, bs)
            out[f"{name}_H_{bs}"] = H.numpy()
            Wb = Wh.reshape(M, K // bs, bs)
            fn = getattr(q, f"{name}_optimal_hessian")
            s, qq, dq = fn(Wb, return_dequant=True, H_blocks=H)
            out[f"{name}_hH_{bs}_scales"], out[f"{name}_hH_{bs}_quants"] = s.numpy(), qq.numpy()
            s, qq, dq = fn(Wb, return_dequant=True, X=X)
            out[f"{name}_hX_{bs}_scales"] = s.numpy()
    np.savez_compressed(os.path.join(HERE, "int_small.npz"), **out)


def make_int_digests(q):
    """SHA-256 of the reference's NVINT4 / INT8 naive and optimal outputs on the
    full 2560x9728 config-0/1 weight (seed 0): int_digests.json."""
    Wf = make_weight(2560, 9728, seed=0)
    dg = {"weight_sha256": hashlib.sha256(bits(Wf).tobytes()).hexdigest(),
          "M": 2560, "K": 9728, "seed": 0, "torch": torch.__version__}
    for name, bss in (("nvint4", (16, 32)), ("int8", (32, 64, 128, 256))):
        for bs in bss:
            Wb = Wf.reshape(2560, 9728 // bs, bs)
            for fn in ("naive", "optimal"):
                s, qq, dq = getattr(q, f"{name}_{fn}")(Wb, return_dequant=True)
                dg[f"{name}_{fn}_{bs}"] = {"scales": digest(s), "quants": digest(qq), "dq": digest(dq)}
                print(name, fn, bs, flush=True)
    with open(os.path.join(HERE, "int_digests.json"), "w") as f:
        json.dump(dg, f, indent=1, sort_keys=True)


def scale_codes(s: torch.Tensor, fmt: int) -> np.ndarray:
    """One byte per block: the E4M3 byte of an NVFP4 scale (0x7f for NaN) or
    the UE8M0 biased exponent of an MXFP4 scale (0xff for NaN)."""
    if fmt == 0:
        return s.to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(-1)
    b = s.contiguous().view(torch.int32).numpy().reshape(-1).astype(np.int64)
    e = (b >> 23) & 0xFF
    return np.where(np.isnan(s.numpy().reshape(-1)), 0xFF, e).astype(np.uint8)


def make_hessian_config2(q):
    """H-optimal at the BASELINE config-2 weight (2560x9728, seed 0): the
    reference's nvfp4_optimal_hessian (nvfp4/reference.py:266-407) and the
    repaired mxfp4_optimal_hessian (mxfp4/reference.py:241-374) fed the same
    block Hessians, built by the reference's own fp32 addmm loop from 32,768
    seeded synthetic activation tokens.  Stores H and one scale byte per
    block (hessian_config2.npz, about 4 MB)."""
    M, K, T = 2560, 9728, 32768
    Wf = make_weight(M, K, seed=0)
    X = make_activations(T, K, seed=41, chunk_tokens=8192)
    out = {"weight_sha256": hashlib.sha256(bits(Wf).tobytes()).hexdigest(),
           "X_sha256": hashlib.sha256(bits(X).tobytes()).hexdigest(),
           "M": M, "K": K, "T": T, "w_seed": 0, "x_seed": 41, "x_chunk": 8192, "torch": torch.__version__}
    mx_hess = fixed_mxfp4_hessian(q)
    for bs in (16, 32):
        H = ref_block_hessians(X, bs)
        out[f"H_{bs}"] = H.numpy()
        Wb = Wf.reshape(M, K // bs, bs)
        s, _ = q.nvfp4_optimal_hessian(Wb, H_blocks=H)
        out[f"nv_{bs}_codes"] = scale_codes(s, 0)
        assert np.array_equal(torch.from_numpy(out[f"nv_{bs}_codes"]).view(torch.float8_e4m3fn).float().numpy()
                              .view(np.uint32), s.reshape(-1).numpy().view(np.uint32))
        print("nvfp4 hessian", bs, flush=True)
        s, _ = mx_hess(Wb, H_blocks=H)
        out[f"mx_{bs}_codes"] = scale_codes(s, 1)
        print("mxfp4 hessian", bs, flush=True)
    np.savez_compressed(os.path.join(HERE, "hessian_config2.npz"), **out)


def make_tail(q):
    """Ragged block counts (tail_small.npz): a 37 x 544 weight is 1258 blocks of
    16 or 629 blocks of 32, neither a multiple of the 32-block chunk a warp
    owns, through every naive / optimal / *_torch function and the H-optimal
    searches (block Hessians from seeded activations)."""
    W = make_weight(37, 544, seed=51)
    X = make_activations(3000, 544, seed=52, chunk_tokens=1024)
    out = {"W": bits(W)}
    mx_hess = fixed_mxfp4_hessian(q)
    for bs in (16, 32):
        Wb = W.reshape(37, 544 // bs, bs)
        for name, _, _ in QUANT_FUNCS:
            s, qq, dq = getattr(q, name)(Wb, return_dequant=True)
            key = f"{name}_{bs}"
            out[key + "_scales"], out[key + "_quants"], out[key + "_dq"] = s.numpy(), qq.numpy(), dq.numpy()
        H = ref_block_hessians(X, bs)
        out[f"H_{bs}"] = H.numpy()
        s, qq, dq = q.nvfp4_optimal_hessian(Wb, return_dequant=True, H_blocks=H)
        out[f"nv_H_{bs}_scales"], out[f"nv_H_{bs}_quants"] = s.numpy(), qq.numpy()
        s, qq, dq = mx_hess(Wb, return_dequant=True, H_blocks=H)
        out[f"mx_H_{bs}_scales"], out[f"mx_H_{bs}_quants"] = s.numpy(), qq.numpy()
    np.savez_compressed(os.path.join(HERE, "tail_small.npz"), **out)


def main(ref_root: str, skip_digests: bool = False, only: str = None):
    sys.path.insert(0, ref_root)
    import qwantize as q

    torch.set_num_threads(os.cpu_count() or 1)

    # ---- small quantization fixtures --------------------------------------
    W = make_weight(48, 1024, seed=11)
    E = edge_blocks().to(torch.bfloat16)
    if only == "tail":
        make_tail(q)
        return
    if only == "hessian-config2":
        make_hessian_config2(q)
        return
    if only == "int-digests":
        make_int_digests(q)
        return
    if only == "int":
        Wh = make_weight(64, 512, seed=21)
        X = make_activations(4096, 512, seed=22, chunk_tokens=2048)
        make_int(q, W, E, Wh, X)
        return
    out = {"W": bits(W), "E": bits(E)}
    for bs in (16, 32):
        for src_name, src in (("W", W), ("E", E)):
            Wb = src.reshape(src.shape[0], -1, bs)
            for name, _, _ in QUANT_FUNCS:
                s, qq, dq = getattr(q, name)(Wb, return_dequant=True)
                key = f"{src_name}_{name}_{bs}"
                out[key + "_scales"] = s.numpy()
                out[key + "_quants"] = qq.numpy()
                out[key + "_dq"] = dq.numpy()
    # non-default dim: block dimension first
    Wt = W[:, :512].reshape(48, 32, 16).permute(2, 0, 1).contiguous()  # (16, 48, 32)
    s, qq, dq = q.nvfp4_optimal(Wt, dim=0, return_dequant=True)
    out["Wdim0"] = bits(Wt)
    out["Wdim0_nvfp4_optimal_16_scales"] = s.numpy()
    out["Wdim0_nvfp4_optimal_16_quants"] = qq.numpy()
    out["Wdim0_nvfp4_optimal_16_dq"] = dq.numpy()
    np.savez_compressed(os.path.join(HERE, "quant_small.npz"), **out)

    # ---- Hessian fixtures ---------------------------------------------------
    M, K, T = 64, 512, 4096
    Wh = make_weight(M, K, seed=21)
    X = make_activations(T, K, seed=22, chunk_tokens=2048)
    hout = {"W": bits(Wh), "X_sha256": hashlib.sha256(bits(X).tobytes()).hexdigest(),
            "M": M, "K": K, "T": T, "w_seed": 21, "x_seed": 22, "x_chunk": 2048}
    mx_hess = fixed_mxfp4_hessian(q)
    for bs in (16, 32):
        H = ref_block_hessians(X, bs)
        hout[f"H_{bs}"] = H.numpy()
        Wb = Wh.reshape(M, K // bs, bs)
        s, qq, dq = q.nvfp4_optimal_hessian(Wb, return_dequant=True, X=X)
        hout[f"nv_X_{bs}_scales"], hout[f"nv_X_{bs}_quants"] = s.numpy(), qq.numpy()
        s, qq, dq = q.nvfp4_optimal_hessian(Wb, return_dequant=True, H_blocks=H)
        hout[f"nv_H_{bs}_scales"], hout[f"nv_H_{bs}_quants"] = s.numpy(), qq.numpy()
        s, qq, dq = mx_hess(Wb, return_dequant=True, H_blocks=H)
        hout[f"mx_H_{bs}_scales"], hout[f"mx_H_{bs}_quants"] = s.numpy(), qq.numpy()
        s, qq, dq = mx_hess(Wb, return_dequant=True, X=X)
        hout[f"mx_X_{bs}_scales"] = s.numpy()
        s, qq, dq = q.nvfp4_admm(Wb, return_dequant=True, X=X)
        hout[f"admm_X_{bs}_scales"], hout[f"admm_X_{bs}_quants"] = s.numpy(), qq.numpy()
    np.savez_compressed(os.path.join(HERE, "hessian_small.npz"), **hout)
    make_int(q, W, E, Wh, X)

    # ---- GPTQ (experiments/quant_gptq_strided.py:49-135) on the same W and
    # H = X^T X / T (double, rounded once), with the reference's own quantizers
    sys.path.insert(0, os.path.join(ref_root, "experiments"))
    import quant_gptq_strided as gq
    Hg = (X.double().T @ X.double() / T).float()
    gout = {"W": bits(Wh)}
    for bs in (16, 32):
        Jb = K // bs
        Hbd = torch.stack([Hg[j * bs:(j + 1) * bs, j * bs:(j + 1) * bs] for j in range(Jb)])
        fns = {
            "naive": lambda w, j, bs=bs: q.nvfp4_naive(w, return_dequant=True)[2],
            "optimal": lambda w, j, bs=bs: q.nvfp4_optimal(w, return_dequant=True)[2],
            "hoptimal": lambda w, j, bs=bs, Hbd=Hbd: q.nvfp4_optimal_hessian(
                w, return_dequant=True, H_blocks=Hbd[j:j + 1])[2],
        }
        for name, fn in fns.items():
            Q, loss = gq.gptq_strided(Wh.float(), Hg, fn, block_size=bs)
            gout[f"{name}_{bs}_Q"] = Q.numpy()
            gout[f"{name}_{bs}_loss"] = np.array([loss])
    np.savez_compressed(os.path.join(HERE, "gptq_small.npz"), **gout)

    # ---- exotic scale grids (experiments/quant_exotic_scales.py:48-182) ------
    import quant_exotic_scales as qe
    from qwantize.exotic_scales import build_ue4m4_scales, build_ue5m3_scales, snap_to_table
    xout = {"W": bits(Wh), "E": bits(E)}
    for tname, table in (("ue4m4", build_ue4m4_scales()), ("ue5m3", build_ue5m3_scales())):
        xout[f"table_{tname}"] = table.numpy()
        snap = (lambda v, t=table: snap_to_table(v, t))
        for bs in (16, 32):
            xout[f"{tname}_{bs}_naive"] = qe.fp4_naive(Wh, snap, bs).numpy()
            xout[f"{tname}_{bs}_optimal"] = qe.fp4_optimal(Wh, table, snap, bs).numpy()
            xout[f"{tname}_{bs}_hoptimal"] = qe.fp4_hoptimal(Wh, X, table, snap, bs).numpy()
            xout[f"E_{tname}_{bs}_optimal"] = qe.fp4_optimal(E, table, snap, bs).numpy()
    np.savez_compressed(os.path.join(HERE, "exotic_small.npz"), **xout)

    # ---- metrics fixture ----------------------------------------------------
    Wm = make_weight(64, 512, seed=31)
    _, _, Wdq = q.nvfp4_optimal(Wm.reshape(64, 32, 16), return_dequant=True)
    Wdq = Wdq.reshape(64, 512)
    Xm = make_activations(5000, 512, seed=32, chunk_tokens=2048)
    m = q.compute_metrics(Wm, Wdq, Xm)
    m0 = q.compute_metrics(Wm, Wdq)
    np.savez_compressed(os.path.join(HERE, "metrics_small.npz"), W=bits(Wm), Wdq=Wdq.numpy(),
                        X_sha256=hashlib.sha256(bits(Xm).tobytes()).hexdigest(),
                        T=5000, x_seed=32, x_chunk=2048,
                        with_x=np.array([m["weight_error"], m["weight_error_pct"],
                                         m["output_error"], m["output_error_pct"]]),
                        without_x=np.array([m0["weight_error"], m0["weight_error_pct"]]))

    # ---- fp4_unpack decode table, read from the kernel source --------------
    src = open(os.path.join(ref_root, "qwantize", "fp4.py")).read()
    lut_word = int(re.search(r"mov\.b32 r_lut, (0x[0-9A-Fa-f]+);", src).group(1), 16)
    mags = [(lut_word >> (4 * i)) & 0xF for i in range(8)]
    byte_vals = np.arange(256, dtype=np.uint8)
    dec = np.empty(512, np.int8)
    for b in range(256):
        for h in range(2):
            nib = (b >> (4 * h)) & 0xF
            v = mags[nib & 7]
            dec[2 * b + h] = -v if nib & 8 else v
    np.savez_compressed(os.path.join(HERE, "unpack_lut.npz"), bytes=byte_vals, decoded=dec,
                        lut_word=np.array([lut_word], np.uint64))

    # ---- full-size digests (config 0 / 1 weight) ---------------------------
    if not skip_digests:
        Wf = make_weight(2560, 9728, seed=0)
        dg = {"weight_sha256": hashlib.sha256(bits(Wf).tobytes()).hexdigest(),
              "M": 2560, "K": 9728, "seed": 0, "torch": torch.__version__}
        for bs in (16, 32):
            Wb = Wf.reshape(2560, 9728 // bs, bs)
            for name, _, _ in QUANT_FUNCS:
                s, qq, dq = getattr(q, name)(Wb, return_dequant=True)
                dg[f"{name}_{bs}"] = {"scales": digest(s), "quants": digest(qq), "dq": digest(dq)}
                print(name, bs, flush=True)
        with open(os.path.join(HERE, "digests.json"), "w") as f:
            json.dump(dg, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    args = [a for i, a in enumerate(sys.argv[1:], 1)
            if not a.startswith("--") and sys.argv[i - 1] != "--only"]
    if not args:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout> [--only NAME] [--skip-digests]")
    main(args[0], skip_digests="--skip-digests" in sys.argv,
         only=sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None)
