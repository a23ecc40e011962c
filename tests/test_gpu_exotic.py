"""Exotic 8-bit scale grids (UE4M4, UE5M3; experiments/quant_exotic_scales.py)
through qz_quantize_table: naive and SSE bit-exact against the reference
experiment's outputs, Hessian-optimal bit-exact against the oracle given the
same H and >= 99.9% against the reference (its H is built by fp32 addmm)."""
import numpy as np
import pytest
import torch

from tests._golden import hessian_parity, load, n_diff_bits, same_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("tname", ["ue4m4", "ue5m3"])
def test_exotic_naive_optimal_bit_exact(tname, bs):
    from qwantize_b200 import exotic
    g = load("exotic_small.npz")
    t = torch.from_numpy(g[f"table_{tname}"])
    W = _bf(g["W"]).to(DEV)
    for name, fn in (("naive", exotic.fp4_naive), ("optimal", exotic.fp4_optimal)):
        dq = fn(W, t, bs).cpu().numpy()
        assert same_bits(dq, g[f"{tname}_{bs}_{name}"]), (name, n_diff_bits(dq, g[f"{tname}_{bs}_{name}"]))
    dqE = exotic.fp4_optimal(_bf(g["E"]).to(DEV), t, bs).cpu().numpy()
    assert same_bits(dqE, g[f"E_{tname}_{bs}_optimal"])


@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("tname", ["ue4m4", "ue5m3"])
def test_exotic_hoptimal(oracle, tname, bs):
    from qwantize_b200 import exotic
    from qwantize_b200.synthetic import make_activations
    from tests._golden import ref_admm_matrices
    g = load("exotic_small.npz")
    h = load("hessian_small.npz")
    t = torch.from_numpy(g[f"table_{tname}"])
    W = _bf(g["W"]).to(DEV)
    M, K = W.shape
    X = make_activations(int(h["T"]), K, seed=int(h["x_seed"]), chunk_tokens=int(h["x_chunk"]))
    H = ref_admm_matrices(X, bs)[0]
    s, qq, dq = exotic.quantize_table(W.reshape(M, K // bs, bs), t, "hoptimal", return_dequant=True, H_blocks=H)
    os_, oq, odq = oracle.quantize_table(g["W"], bs, 2, g[f"table_{tname}"], H=H.numpy())
    assert same_bits(s.cpu().numpy(), os_) and same_bits(dq.cpu().numpy(), odq)
    ref = g[f"{tname}_{bs}_hoptimal"]
    xf = W.float().cpu().numpy()
    hessian_parity(xf, dq.cpu().numpy(), ref, H.numpy(), grid="dq")
    dq2 = exotic.fp4_hoptimal(W, X.to(DEV), t, bs)
    hessian_parity(xf, dq2.cpu().numpy(), ref, H.numpy(), grid="dq")


@pytest.mark.parametrize("bs", [16, 32])
def test_table_first_entry_wins(oracle, bs):
    """A coarse table whose smallest entry is often the SSE-best scale while
    the naive snap picks the next one: index 0 must be selectable."""
    from qwantize_b200 import exotic
    t = np.array([0.01, 0.011, 0.05, 0.2], np.float32)
    g = torch.Generator().manual_seed(11)
    M, K = 64, 256
    mag = torch.exp(torch.empty(M, K // bs, 1).uniform_(np.log(0.02), np.log(0.1), generator=g))
    W = (torch.randn(M, K // bs, bs, generator=g) * mag).reshape(M, K).to(torch.bfloat16)
    u16 = W.view(torch.int16).numpy().view(np.uint16)
    s, qq, dq = exotic.quantize_table(W.to(DEV).reshape(M, K // bs, bs), torch.from_numpy(t), "optimal",
                                      return_dequant=True)
    os_, oq, odq = oracle.quantize_table(u16, bs, 1, t)
    s = s.cpu().numpy().reshape(-1)
    assert same_bits(s, os_) and same_bits(dq.cpu().numpy().reshape(-1), odq.reshape(-1))
    naive = exotic.quantize_table(W.to(DEV).reshape(M, K // bs, bs), torch.from_numpy(t), "naive")[0]
    first = (s == t[0]) & (naive.cpu().numpy().reshape(-1) != t[0])
    assert first.sum() > 0  # the case under test occurs
