"""Pins the oracle's integer formats (qzo_quantize_int: NVINT4 and INT8) against
the reference's own outputs in tests/golden/int_small.npz."""
import numpy as np
import pytest
import torch

from tests._golden import hessian_parity, load, n_diff_bits, same_bits

INT_CASES = [("nvint4", 3, bs) for bs in (16, 32)] + [("int8", 4, bs) for bs in (32, 64, 128, 256)]


@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
@pytest.mark.parametrize("method", [0, 1])
@pytest.mark.parametrize("src", ["W", "E", "T"])
def test_oracle_int_bit_exact(oracle, name, fmt, bs, method, src):
    g = load("int_small.npz")
    key = f"{name}_{src}_{('naive', 'optimal')[method]}_{bs}"
    if key + "_scales" not in g:
        pytest.skip("no such fixture (INT8 has no tie rows)")
    x = g[src]
    s, q, dq = oracle.quantize_int(x, bs, fmt, method)
    for got, k in ((s, "_scales"), (q, "_quants"), (dq, "_dq")):
        assert same_bits(got, g[key + k]), (k, n_diff_bits(got, g[key + k]))


@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
def test_oracle_int_hessian_vs_reference(oracle, name, fmt, bs):
    """H-optimal with the reference's own H: the oracle's r^T H r uses a fixed
    FMA order, the reference einsum / bmm; >= 99.9% identical scales and every
    differing block's objective within 1e-5 relative."""
    g = load("int_small.npz")
    H = g[f"{name}_H_{bs}"]
    s, q, _ = oracle.quantize_int(g["Wh"], bs, fmt, 2, H=H)
    ref = g[f"{name}_hH_{bs}_scales"].reshape(-1)
    xf = torch.from_numpy(g["Wh"].view(np.int16)).view(torch.bfloat16).float().numpy()
    hessian_parity(xf, s, ref, H, grid=7 if fmt == 3 else 127)
    refq = g[f"{name}_hH_{bs}_quants"].reshape(-1)
    same_blocks = (s == ref)
    qb = q.reshape(-1, bs)[same_blocks]
    assert same_bits(qb, refq.reshape(-1, bs)[same_blocks])


def test_int_ties_round_half_even(oracle):
    """Exact half-integer multiples of the scale round to the even integer."""
    g = load("int_small.npz")
    q = g["nvint4_T_naive_32_quants"].reshape(-1)
    s = g["nvint4_T_naive_32_scales"].reshape(-1)
    assert (s == 0.25).all()
    x = g["T"].reshape(-1).astype(np.uint32) << 16
    xf = x.view(np.float32)
    half = np.abs(xf / 0.25 - np.round(xf / 0.25)) == 0.5
    assert half.sum() > 50
    assert (np.abs(q[half]) % 2 == 0).all()


@pytest.mark.slow
@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
def test_oracle_int_full_config_digests(oracle, name, fmt, bs):
    """Full 2560x9728 weight: the oracle's outputs hash to the reference's."""
    import hashlib
    import json
    import os

    import torch

    from qwantize_b200.synthetic import make_weight
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "int_digests.json")) as f:
        d = json.load(f)
    W = make_weight(d["M"], d["K"], d["seed"])
    wb = W.view(torch.int16).numpy().view(np.uint16)
    for mi, method in ((0, "naive"), (1, "optimal")):
        s, q, dq = oracle.quantize_int(wb, bs, fmt, mi)
        ref = d[f"{name}_{method}_{bs}"]
        for t, k in ((s, "scales"), (q, "quants"), (dq, "dq")):
            assert hashlib.sha256(t.tobytes()).hexdigest() == ref[k], (method, k)
