"""NVINT4 and INT8 on the GPU (qz_int.cu through the drop-in API):
naive / SSE bit-exact against the reference's outputs (int_small.npz, made by
the reference itself) and against the oracle on larger random weights in
every input dtype; H-optimal bit-exact against the oracle given the same H and
>= 99.9% against the reference; packed layouts; block-diagonal Grams of the
INT8 block sizes."""
import numpy as np
import pytest
import torch

from tests._golden import hessian_parity, load, n_diff_bits, same_bits

pytestmark = pytest.mark.gpu
DEV = "cuda"
INT_CASES = [("nvint4", 3, bs) for bs in (16, 32)] + [("int8", 4, bs) for bs in (32, 64, 128, 256)]


def _bf(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


def _mod(name):
    import qwantize_b200 as q
    return q


@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
@pytest.mark.parametrize("method", ["naive", "optimal"])
@pytest.mark.parametrize("src", ["W", "E", "T"])
def test_int_bit_exact_vs_reference(name, fmt, bs, method, src):
    g = load("int_small.npz")
    key = f"{name}_{src}_{method}_{bs}"
    if key + "_scales" not in g:
        pytest.skip("INT8 has no tie rows")
    X = _bf(g[src])
    X = X.reshape(-1, 256) if (name == "int8" and src == "E") else X
    Wb = X.to(DEV).reshape(X.shape[0], -1, bs)
    s, qq, dq = getattr(_mod(name), f"{name}_{method}")(Wb, return_dequant=True)
    for got, k in ((s, "_scales"), (qq, "_quants"), (dq, "_dq")):
        ref = g[key + k]
        assert same_bits(got.cpu().numpy(), ref), (k, n_diff_bits(got.cpu().numpy(), ref))


@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_int_random_vs_oracle(oracle, name, fmt, bs, dtype):
    """A larger seeded weight (heavy tails), every input dtype, naive and SSE."""
    from qwantize_b200.synthetic import make_weight
    W = make_weight(96, 2048, seed=40 + bs).to(dtype)
    if dtype == torch.float32:
        W = W + torch.randn(W.shape, generator=torch.Generator().manual_seed(3)) * 1e-4
        xo = W.numpy()
        kw = {"bf16": False}
    elif dtype == torch.float16:
        xo = W.numpy()
        kw = {"bf16": False}
    else:
        xo = W.view(torch.int16).numpy().view(np.uint16)
        kw = {}
    for mi, method in ((0, "naive"), (1, "optimal")):
        s, qq, dq = getattr(_mod(name), f"{name}_{method}")(W.to(DEV).reshape(96, -1, bs), return_dequant=True)
        os_, oq, odq = oracle.quantize_int(xo, bs, fmt, mi, **kw)
        assert same_bits(s.cpu().numpy(), os_), (method, n_diff_bits(s.cpu().numpy(), os_))
        assert same_bits(qq.cpu().numpy(), oq) and same_bits(dq.cpu().numpy(), odq), method


@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
def test_int_hessian(oracle, name, fmt, bs):
    g = load("int_small.npz")
    W = _bf(g["Wh"])
    M, K = W.shape
    H = torch.from_numpy(g[f"{name}_H_{bs}"])
    fn = getattr(_mod(name), f"{name}_optimal_hessian")
    s, qq, dq = fn(W.to(DEV).reshape(M, K // bs, bs), return_dequant=True, H_blocks=H)
    os_, oq, _ = oracle.quantize_int(g["Wh"], bs, fmt, 2, H=H.numpy())
    assert same_bits(s.cpu().numpy(), os_), n_diff_bits(s.cpu().numpy(), os_)
    assert same_bits(qq.cpu().numpy(), oq)
    hessian_parity(W.float().numpy(), s.cpu().numpy(), g[f"{name}_hH_{bs}_scales"], H.numpy(),
                   grid=7 if fmt == 3 else 127)


@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
def test_int_hessian_from_x(name, fmt, bs):
    """X path: block Hessians on the tensor cores (blocks of 64 / 128 on the
    block-diagonal Gram, 256 through column-slice Grams), >= 99.9% of the
    reference's scales."""
    from qwantize_b200.synthetic import make_activations
    g = load("int_small.npz")
    W = _bf(g["Wh"])
    M, K = W.shape
    X = make_activations(4096, K, seed=22, chunk_tokens=2048)
    fn = getattr(_mod(name), f"{name}_optimal_hessian")
    s, _ = fn(W.to(DEV).reshape(M, K // bs, bs), X=X.to(DEV))
    hessian_parity(W.float().numpy(), s.cpu().numpy(), g[f"{name}_hX_{bs}_scales"], g[f"{name}_H_{bs}"],
                   grid=7 if fmt == 3 else 127)


@pytest.mark.parametrize("bs", [64, 128, 256])
def test_block_gram_wide_blocks(bs):
    from qwantize_b200.hessian import block_hessians
    g = torch.Generator().manual_seed(bs)
    X = (torch.randn(5000, 1024, generator=g) * 0.5).to(torch.bfloat16)
    H = block_hessians(X.to(DEV), bs).cpu().double()
    Xd = X.double().reshape(5000, 1024 // bs, bs)
    ref = torch.einsum("tja,tjb->jab", Xd, Xd)
    # fp32 accumulation over 5000 rows (values up to ~1300): 1e-4 relative
    assert torch.allclose(H, ref, rtol=1e-4, atol=1e-2), (H - ref).abs().max()


@pytest.mark.parametrize("name,fmt,bs", [("nvint4", 3, 16), ("nvint4", 3, 32), ("int8", 4, 64)])
def test_int_packed_layout(name, fmt, bs):
    """Native outputs decode to the fp32 results: E4M3 scale codes, two's
    complement nibbles (NVINT4, element 2i low) or int8 bytes, bf16 dequant."""
    from qwantize_b200.synthetic import make_weight
    mod = _mod(name)
    W = make_weight(64, 1024, seed=9).to(DEV).reshape(64, -1, bs)
    s, qq, dq = getattr(mod, f"{name}_optimal")(W, return_dequant=True)
    codes, packed, dqb = getattr(mod, f"{name}_quantize_packed")(W, method="optimal", return_dequant=True)
    e4 = torch.from_numpy(np.array([0.0] + [(m / 512.0 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7))
                                     for c in range(1, 127) for e, m in [(c >> 3, c & 7)]], np.float32))
    sv = e4[codes.cpu().long()]
    if name == "int8":
        sv = sv / 127.0
        q = packed.cpu().view(torch.int8).float()
    else:
        p = packed.cpu().to(torch.int32)
        lo, hi = p & 15, p >> 4
        q = torch.stack([lo, hi], -1).reshape(*packed.shape[:-1], bs)
        q = torch.where(q >= 8, q - 16, q).float()
    assert same_bits(sv.numpy(), s.cpu().numpy())
    assert torch.equal(q, qq.cpu())
    assert torch.equal(dqb.float().cpu(), dq.cpu().to(torch.bfloat16).float())


def test_int_dequantize_and_errors():
    import qwantize_b200 as q
    g = load("int_small.npz")
    W = _bf(g["W"]).to(DEV).reshape(48, -1, 32)
    s, qq, dq = q.nvint4_optimal(W, return_dequant=True)
    assert same_bits(q.nvint4_dequantize(s, qq).cpu().numpy(), dq.cpu().numpy())
    W8 = _bf(g["W"]).to(DEV).reshape(48, -1, 128)
    s, qq, dq = q.int8_optimal(W8, return_dequant=True)
    assert same_bits(q.int8_dequantize(s, qq).cpu().numpy(), dq.cpu().numpy())
    with pytest.raises(AssertionError):
        q.nvint4_naive(_bf(g["W"]).to(DEV).reshape(48, -1, 64))
    with pytest.raises(AssertionError):
        q.int8_naive(_bf(g["W"]).to(DEV).reshape(48, -1, 16))
    with pytest.raises(AssertionError):
        q.int8_optimal_hessian(W8)


@pytest.mark.parametrize("name,fmt,bs", INT_CASES)
def test_int_full_config_digests(name, fmt, bs):
    """Full 2560x9728 config-0/1 weight: SHA-256 of every output equals the
    digest of the reference's own output (int_digests.json)."""
    import hashlib
    import json
    import os
    from qwantize_b200.synthetic import make_weight
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "int_digests.json")) as f:
        d = json.load(f)
    W = make_weight(d["M"], d["K"], d["seed"])
    assert hashlib.sha256(W.view(torch.int16).numpy().tobytes()).hexdigest() == d["weight_sha256"]
    Wb = W.to(DEV).reshape(d["M"], d["K"] // bs, bs)
    for method in ("naive", "optimal"):
        s, qq, dq = getattr(_mod(name), f"{name}_{method}")(Wb, return_dequant=True)
        ref = d[f"{name}_{method}_{bs}"]
        for t, k in ((s, "scales"), (qq, "quants"), (dq, "dq")):
            assert hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest() == ref[k], (method, k)


@pytest.mark.parametrize("name,bs", [("nvint4", 16), ("int8", 64)])
def test_int_dim0_and_cpu_input(name, bs):
    """Block dimension first (dim=0) gives the same per-block results as the
    default layout; a CPU input returns CPU tensors with the same values."""
    from qwantize_b200.synthetic import make_weight
    mod = _mod(name)
    W = make_weight(24, 4 * bs, seed=5).reshape(24, 4, bs)
    s, qq, dq = getattr(mod, f"{name}_optimal")(W.to(DEV), return_dequant=True)
    Wt = W.permute(2, 0, 1).contiguous()  # (bs, 24, 4)
    st, qt, dqt = getattr(mod, f"{name}_optimal")(Wt.to(DEV), dim=0, return_dequant=True)
    assert st.shape == (24, 4) and qt.shape == Wt.shape
    assert same_bits(st.cpu().numpy(), s.cpu().numpy())
    assert same_bits(qt.permute(1, 2, 0).cpu().numpy(), qq.cpu().numpy())
    sc, qc = getattr(mod, f"{name}_optimal")(W)
    assert sc.device.type == "cpu" and qc.device.type == "cpu"
    assert same_bits(sc.numpy(), s.cpu().numpy()) and same_bits(qc.numpy(), qq.cpu().numpy())
