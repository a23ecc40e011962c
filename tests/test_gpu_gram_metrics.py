"""GPU checks of the tcgen05 Gram (H = X^T X) and the fused output-error GEMM.

Floating point (exact bf16 products, fp32 accumulation on the tensor cores):
each entry of H must match a double-precision Gram within the worst-case bound
for an fp32 sum of T terms in any order, |H - H64| <= T * 2^-24 * (|X|^T |X|);
the H-optimal search fed with this H must pick the reference's scale in
>= 99.9% of blocks (the Hessian parity bar)."""
import hashlib

import numpy as np
import pytest
import torch

from tests._golden import hessian_parity, load

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _x(T, K, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(T, K, generator=g) * torch.exp(torch.randn(K, generator=g))).to(torch.bfloat16)


def _check_h(H, X):
    Xd = X.double()
    ref = Xd.T @ Xd
    bound = Xd.abs().T @ Xd.abs()
    err = (H.double().cpu() - ref).abs()
    tol = X.shape[0] * 2.0 ** -24
    assert bool((err <= tol * bound + 1e-30).all()), float((err / (bound + 1e-30)).max())


@pytest.mark.parametrize("T,K", [(1000, 384), (4160, 512), (77, 264), (1, 256)])
def test_gram_full(T, K):
    from qwantize_b200.hessian import gram
    X = _x(T, K, T + K)
    H = gram(X.to(DEV), "full")
    torch.cuda.synchronize()
    assert torch.equal(H, H.T), "H must be exactly symmetric"
    _check_h(H, X)


def test_gram_full_multi_segment():
    """600,000 tokens is three 262,144-row segments of the full Gram: each
    tile's segments are added in segment order through per-tile counters, so
    H is deterministic (two calls agree bit for bit) and exactly symmetric."""
    from qwantize_b200.hessian import gram
    X = _x(600000, 256, 5)
    Xg = X.to(DEV)
    H = gram(Xg, "full")
    H2 = gram(Xg, "full")
    torch.cuda.synchronize()
    assert torch.equal(H, H2)
    assert torch.equal(H, H.T)
    _check_h(H, X)


@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("T,K", [(2048, 512), (300, 96)])
def test_gram_blockdiag(bs, T, K):
    from qwantize_b200.hessian import gram
    X = _x(T, K, 7 * T + K)
    Hb = gram(X.to(DEV), "blockdiag", bs).cpu()
    Hf = gram(X.to(DEV), "full").cpu()
    J = K // bs
    for j in range(J):
        blk = Hf[j * bs:(j + 1) * bs, j * bs:(j + 1) * bs]
        assert torch.equal(Hb[j], blk)


def test_gram_accumulate_token_chunks():
    from qwantize_b200.hessian import gram
    X = _x(3000, 256, 3)
    H = gram(X[:1234].to(DEV), "full")
    gram(X[1234:].to(DEV), "full", out=H, accumulate=True)
    _check_h(H, X)


def test_gram_empty_tokens_is_zero():
    from qwantize_b200.hessian import gram
    H = gram(torch.zeros(0, 128, dtype=torch.bfloat16, device=DEV), "full")
    assert torch.count_nonzero(H) == 0


def test_hessian_X_path_vs_reference():
    """nvfp4_optimal_hessian(W, X=X) / mxfp4 with the tensor-core Gram against
    the reference's X path: >= 99.9% identical scales, differing blocks within
    1e-5 relative objective."""
    import qwantize_b200 as q
    from qwantize_b200.synthetic import make_activations
    g = load("hessian_small.npz")
    X = make_activations(int(g["T"]), int(g["K"]), seed=int(g["x_seed"]), chunk_tokens=int(g["x_chunk"]))
    assert hashlib.sha256(X.view(torch.int16).numpy().tobytes()).hexdigest() == str(g["X_sha256"])
    W = torch.from_numpy(g["W"].view(np.int16)).view(torch.bfloat16)
    M, K = W.shape
    for bs in (16, 32):
        Wb = W.to(DEV).reshape(M, K // bs, bs)
        Hb = q.hessian.block_hessians(X.to(DEV), bs).cpu()
        Href = torch.from_numpy(g[f"H_{bs}"])
        rel = ((Hb - Href).abs().max() / Href.abs().max()).item()
        assert rel < 1e-4, rel  # two fp32 summation orders of T = 4096 terms
        xf = W.float().numpy()
        s, _ = q.nvfp4_optimal_hessian(Wb, X=X.to(DEV))
        # objectives of differing blocks measured with the reference's H
        hessian_parity(xf, s.cpu().numpy(), g[f"nv_X_{bs}_scales"], g[f"H_{bs}"])
        s2, _ = q.nvfp4_optimal_hessian_triton(Wb, X=X.to(DEV))
        assert torch.equal(s, s2)
        s, _ = q.mxfp4_optimal_hessian(Wb, X=X.to(DEV))
        hessian_parity(xf, s.cpu().numpy(), g[f"mx_X_{bs}_scales"], g[f"H_{bs}"])


def test_compute_metrics_vs_reference():
    import qwantize_b200 as q
    from qwantize_b200.synthetic import make_activations
    g = load("metrics_small.npz")
    X = make_activations(int(g["T"]), 512, seed=int(g["x_seed"]), chunk_tokens=int(g["x_chunk"]))
    W = torch.from_numpy(g["W"].view(np.int16)).view(torch.bfloat16)
    Wdq = torch.from_numpy(g["Wdq"])
    m = q.compute_metrics(W.to(DEV), Wdq.to(DEV), X.to(DEV))
    ref = g["with_x"]
    # the reference's norm accumulates in fp32, this one in double
    assert abs(m["weight_error"] - ref[0]) <= 1e-5 * ref[0]
    assert abs(m["weight_error_pct"] - ref[1]) <= 1e-5 * ref[1]
    assert abs(m["output_error"] - ref[2]) <= 1e-4 * ref[2]
    assert abs(m["output_error_pct"] - ref[3]) <= 1e-4 * ref[3]


@pytest.mark.parametrize("T,M,K", [(1000, 200, 256), (129, 128, 64), (4096, 384, 1024)])
def test_output_error_sums_vs_double(T, M, K):
    from qwantize_b200.metrics import output_error_sums
    g = torch.Generator().manual_seed(T + M + K)
    X = torch.randn(T, K, generator=g).to(torch.bfloat16)
    W = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16)
    Wq = (W.float() + torch.randn(M, K, generator=g) * 1e-3).to(torch.bfloat16)
    s = output_error_sums(W.to(DEV), Wq.to(DEV), X.to(DEV)).cpu()
    ref = X.double() @ W.double().T
    dq = X.double() @ Wq.double().T
    e = ((dq - ref) ** 2).sum().item()
    r = (ref ** 2).sum().item()
    assert abs(s[1].item() - r) <= 1e-5 * r
    assert abs(s[0].item() - e) <= 1e-3 * e


@pytest.mark.parametrize("bs", [16, 32])
def test_admm_kernel_vs_oracle_and_reference(oracle, bs):
    """qz_admm fed the same H / H_norm / M_inv as the oracle: identical scales
    and codes (same operation order); nvfp4_admm end to end (tensor-core H,
    device eigen/inverse routines) against the reference's own output: the
    iteration is discrete, so a last-bit difference in H can flip a code --
    the bar is >= 99% identical scales."""
    import qwantize_b200 as q
    from qwantize_b200.core import admm_fp32
    from qwantize_b200.synthetic import make_activations
    from tests._golden import ref_admm_matrices
    g = load("hessian_small.npz")
    X = make_activations(int(g["T"]), int(g["K"]), seed=int(g["x_seed"]), chunk_tokens=int(g["x_chunk"]))
    W = torch.from_numpy(g["W"].view(np.int16)).view(torch.bfloat16)
    M, K = W.shape
    Wb = W.reshape(M, K // bs, bs)
    H, Hn, Minv = ref_admm_matrices(X, bs)
    s, qq = admm_fp32(Wb.to(DEV), -1, False, H, Hn, Minv)
    os_, oq = oracle.admm(g["W"], bs, H.numpy(), Hn.numpy(), Minv.numpy())
    assert np.array_equal(s.cpu().numpy().reshape(-1).view(np.uint32), os_.view(np.uint32))
    assert np.array_equal(qq.cpu().numpy().reshape(-1).view(np.uint32), oq.view(np.uint32))
    s2, q2, dq2 = q.nvfp4_admm(Wb.to(DEV), X=X.to(DEV), return_dequant=True)
    same = (s2.cpu().numpy().reshape(-1) == g[f"admm_X_{bs}_scales"].reshape(-1)).mean()
    assert same >= 0.99, same
    assert torch.equal(dq2.cpu(), q2.cpu() * s2.cpu().unsqueeze(-1))


@pytest.mark.parametrize("T,K", [(3000, 1000), (300000, 520), (5000, 9728), (64, 256)])
def test_gram_upper_tiles_unpack_equals_full(T, K):
    """QZ_GRAM_FULL_UPPER_TILES + qz_gram_unpack gives QZ_GRAM_FULL's H bit for
    bit (ragged K, several 262,144-token segments, accumulate); the packed
    tiles follow the documented layout (upper-triangle order, column-major)."""
    from qwantize_b200.hessian import gram, unpack_upper_tiles
    g = torch.Generator().manual_seed(T + K)
    X = (torch.randn(T, K, generator=g) * torch.exp(torch.randn(K, generator=g))).to(torch.bfloat16).to(DEV)
    H = gram(X, "full")
    P = gram(X, "upper_tiles")
    assert torch.equal(unpack_upper_tiles(P, K), H)
    t = (K + 255) // 256
    Hp = torch.zeros(t * 256, t * 256, device=DEV)
    Hp[:K, :K] = H
    k = 0
    for mi in range(t):
        for nj in range(mi, t):
            assert torch.equal(P[k], Hp[mi * 256:(mi + 1) * 256, nj * 256:(nj + 1) * 256].t())
            k += 1
    # accumulate: a second Gram added into both forms
    gram(X, "full", out=H, accumulate=True)
    gram(X, "upper_tiles", out=P, accumulate=True)
    assert torch.equal(unpack_upper_tiles(P, K), H)
