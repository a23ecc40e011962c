"""GPTQ on the full Hessian (experiments/quant_gptq_strided.py) with this
library's quantization kernels, against the reference's gptq_strided run with
its own quantizers on the same W and H = X^T X / T.  Error propagation
reassociates fp32 sums (lazy-batched groups, batched GEMMs; still a code that
flips early changes every later column's input, so the bar is statistical:
the GPTQ loss within 0.5% and >= 97% of dequantized weights identical."""
import numpy as np
import pytest
import torch

from tests._golden import load

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs():
    from qwantize_b200.synthetic import make_activations
    g = load("hessian_small.npz")
    X = make_activations(int(g["T"]), int(g["K"]), seed=int(g["x_seed"]), chunk_tokens=int(g["x_chunk"]))
    H = (X.double().T @ X.double() / X.shape[0]).float()
    W = torch.from_numpy(g["W"].view(np.int16)).view(torch.bfloat16)
    return W, H


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("method", ["naive", "optimal", "hoptimal"])
def test_gptq_vs_reference(method, bs, group):
    """Column groups of 32, 64 and 128 (the in-group update in the group
    kernel, the rest on the tensor-core tf32x3 GEMM) all reach the bar."""
    from qwantize_b200.gptq import gptq
    W, H = _inputs()
    gg = load("gptq_small.npz")
    Q, loss = gptq(W.to(DEV), H.to(DEV), "nvfp4", method, bs, group=group)
    Qr = gg[f"{method}_{bs}_Q"]
    ref_loss = float(gg[f"{method}_{bs}_loss"][0])
    same = (Q.cpu().numpy() == Qr).mean()
    print(method, bs, "identical", same, "loss", loss, ref_loss)
    assert abs(loss - ref_loss) <= 1e-5 * ref_loss
    assert same >= 0.999


def test_gptq_ordered_runs_and_beats_naive_quantization():
    import qwantize_b200 as q
    from qwantize_b200.gptq import gptq_ordered
    W, H = _inputs()
    Wd = W.to(DEV)
    Q, loss = gptq_ordered(Wd, H.to(DEV), "nvfp4", "optimal", 16)
    # output-space error tr(E H E^T) below plain SSE-optimal quantization
    _, _, dq = q.nvfp4_optimal(Wd.reshape(W.shape[0], -1, 16), return_dequant=True)
    Hd = H.to(DEV)

    def out_err(Qm):
        E = Qm.float() - Wd.float()
        return float((E @ Hd * E).sum())
    assert out_err(Q) < out_err(dq.reshape(W.shape))


@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
def test_gptq_ragged_rows_vs_strided_loop(fmt):
    """200 rows (not a multiple of the 64-row CTA or the 128-row GEMM tile), K =
    640: the fused group kernels + tf32x3 update against the reference's
    strided loop (experiments/quant_gptq_strided.py:95-133) written in fp64
    torch with this library's quantizer per block."""
    import qwantize_b200 as q
    from qwantize_b200.gptq import _inverse_hessian, gptq
    from qwantize_b200.synthetic import make_activations, make_weight
    M, K, bs = 200, 640, 16
    W = make_weight(M, K, seed=61).float().to(DEV)
    X = make_activations(2048, K, seed=62, chunk_tokens=1024).to(DEV)
    H = (X.double().T @ X.double() / X.shape[0]).float()
    Q, loss = gptq(W, H, fmt, "optimal", bs)
    Hi = _inverse_hessian(H, 0.01).double()
    Wr = W.double().clone()
    Qr = torch.zeros_like(Wr)
    ref_loss = 0.0
    fn = getattr(q, f"{fmt}_optimal")
    for b in range(K // bs):
        cs, ce = b * bs, (b + 1) * bs
        wb = Wr[:, cs:ce].float()
        _, _, dq = fn(wb.reshape(M, 1, bs), return_dequant=True)
        dq = dq.reshape(M, bs).double()
        Qr[:, cs:ce] = dq
        hd = Hi.diagonal()[cs:ce]
        err = (wb.double() - dq) / hd
        ref_loss += float(((wb.double() - dq) ** 2 / hd).sum())
        Wr[:, ce:] -= err @ Hi[cs:ce, ce:]
    same = (Q.double() == Qr).double().mean().item()
    assert abs(loss - ref_loss / M) <= 1e-4 * ref_loss / M, (loss, ref_loss / M)
    assert same >= 0.99, same


@pytest.mark.parametrize("n", [32, 128, 160, 416, 1024, 2080])
def test_spd_inverse_vs_double(n):
    """qz_spd_inverse (Schur-complement recursion, tf32x3 tensor-core products,
    double-precision leaf blocks) against the float64 inverse: within the
    accuracy of an fp32 inverse, |X - X64| <= 1e-5 * cond-scaled max |X64|."""
    from qwantize_b200.gptq import spd_inverse
    g = torch.Generator().manual_seed(n)
    Xa = torch.randn(4 * n, n, generator=g, dtype=torch.float64) * torch.exp(torch.randn(n, generator=g,
                                                                                          dtype=torch.float64))
    A = Xa.T @ Xa / (4 * n)
    A.diagonal().add_(0.01 * A.diagonal().mean())
    ref = torch.linalg.inv(A)
    Xi = spd_inverse(A.float().to(DEV)).double().cpu()
    cond = float(torch.linalg.cond(A))
    err = float((Xi - ref).abs().max() / ref.abs().max())
    assert err <= 2e-7 * cond, (err, cond)


def test_spd_inverse_rejects_indefinite():
    from qwantize_b200.gptq import spd_inverse
    A = torch.eye(64, device=DEV)
    A[5, 5] = -1.0
    with pytest.raises(torch.linalg.LinAlgError):
        spd_inverse(A)
