"""Exhaustive CPU proofs of the exact-rounding shortcuts the kernels use
(every finite non-negative bf16 and fp16 magnitude x every E4M3 and UE8M0
scale), compared with the reference's torch.bucketize(|x| / s)."""
import numpy as np
import pytest
import torch

B = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)


def _scales():
    from qwantize_b200 import _lib
    return _lib.scale_table(0).numpy(), _lib.scale_table(1).numpy()


def _mags():
    f16 = torch.arange(0, 0x7C00, dtype=torch.int32).to(torch.int16).view(torch.float16).float().numpy()
    bf = torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).float().numpy()
    return {"fp16": f16, "bf16": bf}


def _ref_bucket(a, s):
    return torch.bucketize(torch.from_numpy(a) / float(s), torch.from_numpy(B)).numpy()


def e2m1_rne_satfinite(y):
    """Round-to-nearest-even onto {0,.5,1,1.5,2,3,4,6} (code LSB even on ties),
    saturating to 6: the semantics of cvt.rn.satfinite.e2m1x2.f32 for y >= 0."""
    idx_lo = np.searchsorted(B, y, side="left")    # #{k: B_k < y}
    idx_hi = np.searchsorted(B, y, side="right")   # #{k: B_k <= y}
    tie = idx_lo != idx_hi                         # y equals a boundary
    even = np.where(idx_lo % 2 == 0, idx_lo, idx_hi)
    return np.where(tie, even, idx_lo), tie


@pytest.mark.parametrize("kind", ["fp16", "bf16"])
def test_biased_hardware_rounding_equals_bucketize(kind):
    """y' = |x| * c with c = RN(RN(1/s) * (1 - 2^-13)) never lands on a tie, and
    RNE(y') equals bucketize(|x| / s) with the reference's ties-to-smaller."""
    nv, mx = _scales()
    a = _mags()[kind]
    bias = np.float32(1.0 - 2.0 ** -13)
    for s in np.concatenate([nv, mx]):
        c = np.float32(np.float32(np.float32(1.0) / np.float32(s)) * bias)
        with np.errstate(over="ignore"):
            y = (a * c).astype(np.float32)
        got, tie = e2m1_rne_satfinite(y)
        assert not tie.any(), float(s)
        ref = _ref_bucket(a, s)
        assert np.array_equal(got, ref), (kind, float(s), int((got != ref).sum()))


MID = np.array([0.25 + 2.0 ** -26, 0.75 + 2.0 ** -25, 1.25 + 2.0 ** -24, 1.75 + 2.0 ** -24, 2.5 + 2.0 ** -23,
                3.5 + 2.0 ** -23, 5.0 + 2.0 ** -22], np.float64)


def _rd32(x):
    """Round float64 toward -inf to float32."""
    f = x.astype(np.float32)
    return np.where(f.astype(np.float64) > x, np.nextafter(f, np.float32(-np.inf)), f)


def test_division_free_bucketize_for_fp32_input():
    """fp32 inputs: fl32(a / s) > B_k  <=>  a > RD32(s * (B_k + ulp(B_k) / 2)).
    Checked against the IEEE quotient for every E4M3 / UE8M0 scale and random
    fp32 table scales, over random fp32 magnitudes plus, for each scale, the
    floats next to every threshold (where the two tests could disagree)."""
    nv, mx = _scales()
    g = np.random.default_rng(3)
    tab = np.sort(np.exp(g.uniform(-30, 30, 400))).astype(np.float32)
    for s in np.concatenate([nv, mx[(mx > 1e-30) & (mx < 1e30)], tab]):
        s = np.float32(s)
        T = _rd32(np.float64(s) * MID)
        a = np.concatenate([
            (np.exp(g.uniform(-12, 3, 4000)) * s).astype(np.float32),
            T, np.nextafter(T, np.float32(np.inf)), np.nextafter(T, np.float32(0)),
            (B.astype(np.float64) * s).astype(np.float32),
        ]).astype(np.float32)
        a = a[np.isfinite(a)]
        with np.errstate(over="ignore"):
            q = (a / s).astype(np.float32)
        want = (q[:, None] > B[None, :])
        got = (a[:, None] > T[None, :])
        assert np.array_equal(want, got), float(s)
