"""qz_quantize_grouped: many inputs in one persistent launch must give exactly
the outputs of one qz_quantize per input (the reference's row-chunked caller
loops, experiments/quant_bench.py:107-117, call one function per chunk)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _weights(shapes, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    out = []
    for M, K in shapes:
        w = torch.randn(M, K, generator=g) * torch.exp(torch.randn(M, K, generator=g) * 2) * 0.02
        out.append(w.to(dtype).to(DEV))
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("fmt", ["nvfp4", "mxfp4"])
@pytest.mark.parametrize("method", ["naive", "optimal"])
def test_grouped_equals_per_item(dtype, bs, fmt, method):
    import qwantize_b200 as q
    # ragged row counts (partial last chunks), an empty matrix, a single block
    shapes = [(37, 544), (1, bs), (0, 64), (128, 2560), (5, 96), (300, 1024)]
    ws = _weights(shapes, 11 + bs, dtype)
    got = q.quantize_many(ws, fmt, method, bs, packed=True, return_dequant=True)
    got32 = q.quantize_many(ws, fmt, method, bs, packed=False, return_dequant=True)
    fn_p = getattr(q, f"{fmt}_quantize_packed")
    fn_f = getattr(q, f"{fmt}_{method}")
    for w, (c, p, d), (s, qq, dq) in zip(ws, got, got32):
        if w.numel() == 0:
            continue
        wb = w.reshape(w.shape[0], -1, bs)
        c2, p2, d2 = fn_p(wb, method=method, return_dequant=True)
        assert torch.equal(c, c2) and torch.equal(p, p2)
        assert torch.equal(d.view(torch.int16), d2.view(torch.int16))
        s2, q2, dq2 = fn_f(wb, return_dequant=True)
        assert torch.equal(s.view(torch.int32), s2.view(torch.int32))
        assert torch.equal(qq.view(torch.int32), q2.view(torch.int32))
        assert torch.equal(dq.view(torch.int32), dq2.view(torch.int32))


def test_grouped_more_than_one_launch():
    """300 inputs: two launches of at most 256 descriptors."""
    import qwantize_b200 as q
    ws = _weights([(3 + (i % 7), 64 * (1 + i % 3)) for i in range(300)], 5)
    got = q.quantize_many(ws, "nvfp4", "optimal", 16)
    for w, (c, p) in zip(ws, got):
        c2, p2 = q.nvfp4_quantize_packed(w.reshape(w.shape[0], -1, 16), method="optimal")
        assert torch.equal(c, c2) and torch.equal(p, p2)


def test_grouped_rejects_bad_arguments():
    import ctypes

    from qwantize_b200 import _lib
    L = _lib.load()
    items = (_lib.QzQuantItem * 1)()
    items[0].x, items[0].n_blocks = 8, 4  # misaligned
    assert L.qz_quantize_grouped(items, 1, _lib.DTYPE_BF16, 16, _lib.FMT_NVFP4, _lib.METHOD_SSE, None) == \
        _lib.QZ_ERR_INVALID
    assert L.qz_quantize_grouped(items, 1, _lib.DTYPE_BF16, 16, _lib.FMT_NVFP4, _lib.METHOD_HESSIAN, None) == \
        _lib.QZ_ERR_INVALID
    assert L.qz_quantize_grouped(ctypes.c_void_p(0), 0, _lib.DTYPE_BF16, 16, _lib.FMT_NVFP4, _lib.METHOD_SSE,
                                 None) == _lib.QZ_OK


def test_grouped_preallocated_outputs():
    """outputs=: results written into the caller's tensors equal a fresh call;
    a tensor of the wrong shape or dtype is refused before any launch."""
    import qwantize_b200 as q
    ws = _weights([(37, 544), (5, 96)], 23)
    ref = q.quantize_many(ws, "nvfp4", "optimal", 16, packed=True, return_dequant=True)
    outs = [tuple(torch.full_like(t, 7) for t in r) for r in ref]
    got = q.quantize_many(ws, "nvfp4", "optimal", 16, packed=True, return_dequant=True, outputs=outs)
    for r, g, o in zip(ref, got, outs):
        for a, b, c in zip(r, g, o):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)) and b.data_ptr() == c.data_ptr()
    bad = [outs[0], (outs[1][0], outs[1][1][:, :-1], outs[1][2])]
    with pytest.raises(AssertionError):
        q.quantize_many(ws, "nvfp4", "optimal", 16, packed=True, return_dequant=True, outputs=bad)
    bad = [outs[0], (outs[1][0], outs[1][1], outs[1][2].float())]
    with pytest.raises(AssertionError):
        q.quantize_many(ws, "nvfp4", "optimal", 16, packed=True, return_dequant=True, outputs=bad)
