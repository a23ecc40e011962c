"""CPU callers of the drop-in API: uploads and results move through the
library's two page-locked staging buffers (qwantize_b200._staging) in chunks.
Round trips of empty, tiny, odd-sized, multi-chunk and non-contiguous tensors
of several dtypes, and drop-in calls on CPU input that must equal the same
calls on device input bit for bit, results handed back as ordinary CPU tensors."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("n", [0, 1, 7, 4096, (8 << 20) // 4 + 3, 5 * (8 << 20) // 2 + 1])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.uint8])
def test_round_trip(n, dtype):
    from qwantize_b200 import _staging
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(n, generator=g) * 100).to(dtype)
    d = _staging.to_device(x, DEV)
    assert d.device.type == "cuda" and torch.equal(d.cpu(), x)
    (h,) = _staging.to_host([d], DEV)
    assert h.device.type == "cpu" and not h.is_pinned() and torch.equal(h, x)


def test_several_tensors_and_views():
    from qwantize_b200 import _staging
    a = torch.randn(3000, 1000, device=DEV)
    b = torch.arange(12345, device=DEV, dtype=torch.int32)
    c = a.t()  # non-contiguous
    ha, hb, hc = _staging.to_host([a, b, c], DEV)
    assert torch.equal(ha, a.cpu()) and torch.equal(hb, b.cpu()) and torch.equal(hc, c.cpu())
    assert hc.shape == c.shape
    x = torch.randn(500, 64).t()  # a non-contiguous CPU upload
    assert torch.equal(_staging.to_device(x, DEV).cpu(), x)


@pytest.mark.parametrize("dim", [-1, 0])
def test_dropin_cpu_input_matches_device_input(dim):
    import qwantize_b200 as q
    from qwantize_b200.synthetic import make_weight
    W = make_weight(640, 2048, 5)
    W = W.reshape(640, 128, 16) if dim == -1 else W.reshape(16, 128, 640)
    cpu = q.nvfp4_optimal(W, dim=dim, return_dequant=True)
    gpu = q.nvfp4_optimal(W.to(DEV), dim=dim, return_dequant=True)
    for c, g in zip(cpu, gpu):
        assert c.device.type == "cpu" and c.shape == g.shape and torch.equal(c, g.cpu())
    # kept results stay valid while later calls reuse the staging buffers
    again = q.mxfp4_naive(W, dim=dim, return_dequant=True)
    for c, g in zip(cpu, gpu):
        assert torch.equal(c, g.cpu())
    assert torch.equal(again[0], q.mxfp4_naive(W.to(DEV), dim=dim)[0].cpu())


def test_quantize_many_cpu_inputs():
    """The grouped call on CPU weights returns CPU results equal to the same
    call on device weights."""
    from qwantize_b200.core import quantize_many
    from qwantize_b200 import _lib
    from qwantize_b200.synthetic import make_weight
    ws = [make_weight(m, 512, 10 + m) for m in (1, 37, 256)]
    for packed in (True, False):
        cpu = quantize_many(ws, _lib.FMT_NVFP4, _lib.METHOD_SSE, 16, packed=packed, return_dequant=True)
        gpu = quantize_many([w.to(DEV) for w in ws], _lib.FMT_NVFP4, _lib.METHOD_SSE, 16, packed=packed,
                            return_dequant=True)
        for rc, rg in zip(cpu, gpu):
            for c, g in zip(rc, rg):
                assert c.device.type == "cpu" and torch.equal(c, g.cpu())
