"""Host logic of the multi-GPU path, run as world-size-2 gloo process groups on
CPU.  The compute steps are the CPU oracle here (the GPU kernels are exercised
by the gpu-marked tests); what is tested is the sharding, gathering and
all-reduce plumbing, and that a rank that never arrives becomes an error on the
others within the process-group timeout instead of a hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwantize_b200.distributed import (compute_metrics_sharded, gram_sharded, hessian_search_sharded,
                                       quantize_sharded, shard_range, token_chunks)


def test_shard_range_covers_and_balances():
    for n in (0, 1, 7, 2560, 9999):
        for world in (1, 2, 3, 8):
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_token_chunks_whole_chunks():
    T = 1048576 + 1000
    for world in (1, 2, 4, 8):
        rs = [token_chunks(T, world, r) for r in range(world)]
        assert rs[0][0] == 0 and rs[-1][1] == T
        for a, b in rs[:-1]:
            assert a % 65536 == 0 and b % 65536 == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_fn(fmt, method):
    from oracle import oracle

    def fn(W, dim=-1, return_dequant=False, **kw):
        dim = dim % W.ndim
        bs = W.shape[dim]
        x = W.movedim(dim, -1).contiguous()
        s, q, dq, _ = oracle.quantize(x.view(torch.int16).numpy().view(np.uint16), bs, fmt, method)
        bshape = x.shape[:-1]
        res = (torch.from_numpy(s).reshape(bshape),
               torch.from_numpy(q).reshape(x.shape).movedim(-1, dim))
        if return_dequant:
            res += (torch.from_numpy(dq).reshape(x.shape).movedim(-1, dim),)
        return res
    return fn


def _oracle_gram(X, mode, bs):
    from oracle import oracle
    xb = X.contiguous().view(torch.int16).numpy().view(np.uint16)
    H = oracle.gram(xb) if mode == "full" else oracle.block_gram(xb, bs)
    return torch.from_numpy(H).double()  # double so sums of shards are exact enough


def _pack_upper(H):
    """The layout of qz_gram's QZ_GRAM_FULL_UPPER_TILES: tiles (mi, nj >= mi)
    of 256 x 256 in upper-triangle order, each column-major, zero beyond K."""
    K = H.shape[0]
    t = (K + 255) // 256
    Hp = torch.zeros(t * 256, t * 256, dtype=H.dtype)
    Hp[:K, :K] = H
    tiles = [Hp[mi * 256:(mi + 1) * 256, nj * 256:(nj + 1) * 256].t() for mi in range(t) for nj in range(mi, t)]
    return torch.stack(tiles).contiguous()


def _unpack_upper(P, K):
    t = (K + 255) // 256
    Hp = torch.zeros(t * 256, t * 256, dtype=P.dtype)
    k = 0
    for mi in range(t):
        for nj in range(mi, t):
            Hp[mi * 256:(mi + 1) * 256, nj * 256:(nj + 1) * 256] = P[k].t()
            k += 1
    U = torch.triu(Hp[:K, :K])
    return U + torch.triu(U, 1).t()


def _oracle_gram_tiles(X, mode, bs):
    return _pack_upper(_oracle_gram(X, "full", bs)) if mode == "upper_tiles" else _oracle_gram(X, mode, bs)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from qwantize_b200.synthetic import make_activations, make_weight
    W = make_weight(37, 256, seed=5)
    res = {}
    for dim, shape in ((-1, (37, 16, 16)), (0, None)):
        Wb = W.reshape(37, 16, 16) if dim == -1 else W.reshape(37, 16, 16).permute(2, 0, 1).contiguous()
        _, full = quantize_sharded(_oracle_fn(0, 1), Wb, dim=dim, return_dequant=True, gather=True)
        ref = _oracle_fn(0, 1)(Wb, dim=dim, return_dequant=True)
        res[f"q{dim}"] = all(torch.equal(a, b) for a, b in zip(full, ref))
    # token-sharded Gram
    X = make_activations(300, 64, seed=9, chunk_tokens=64)
    t0, t1 = token_chunks(300, world, rank, chunk=64)
    H = gram_sharded(X[t0:t1], "full", gram_fn=_oracle_gram)
    Href = _oracle_gram(X, "full", 16)
    # per-shard partial Grams are rounded to fp32 once each: tolerance relative
    # to the largest entry
    res["gram"] = bool(((H - Href).abs() <= 1e-6 * Href.abs().max()).all())
    # the packed upper tiles are all-reduced and expanded (K = 520: three tile
    # rows, ragged last tiles)
    X2 = make_activations(200, 520, seed=10, chunk_tokens=64)
    u0, u1 = token_chunks(200, world, rank, chunk=64)
    H2 = gram_sharded(X2[u0:u1], "full", gram_fn=_oracle_gram_tiles, unpack_fn=_unpack_upper)
    H2ref = _oracle_gram(X2, "full", 16)
    res["gram_tiles"] = bool(((H2 - H2ref).abs() <= 1e-6 * H2ref.abs().max()).all()) and torch.equal(H2, H2.t())
    Hb = gram_sharded(X[t0:t1], "blockdiag", 16, gram_fn=_oracle_gram)
    Hbr = _oracle_gram(X, "blockdiag", 16)
    res["gram_bd"] = bool(((Hb - Hbr).abs() <= 1e-6 * Hbr.abs().max()).all())

    # H-optimal: token-sharded block Gram + all-reduce, then rows sharded
    def hess_fn(W_, dim=-1, return_dequant=False, H_blocks=None):
        from oracle import oracle
        x = W_.contiguous()
        s, q, dq, _ = oracle.quantize(x.view(torch.int16).numpy().view(np.uint16), x.shape[-1], 0, 2,
                                      H=H_blocks.float().numpy())
        r = (torch.from_numpy(s).reshape(x.shape[:-1]), torch.from_numpy(q).reshape(x.shape))
        return r + (torch.from_numpy(dq).reshape(x.shape),) if return_dequant else r
    Wh = W.reshape(37, 16, 16)
    (h0, h1), part = hessian_search_sharded(hess_fn, Wh, X[t0:t1], gram_fn=_oracle_gram)
    H_all = gram_sharded(X[t0:t1], "blockdiag", 16, gram_fn=_oracle_gram)
    whole = hess_fn(Wh, H_blocks=H_all)
    res["hopt_rows"] = (h0, h1) == shard_range(37, world, rank)
    res["hopt"] = all(torch.equal(a, b[h0:h1]) for a, b in zip(part, whole))

    def sums_fn(W_, Wdq_, X_):
        from oracle import oracle
        wb = W_.view(torch.int16).numpy().view(np.uint16)
        xb = None if X_ is None else X_.contiguous().view(torch.int16).numpy().view(np.uint16)
        return torch.from_numpy(oracle.metrics_sums(wb, Wdq_.numpy(), xb))
    Wm = make_weight(8, 64, seed=3)
    _, _, Wdq = _oracle_fn(0, 1)(Wm.reshape(8, 4, 16), return_dequant=True)
    m = compute_metrics_sharded(Wm, Wdq.reshape(8, 64), X[t0:t1], sums_fn=sums_fn)
    s_full = sums_fn(Wm, Wdq.reshape(8, 64), X)
    res["metrics"] = abs(m["output_error"] - float(s_full[2]) ** 0.5) <= 1e-9 * float(s_full[2]) ** 0.5
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_world2_sharding_and_allreduce(tmp_path):
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(tmp_path / f"r{r}.pt")
        assert all(res.values()), (r, res)


def _fault_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # this rank dies between steps, before joining the next all-reduce
        os._exit(0)
    err = ""
    try:
        gram_sharded(torch.zeros(4, 16, dtype=torch.bfloat16), "blockdiag", 16,
                     gram_fn=lambda X, m, b: torch.zeros(1, 16, 16))
    except Exception as e:  # the timeout surfaces as an exception, not a hang
        err = type(e).__name__
    with open(os.path.join(out_dir, "fault.txt"), "w") as f:
        f.write(err)
    os._exit(0)


def test_rank_that_never_arrives_is_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_fault_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=60)
        assert not p.is_alive()
    err = (tmp_path / "fault.txt").read_text()
    assert err != "", "rank 0 should have seen an error"


def _agree_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "bench_under_test", os.path.join(os.path.dirname(os.path.dirname(__file__)), "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    dev = torch.device("cpu")
    res = {"all_ok": bench._all_ranks_ok(True, world, dev),
           "one_failed": bench._all_ranks_ok(rank != 1, world, dev)}
    torch.save(res, os.path.join(out_dir, f"a{rank}.pt"))
    dist.destroy_process_group()


def test_graph_capture_agreement(tmp_path):
    """bench.py times a pipeline with collectives from a CUDA graph only when
    every rank captured it: one rank's failure must put all ranks on eager
    launches, or their collectives would fall out of step."""
    mp.spawn(_agree_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(tmp_path / f"a{r}.pt")
        assert res == {"all_ok": True, "one_failed": False}, (r, res)
