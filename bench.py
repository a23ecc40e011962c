"""Benchmark: G weights/s quantized (NVFP4/MXFP4 naive + SSE-optimal), config 1.

One step = the eight quantizations of configuration 1 -- NVFP4 and MXFP4, block
16 and 32, naive and SSE-optimal -- each over a full 2560x9728 bf16 weight
(the Qwen3-4B down_proj shape; seeded synthetic N(0, 0.02^2) with 0.1% x20
outliers), writing native outputs (scale bytes, packed E2M1 nibbles, bf16
dequant).  The eight calls of a step read eight different weights from a pool
of eight (400 MB > the 126 MB L2), so every call streams its input from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): weak scaling, every rank quantizes its
own pool (rank-seeded); no collective on the data path; time = max over ranks.
The `extras` object adds the other configurations on the same GPUs: the
row-sharded Qwen3-4B stack (config 3, strong scaling, one grouped launch per
rank), the Llama-3-70B stack (config 4, layer by layer), the token-sharded
Gram, all-reduce and row-sharded H-optimal search (config 2; config 4's
down_proj with its full 28672^2 H), compute_metrics, GPTQ, and the drop-in
fp32 API end to end from host memory.

--impl reference times the reference algorithm's CPU implementation (the
oracle restatement, all host threads) on rank 0 only, plus the reference's own
pure-PyTorch nvfp4_optimal on a row sample when its package is installed under
baseline/_ref.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, K = 2560, 9728
WEIGHTS = M * K
CALLS = [(fmt, bs, meth) for fmt in (0, 1) for bs in (16, 32) for meth in (0, 1)]  # 8 per step
FMT_NAME = {0: "nvfp4", 1: "mxfp4"}
METH_NAME = {0: "naive", 1: "optimal"}
POOL = 8
METRIC = "G weights/s quantized (NVFP4/MXFP4 naive+SSE, config 1)"

# Lane-op cost model of the bounded scale search, fixed before the kernels were
# written: per element, 12 lane-ops for the search bounds (sort, prefix sums),
# 10 per full-error evaluation of a candidate (the naive scale's included) and
# 4 per clipping-error evaluation.  The counts come from the reference
# algorithm itself (the CPU restatement's counters) in the same run.
OPS_BOUNDS, OPS_FULL, OPS_CLIP = 12, 10, 4
# DRAM read + write bytes of one launch of NVFP4 bs16 SSE-optimal with native
# outputs on the config-1 weight, from one ncu capture (49.85 MB read + 9.56 MB
# written; most of the 63.8 MB of outputs is still in L2 when the kernel ends).
NCU_TRAFFIC_NVFP4_SSE_BS16 = 59.41e6


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """SM clock and throttle reasons sampled every 20 ms while the timed region
    runs (NVML, read-only; nvidia-smi every 200 ms if NVML is unavailable)."""

    # NVML clocks-event-reason bits
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80, "sw_power_cap": 0x4}

    def __init__(self, cuda_index):
        self.index = cuda_index
        self.samples = []  # (sm_mhz, max_mhz, reason_bits)
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            ids = [v for v in vis.split(",") if v.strip()]
            phys = int(ids[cuda_index]) if ids and ids[cuda_index].strip().isdigit() else cuda_index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self._nvml = pynvml
        except Exception:
            self._nvml = None

    def _sample(self):
        n = self._nvml
        if n is not None:
            sm = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
            mx = n.nvmlDeviceGetMaxClockInfo(self._h, n.NVML_CLOCK_SM)
            try:
                rs = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                rs = n.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
            return sm, mx, rs
        out = subprocess.run(["nvidia-smi", f"--id={self.index}", "--query-gpu=clocks.sm,clocks.max.sm,"
                              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True,
                             timeout=5).stdout.strip().split(",")
        bits = 0
        for name, v in zip(("hw_slowdown", "sw_thermal_slowdown", "hw_thermal_slowdown", "sw_power_cap"), out[2:]):
            if "Active" in v and "Not" not in v:
                bits |= self.REASONS[name]
        return float(out[0]), float(out[1]), bits

    def _run(self):
        period = 0.02 if self._nvml is not None else 0.2
        while not self._stop.is_set():
            try:
                self.samples.append(self._sample())
            except Exception:
                pass
            self._stop.wait(period)

    def __enter__(self):
        try:
            self.samples.append(self._sample())  # one sample even for a short region
        except Exception:
            pass
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock samples"], "samples": 0}
        reasons = sorted({k for _, _, b in self.samples for k, bit in self.REASONS.items() if b & bit})
        return {"sm_mhz": float(np.median([s[0] for s in self.samples])),
                "sm_max_mhz": float(max(s[1] for s in self.samples)), "reasons": reasons,
                "samples": len(self.samples), "source": "nvml" if self._nvml is not None else "nvidia-smi"}


def measured_peaks():
    """(HBM GB/s, bf16 TF/s burst, bf16 TF/s sustained, kind)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return (d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0),
                "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


def make_pool(rank, device):
    from qwantize_b200.synthetic import make_weight_device
    return [make_weight_device(M, K, 1000 * rank + i, device) for i in range(POOL)]


def alloc_outputs(device):
    out = {}
    for bs in (16, 32):
        nb = WEIGHTS // bs
        out[bs] = (torch.empty(nb, dtype=torch.uint8, device=device),
                   torch.empty(nb * bs // 2, dtype=torch.uint8, device=device),
                   torch.empty(WEIGHTS, dtype=torch.bfloat16, device=device))
    return out


def run_step(L, pool, outs, step, stream):
    """Eight C-ABI launches, one per call of the step (inputs resident in HBM)."""
    for k, (fmt, bs, meth) in enumerate(CALLS):
        x = pool[(step * len(CALLS) + k) % POOL]
        codes, packed, dqb = outs[bs]
        st = L.qz_quantize(x.data_ptr(), 1, WEIGHTS // bs, bs, fmt, meth, None, 0, None, None,
                           None, codes.data_ptr(), packed.data_ptr(), dqb.data_ptr(), stream)
        if st:
            raise RuntimeError(L.qz_last_error().decode())


def cpu_oracle_workload(threads):
    """The reference algorithm on the host (oracle restatement): the full
    config-1 workload once.  Returns (seconds, weights, {call: (candidates in
    range, full evaluations)})."""
    from oracle import oracle
    from qwantize_b200.synthetic import make_weight
    W = make_weight(M, K, seed=0).view(torch.int16).numpy().view(np.uint16)
    t0 = time.perf_counter()
    counts = {}
    for fmt, bs, meth in CALLS:
        _, _, _, nc = oracle.quantize(W, bs, fmt, meth, threads=threads, counts=True)
        counts[(fmt, bs, meth)] = nc
    return time.perf_counter() - t0, WEIGHTS * len(CALLS), counts


def reference_torch_sample(threads, rows=256):
    """The reference's own pure-PyTorch nvfp4_optimal (nvfp4/reference.py:
    129-239) on `rows` rows of the config weight (bs16), on the host cores, if
    its package is installed under baseline/_ref.  G weights/s or None."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "qwantize")):
        return None
    sys.path.insert(0, ref)
    try:
        import qwantize
    finally:
        sys.path.remove(ref)
    from qwantize_b200.synthetic import make_weight
    torch.set_num_threads(threads)
    W = make_weight(M, K, seed=0)[:rows].reshape(rows, K // 16, 16)
    qwantize.nvfp4_optimal(W[:8])  # warm-up
    t0 = time.perf_counter()
    qwantize.nvfp4_optimal(W)
    dt = time.perf_counter() - t0
    return {"value": rows * K / dt / 1e9, "unit": "G weights/s", "cores": threads, "kind": "reference",
            "seconds": dt, "sample": f"nvfp4_optimal bs16 on {rows} of the 2560 rows of the config-1 weight",
            "package": "baseline/_ref/qwantize (the reference's pure-PyTorch path)"}


def bench_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cpu_oracle_workload(threads)  # warm-up of the library / page cache
    for _ in range(max(0, args.warmup - 1)):
        cpu_oracle_workload(threads)
    t, n = 0.0, 0
    for _ in range(args.steps):
        dt, w, _ = cpu_oracle_workload(threads)
        t += dt
        n += w
    v = n / t / 1e9
    line = {"impl": "reference", "metric": METRIC,
            "value": v, "unit": "G weights/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1: nvfp4+mxfp4 x bs16+bs32 x naive+optimal on one 2560x9728 bf16 weight",
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": v, "unit": "G weights/s", "cores": threads, "kind": "port",
                             "sample": "the full config-1 workload (8 quantizations of 24.9M weights) per step"},
            "e2e": {"value": v, "unit": "G weights/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "reference_torch": reference_torch_sample(threads)}
    print(json.dumps(line), flush=True)


def _ev_time(fn, stream, reps=1):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _all_ranks_ok(ok, ws, device):
    """True on every rank when ok is true on every rank (one all-reduce)."""
    return _max_over_ranks(0.0 if ok else 1.0, ws, device) == 0.0


def _graph_time(fn, stream, reps, ws, device):
    """Device time of fn per call (max over ranks), replayed from a CUDA graph
    captured once, so no host gap between the call's launches falls inside
    the timed region.  Every rank tries the capture and the ranks agree
    before timing (one failure puts all ranks on eager launches, keeping their
    collectives in step).  Returns (ms, how)."""
    fn()
    torch.cuda.synchronize()
    g, err = None, None
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
    except Exception as ex:  # noqa: BLE001
        g, err = None, type(ex).__name__
        torch.cuda.synchronize()
    if not _all_ranks_ok(g is not None, ws, device):
        how = "eager launches (graph capture failed" + (f": {err})" if err else " on another rank)")
        return _max_over_ranks(_ev_time(fn, stream, reps), ws, device), how
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    return _max_over_ranks(ms, ws, device), "cuda graph replay"


def _max_over_ranks(v, ws, device):
    if ws == 1:
        return v
    t = torch.tensor([v], device=device, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(v, ws, device):
    if ws == 1:
        return v
    t = torch.tensor([v], device=device, dtype=torch.float64)
    torch.distributed.all_reduce(t)
    return float(t.item())


def _barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def roofline(per, counts, sm_mhz, n_sms, hbm_peak, peak_kind):
    """Roofline of the dominant kernel (longest launch of the step).  The SSE
    search is issue-bound: achieved = lane-ops of the reference algorithm's own
    work (cost model above, candidate counts from the CPU restatement in this
    run) / launch time; peak = SMs x 128 FP32 lanes x the median SM clock
    sampled during the timed region.  The HBM figures of the same launch are
    kept as a secondary object."""
    dom = max(per, key=per.get)
    fmt, bs, meth = dom
    t = per[dom] / 1e3
    blocks = WEIGHTS // bs
    bytes_per_w = 2 + 0.5 + 1.0 / bs + 2  # bf16 in; nibbles + scale byte + bf16 dequant out
    hbm_ach = WEIGHTS * bytes_per_w / t / 1e9
    hbm = {"bound": "hbm", "achieved": hbm_ach, "peak": hbm_peak, "unit": "GB/s", "frac": hbm_ach / hbm_peak,
           "peak_kind": peak_kind, "bytes_per_weight": bytes_per_w,
           "traffic": NCU_TRAFFIC_NVFP4_SSE_BS16 if dom == (0, 16, 1) else None,
           "traffic_unit": "DRAM bytes read + written per launch (ncu)"}
    kname = f"quantize {FMT_NAME[fmt]} {METH_NAME[meth]} bs{bs}"
    if meth == 0 or counts is None:
        out = dict(hbm)
        out.update({"kernel": kname, "issue": None})
        if meth != 0:
            out["note"] = "no candidate counts in this run (--no-cpu-baseline): issue roofline not computed"
        return out
    n_in, n_full = counts[dom]
    full_pb, clip_pb = 1.0 + n_full / blocks, n_in / blocks
    ops_pb = bs * (OPS_BOUNDS + OPS_FULL * full_pb + OPS_CLIP * clip_pb)
    ach = blocks * ops_pb / t
    peak = n_sms * 128 * sm_mhz * 1e6
    return {"kernel": kname, "bound": "issue", "achieved": ach / 1e12, "peak": peak / 1e12, "unit": "T lane-op/s",
            "frac": ach / peak, "peak_kind": f"{n_sms} SMs x 128 lanes x median sampled SM clock {sm_mhz:.0f} MHz",
            "traffic": hbm["traffic"], "traffic_unit": hbm["traffic_unit"],
            "model": {"lane_ops_per_weight": ops_pb / bs, "full_evaluations_per_block": full_pb,
                      "clip_evaluations_per_block": clip_pb, "ops_bounds_full_clip_per_element":
                      [OPS_BOUNDS, OPS_FULL, OPS_CLIP], "launch_ms": per[dom]},
            "hbm": hbm}


def bench_ours(args):
    ws, rank, local = dist_env()
    if ws > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from qwantize_b200 import _lib
    L = _lib.load()
    pool = make_pool(rank, device)
    outs = alloc_outputs(device)
    stream = torch.cuda.current_stream(device)
    sp = stream.cuda_stream
    n_sms = torch.cuda.get_device_properties(device).multi_processor_count

    for w in range(args.warmup):
        run_step(L, pool, outs, w, sp)
    torch.cuda.synchronize(device)
    _barrier(ws)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk_s:
        e0.record(stream)
        for s in range(args.steps):
            run_step(L, pool, outs, s, sp)
        e1.record(stream)
        torch.cuda.synchronize(device)
    _barrier(ws)
    ms = _max_over_ranks(e0.elapsed_time(e1), ws, device)
    total_weights = WEIGHTS * len(CALLS) * args.steps * ws
    value = total_weights / (ms / 1e3) / 1e9
    clk = clk_s.summary()

    # ---- each call alone, CUDA events on the launching stream ----
    reps = 20
    per = {}
    for fmt, bs, meth in CALLS:
        codes, packed, dqb = outs[bs]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(stream)
        for r in range(reps):
            x = pool[r % POOL]
            L.qz_quantize(x.data_ptr(), 1, WEIGHTS // bs, bs, fmt, meth, None, 0, None, None, None,
                          codes.data_ptr(), packed.data_ptr(), dqb.data_ptr(), sp)
        ev[1].record(stream)
        torch.cuda.synchronize(device)
        per[(fmt, bs, meth)] = ev[0].elapsed_time(ev[1]) / reps

    # ---- end to end through the public API from host (pinned) buffers ----
    # qwantize_b200.pipeline.HostBatchQuantizer: H2D copy, kernel and D2H copy
    # of consecutive calls overlap on three streams; every step copies each of
    # its 8 inputs in and its native outputs (scale bytes, nibbles, bf16
    # dequant) out.
    from qwantize_b200.pipeline import HostBatchQuantizer
    host_pool = [p.cpu().pin_memory() for p in pool]
    hq = HostBatchQuantizer(WEIGHTS, device=device, slots=3)
    items = [(host_pool[k].reshape(M, K // b, b), FMT_NAME[f], METH_NAME[m], b)
             for k, (f, b, m) in enumerate(CALLS)]
    outs_h = [(torch.empty(WEIGHTS // b, dtype=torch.uint8, pin_memory=True),
               torch.empty(WEIGHTS // 2, dtype=torch.uint8, pin_memory=True),
               torch.empty(WEIGHTS, dtype=torch.bfloat16, pin_memory=True)) for (_, _, _, b) in items]
    h2d = sum(w.numel() * 2 for (w, _, _, _) in items)
    d2h = sum(sum(t.numel() * t.element_size() for t in o) for o in outs_h)
    hq.run_items(items, outs_h)  # warm-up
    torch.cuda.synchronize(device)
    _barrier(ws)
    e2e_steps = max(3, min(args.steps, 10))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        hq.run_items(items, outs_h)
    torch.cuda.synchronize(device)
    e2e_ms = _max_over_ranks((time.perf_counter() - t0) * 1e3, ws, device)
    e2e_value = WEIGHTS * len(CALLS) * e2e_steps * ws / (e2e_ms / 1e3) / 1e9
    del host_pool, hq, outs_h

    cpu, counts = None, None
    if rank == 0 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        dt, w, counts = cpu_oracle_workload(threads)
        cpu = {"value": w / dt / 1e9, "unit": "G weights/s", "cores": threads, "kind": "port",
               "sample": "the full config-1 workload once (8 quantizations of 24.9M weights)",
               "seconds": dt, "reference_torch": reference_torch_sample(threads)}

    hbm_peak, tf_burst, tf_sus, peak_kind = measured_peaks()
    extra = None
    if not args.no_extras:
        del pool
        torch.cuda.empty_cache()
        extra = extras(ws, rank, device, (tf_burst, tf_sus), args)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value, "unit": "G weights/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1: nvfp4+mxfp4 x bs16+bs32 x naive+optimal, 2560x9728 bf16 weight per call, native outputs",
                       "weights_per_step_per_gpu": WEIGHTS * len(CALLS), "parallelism": f"independent x{ws}",
                       "l2": "each call reads a different weight of an 8-weight pool (400 MB > L2)"},
            "gpu_launches": len(CALLS) * args.steps,
            "per_kernel_ms": {f"{FMT_NAME[f]}_{METH_NAME[m]}_bs{b}": v for (f, b, m), v in per.items()},
            "roofline": roofline(per, counts, clk.get("sm_mhz") or 1965.0, n_sms, hbm_peak, peak_kind),
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "G weights/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "path": "qwantize_b200.pipeline.HostBatchQuantizer (pinned host in/out, 3 overlapping streams), host wall clock"},
            "clocks": clk,
            "extras": extra,
        }
        if extra and "config3_qwen3_4b_stack" in extra:
            c3 = extra["config3_qwen3_4b_stack"]
            line["strong_scaling"] = {"workload": "config3: Qwen3-4B stack, NVFP4 bs16 SSE-optimal, rows sharded",
                                      "value": c3["gweights_per_s"], "unit": "G weights/s", "n_gpus": ws,
                                      "one_gpu_same_run": c3.get("one_gpu_gweights_per_s")}
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


def _stack(layer_spec, n_layers, ws, rank, device, seed_base=0):
    """This rank's row shards of every matrix of the stack."""
    from qwantize_b200.distributed import shard_range
    from qwantize_b200.synthetic import layer_seed, make_weight_device
    mats = []
    for layer in range(n_layers):
        for name, Mo, Ki in layer_spec:
            r0, r1 = shard_range(Mo, ws, rank)
            mats.append(make_weight_device(r1 - r0, Ki, layer_seed(layer, name, seed_base), device))
    return mats


def extras(ws, rank, device, peak_tf, args):
    """Configs 2, 3 and 4 on the same GPUs (device-timed, max over ranks)."""
    import qwantize_b200 as q
    from qwantize_b200 import _lib
    from qwantize_b200.core import quantize_native
    from qwantize_b200.distributed import shard_range, token_chunks
    from qwantize_b200.hessian import gram
    from qwantize_b200.metrics import output_error_sums
    from qwantize_b200.synthetic import (LLAMA3_70B_LAYER, LLAMA3_70B_LAYERS, QWEN3_4B_LAYER, QWEN3_4B_LAYERS,
                                         make_activations, make_weight_device)
    stream = torch.cuda.current_stream(device)
    sp = stream.cuda_stream
    Lq = _lib.load()
    out = {}
    Kx = 9728
    n_w = 2560 * Kx
    # ---- NVINT4 / INT8 on the config-1 weight (native outputs), timed first,
    # before the long GEMMs below bring the clocks under the power cap
    W = make_weight_device(2560, Kx, 0, device)
    ints = {}
    c_buf = torch.empty(n_w // 16, dtype=torch.uint8, device=device)
    p_buf = torch.empty(n_w, dtype=torch.uint8, device=device)
    d_buf = torch.empty(n_w, dtype=torch.bfloat16, device=device)
    for fmt, tag, bss in ((_lib.FMT_NVINT4, "nvint4", (16, 32)), (_lib.FMT_INT8, "int8", (32, 64, 128, 256))):
        for bs in bss:
            for meth, mname in ((0, "naive"), (1, "optimal")):
                def run_int(fmt=fmt, bs=bs, meth=meth):
                    Lq.qz_quantize(W.data_ptr(), 1, n_w // bs, bs, fmt, meth, None, 0, None, None, None,
                                   c_buf.data_ptr(), p_buf.data_ptr(), d_buf.data_ptr(), sp)
                ms_i = _ev_time(run_int, stream, 5)
                ints[f"{tag}_{mname}_bs{bs}_ms"] = ms_i
                ints[f"{tag}_{mname}_bs{bs}_gweights_per_s"] = n_w / (ms_i / 1e3) / 1e9
    out["config1_int_formats"] = ints
    del c_buf, p_buf, d_buf

    # ---- config 3: the Qwen3-4B stack, rows sharded, one grouped launch ----
    mats = _stack(QWEN3_4B_LAYER, min(args.stack_layers, QWEN3_4B_LAYERS), ws, rank, device)
    n_local = sum(m.numel() for m in mats)
    outs3 = [(torch.empty(m.numel() // 16, dtype=torch.uint8, device=device),
              torch.empty(m.numel() // 2, dtype=torch.uint8, device=device)) for m in mats]
    items = (_lib.QzQuantItem * len(mats))()
    for it, m, (c, p) in zip(items, mats, outs3):
        it.x, it.n_blocks, it.scale_codes, it.packed = m.data_ptr(), m.numel() // 16, c.data_ptr(), p.data_ptr()

    def stack_grouped():
        _lib.check(Lq.qz_quantize_grouped(items, len(mats), 1, 16, 0, 1, sp), "qz_quantize_grouped")

    def stack_loop():
        for m, (c, p) in zip(mats, outs3):
            Lq.qz_quantize(m.data_ptr(), 1, m.numel() // 16, 16, 0, 1, None, 0, None, None, None,
                           c.data_ptr(), p.data_ptr(), None, sp)
    _barrier(ws)
    ms_g = _max_over_ranks(_ev_time(stack_grouped, stream, 3), ws, device)
    _barrier(ws)
    ms_l = _max_over_ranks(_ev_time(stack_loop, stream, 3), ws, device)
    n_total = int(_sum_over_ranks(n_local, ws, device))
    c3 = {"weights": n_total, "ms": ms_g, "gweights_per_s": n_total / (ms_g / 1e3) / 1e9,
          "launches_per_rank": (len(mats) + 255) // 256,
          "per_matrix_launches_ms": ms_l, "per_matrix_launches_gweights_per_s": n_total / (ms_l / 1e3) / 1e9,
          "method": "nvfp4 bs16 SSE-optimal, scale bytes + packed codes", "sharding": f"rows over {ws} rank(s)"}
    del mats, outs3, items
    torch.cuda.empty_cache()
    if ws > 1:
        # the unsharded stack on rank 0 alone, in the same run (1-GPU figure)
        if rank == 0:
            mats1 = _stack(QWEN3_4B_LAYER, min(args.stack_layers, QWEN3_4B_LAYERS), 1, 0, device)
            o1 = [(torch.empty(m.numel() // 16, dtype=torch.uint8, device=device),
                   torch.empty(m.numel() // 2, dtype=torch.uint8, device=device)) for m in mats1]
            it1 = (_lib.QzQuantItem * len(mats1))()
            for it, m, (c, p) in zip(it1, mats1, o1):
                it.x, it.n_blocks, it.scale_codes, it.packed = m.data_ptr(), m.numel() // 16, c.data_ptr(), p.data_ptr()
            ms1 = _ev_time(lambda: Lq.qz_quantize_grouped(it1, len(mats1), 1, 16, 0, 1, sp), stream, 3)
            c3["one_gpu_ms"] = ms1
            c3["one_gpu_gweights_per_s"] = n_total / (ms1 / 1e3) / 1e9
            del mats1, o1, it1
            torch.cuda.empty_cache()
        _barrier(ws)
    out["config3_qwen3_4b_stack"] = c3

    # ---- config 4: the Llama-3-70B stack, layer by layer (each layer's row
    # shards generated, then quantized in one grouped launch, timed) ----
    if args.config4_layers > 0:
        n4 = min(args.config4_layers, LLAMA3_70B_LAYERS)
        ms4, n4_local = 0.0, 0
        for layer in range(n4):
            from qwantize_b200.synthetic import layer_seed
            mats = []
            for name, Mo, Ki in LLAMA3_70B_LAYER:
                r0, r1 = shard_range(Mo, ws, rank)
                mats.append(make_weight_device(r1 - r0, Ki, layer_seed(layer, name, 70), device))
            o4 = [(torch.empty(m.numel() // 16, dtype=torch.uint8, device=device),
                   torch.empty(m.numel() // 2, dtype=torch.uint8, device=device)) for m in mats]
            it4 = (_lib.QzQuantItem * len(mats))()
            for it, m, (c, p) in zip(it4, mats, o4):
                it.x, it.n_blocks, it.scale_codes, it.packed = m.data_ptr(), m.numel() // 16, c.data_ptr(), p.data_ptr()
            run4 = lambda: Lq.qz_quantize_grouped(it4, len(mats), 1, 16, 0, 1, sp)  # noqa: E731
            if layer == 0:
                run4()  # warm-up
            torch.cuda.synchronize(device)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            ev[0].record(stream)
            run4()
            ev[1].record(stream)
            torch.cuda.synchronize(device)
            ms4 += ev[0].elapsed_time(ev[1])
            n4_local += sum(m.numel() for m in mats)
            del mats, o4, it4
        ms4 = _max_over_ranks(ms4, ws, device)
        n4_total = int(_sum_over_ranks(n4_local, ws, device))
        out["config4_llama3_70b_stack"] = {
            "layers": n4, "weights": n4_total, "ms": ms4, "gweights_per_s": n4_total / (ms4 / 1e3) / 1e9,
            "method": "nvfp4 bs16 SSE-optimal, scale bytes + packed codes, one grouped launch per layer",
            "sharding": f"rows over {ws} rank(s)", "timing": "sum of the per-layer launch times (inputs resident)"}
        torch.cuda.empty_cache()

    # ---- config 2: tokens sharded (whole 65,536-token chunks), H-optimal ----
    T = args.gram_tokens
    t0, t1 = token_chunks(T, ws, rank)
    X = make_activations(t1 - t0, Kx, seed=1, device=device, t0=t0)
    W = make_weight_device(2560, Kx, 0, device)
    Wb = W.reshape(2560, Kx // 16, 16)
    Hb = torch.empty(Kx // 16, 16, 16, device=device)
    r0, r1 = shard_range(2560, ws, rank)

    def hopt(fmt):
        # block-diagonal Gram of this rank's tokens, all-reduce, then this
        # rank's rows of the search (native outputs)
        gram(X, "blockdiag", 16, out=Hb)
        if ws > 1:
            torch.distributed.all_reduce(Hb)
        return quantize_native(Wb[r0:r1], -1, False, fmt, _lib.METHOD_HESSIAN, H_blocks=Hb)
    _barrier(ws)
    ms_diag, diag_how = _graph_time(lambda: gram(X, "blockdiag", 16, out=Hb), stream, 3, ws, device)
    _barrier(ws)
    hopt_nv, hopt_how = _graph_time(lambda: hopt(_lib.FMT_NVFP4), stream, 3, ws, device)
    _barrier(ws)
    hopt_mx, _ = _graph_time(lambda: hopt(_lib.FMT_MXFP4), stream, 3, ws, device)
    ar_bd = None
    if ws > 1:
        _barrier(ws)
        ar_bd = _max_over_ranks(_ev_time(lambda: torch.distributed.all_reduce(Hb), stream, 3), ws, device)
    # the search alone on the full weight (one GPU's share when N = 1)
    ms_nv = _ev_time(lambda: q.nvfp4_optimal_hessian(Wb, H_blocks=Hb), stream, 3)
    ms_mx = _ev_time(lambda: q.mxfp4_optimal_hessian(Wb, H_blocks=Hb), stream, 3)
    out["config1_int_formats"]["nvint4_hoptimal_bs16_search_ms"] = _ev_time(
        lambda: q.nvint4_optimal_hessian(Wb, H_blocks=Hb), stream, 3)
    from qwantize_b200.core import admm_fp32
    from qwantize_b200.hessian import admm_setup
    Hn, Minv = admm_setup(Hb)
    ms_admm = _ev_time(lambda: admm_fp32(Wb, -1, False, Hb, Hn, Minv), stream, 3)
    H = torch.empty(Kx, Kx, device=device)
    _barrier(ws)
    ms_full = _max_over_ranks(_ev_time(lambda: gram(X, "full", out=H), stream, 3), ws, device)
    ar_ms = None
    if ws > 1:
        # the reduction of distributed.gram_sharded: the upper 256 x 256 tiles
        # (about half of H) all-reduced, then expanded to the symmetric H
        from qwantize_b200.hessian import unpack_upper_tiles
        P = gram(X, "upper_tiles")

        def reduce_full():
            torch.distributed.all_reduce(P)
            unpack_upper_tiles(P, Kx, out=H)
        _barrier(ws)
        ar_ms = _max_over_ranks(_ev_time(reduce_full, stream, 3), ws, device)
        del P
    flop = T * Kx * (Kx + 1)
    out["config2_gram"] = {
        "tokens": T, "K": Kx, "ms_full": ms_full, "tflops_full_whole_job": flop / ms_full / 1e9,
        "tflops_full_per_gpu": flop / ms_full / 1e9 / ws,
        # a ~100 ms kernel runs under the power cap: the sustained peak is its denominator
        "frac_of_measured_bf16_peak_sustained": flop / ms_full / 1e9 / ws / peak_tf[1],
        "frac_of_measured_bf16_peak_burst": flop / ms_full / 1e9 / ws / peak_tf[0],
        "ms_blockdiag": ms_diag, "blockdiag_timing": diag_how, "blockdiag_GBps": 2 * (t1 - t0) * Kx / ms_diag / 1e6,
        "allreduce_full_H_ms": ar_ms, "allreduce_blockdiag_H_ms": ar_bd,
        "full_H_reduction": "upper 256x256 tiles all-reduced (about half of H), then expanded",
        "sharding": f"tokens over {ws} rank(s), whole 65536-token chunks"}
    _, _, dq = q.nvfp4_optimal(Wb, return_dequant=True)
    dqb = dq.reshape(2560, Kx).to(torch.bfloat16)
    _barrier(ws)
    ms_m = _max_over_ranks(_ev_time(lambda: output_error_sums(W, dqb, X), stream), ws, device)
    mflop = 4 * (t1 - t0) * Kx * 2560
    out["config2_hopt"] = {
        "weights": n_w,
        "nvfp4_hopt_ms": hopt_nv, "nvfp4_hopt_gweights_per_s": n_w / (hopt_nv / 1e3) / 1e9,
        "mxfp4_hopt_ms": hopt_mx, "mxfp4_hopt_gweights_per_s": n_w / (hopt_mx / 1e3) / 1e9,
        "hopt_pipeline": "block-diagonal Gram of this rank's tokens + all-reduce + this rank's rows of the "
                         "search, one timed region, max over ranks",
        "hopt_timing": hopt_how,
        "nvfp4_bs16_search_full_weight_ms": ms_nv, "mxfp4_bs16_search_full_weight_ms": ms_mx,
        "nvfp4_admm_bs16_ms": ms_admm,
        "metrics_output_error_ms": ms_m, "metrics_tflops_per_gpu": mflop / ms_m / 1e9,
        "metrics_frac_of_measured_bf16_peak_sustained": mflop / ms_m / 1e9 / peak_tf[1]}
    del dq, dqb, Hn, Minv
    # GPTQ (NVFP4 bs16 SSE-optimal) of the 2560x9728 weight on the full H / T
    from qwantize_b200.gptq import gptq
    H.div_(T)
    t_g = time.perf_counter()
    gptq(W, H, "nvfp4", "optimal", 16)  # the first call also loads the solver libraries
    torch.cuda.synchronize()
    out["config2_hopt"]["gptq_nvfp4_optimal_bs16_first_call_ms"] = (time.perf_counter() - t_g) * 1e3
    t_g = time.perf_counter()
    gptq(W, H, "nvfp4", "optimal", 16)
    torch.cuda.synchronize()
    out["config2_hopt"]["gptq_nvfp4_optimal_bs16_ms"] = (time.perf_counter() - t_g) * 1e3
    del X, H
    torch.cuda.empty_cache()

    # ---- the drop-in fp32 API end to end from host memory: the call a
    # reference user makes, nvfp4_optimal(W_cpu, return_dequant=True), with a
    # pageable CPU weight in and fp32 scales / quants / dequant back ----
    W_cpu = W.cpu()
    Wc = W_cpu.reshape(2560, Kx // 16, 16)
    q.nvfp4_optimal(Wc, return_dequant=True)
    torch.cuda.synchronize()
    reps = 5
    kept = []  # a caller quantizing a model keeps every result
    t_d = time.perf_counter()
    for _ in range(reps):
        kept.append(q.nvfp4_optimal(Wc, return_dequant=True))
    torch.cuda.synchronize()
    ms_d = (time.perf_counter() - t_d) * 1e3 / reps
    s_, q_, d_ = kept[-1]
    del kept
    out["dropin_fp32_e2e"] = {
        "call": "nvfp4_optimal(W_cpu, return_dequant=True), bs16, 2560x9728 bf16 pageable host weight, "
                "results kept (pageable CPU tensors)",
        "ms": ms_d, "gweights_per_s": n_w / (ms_d / 1e3) / 1e9,
        "h2d_bytes": n_w * 2, "d2h_bytes": n_w * 8 + n_w // 16 * 4, "timing": "host wall clock, synchronized"}
    del W_cpu, Wc, s_, q_, d_, W, Wb, Hb
    torch.cuda.empty_cache()

    # ---- config 4 H-optimal: the 8192x28672 down_proj with its full 28672^2
    # H, built token-sharded and all-reduced; the search uses H's diagonal
    # blocks, rows sharded ----
    if args.config4_tokens > 0:
        K4, M4, T4 = 28672, 8192, args.config4_tokens
        a0, a1 = token_chunks(T4, ws, rank)
        X4 = make_activations(a1 - a0, K4, seed=4, device=device, t0=a0)
        H4 = torch.empty(K4, K4, device=device)
        _barrier(ws)
        ms_g4 = _max_over_ranks(_ev_time(lambda: gram(X4, "full", out=H4), stream, 2), ws, device)
        ar4 = None
        if ws > 1:
            from qwantize_b200.hessian import unpack_upper_tiles
            P4 = gram(X4, "upper_tiles")

            def reduce_full4():
                torch.distributed.all_reduce(P4)
                unpack_upper_tiles(P4, K4, out=H4)
            _barrier(ws)
            ar4 = _max_over_ranks(_ev_time(reduce_full4, stream), ws, device)
            del P4
        del X4
        torch.cuda.empty_cache()
        W4 = make_weight_device(M4, K4, 7, device).reshape(M4, K4 // 16, 16)
        J4 = K4 // 16
        Hb4 = H4.reshape(J4, 16, J4, 16).diagonal(dim1=0, dim2=2).permute(2, 0, 1).contiguous()
        s0, s1 = shard_range(M4, ws, rank)
        _barrier(ws)
        ms_s4 = _max_over_ranks(_ev_time(
            lambda: quantize_native(W4[s0:s1], -1, False, _lib.FMT_NVFP4, _lib.METHOD_HESSIAN, H_blocks=Hb4),
            stream, 3), ws, device)
        f4 = T4 * K4 * (K4 + 1)
        tot = ms_g4 + (ar4 or 0.0) + ms_s4
        out["config4_hopt_down_proj"] = {
            "tokens": T4, "K": K4, "M": M4, "ms_full_gram": ms_g4, "tflops_full_per_gpu": f4 / ms_g4 / 1e9 / ws,
            "frac_of_measured_bf16_peak_sustained": f4 / ms_g4 / 1e9 / ws / peak_tf[1],
            "allreduce_full_H_ms": ar4, "H_bytes": K4 * K4 * 4,
            "allreduced_bytes": ((K4 + 255) // 256) * ((K4 + 255) // 256 + 1) // 2 * 65536 * 4,
            "nvfp4_search_ms": ms_s4,
            "total_ms": tot, "gweights_per_s": M4 * K4 / (tot / 1e3) / 1e9,
            "sharding": f"tokens over {ws} rank(s) for H, rows for the search"}
        del H4, Hb4, W4
        torch.cuda.empty_cache()
    return out


def profile_call(spec):
    """Three launches of one quantization of the config-1 weight (native
    outputs), for ncu captures of a single kernel: spec "fmt,bs,method", e.g.
    "nvfp4,16,optimal" or "int8,32,optimal" ("hoptimal": the Hessian search with
    H blocks from 65,536 config-2 tokens); "gram" runs three full Grams of
    65,536 tokens, "gptq" one GPTQ of the config weight."""
    from qwantize_b200 import _lib
    from qwantize_b200.synthetic import make_weight_device
    if spec == "gram":  # three full Grams of 65,536 config-2 tokens (X 1.27 GB)
        from qwantize_b200.hessian import gram
        from qwantize_b200.synthetic import make_activations
        dev = torch.device("cuda", 0)
        X = make_activations(65536, K, seed=1, device=dev)
        for _ in range(3):
            gram(X, "full")
        torch.cuda.synchronize(dev)
        return
    if spec == "gptq":  # one GPTQ run: NVFP4 bs16 SSE-optimal, H from 65,536 tokens
        from qwantize_b200.gptq import gptq
        from qwantize_b200.hessian import gram
        from qwantize_b200.synthetic import make_activations
        dev = torch.device("cuda", 0)
        X = make_activations(65536, K, seed=1, device=dev)
        H = gram(X, "full") / 65536
        del X
        gptq(make_weight_device(M, K, 0, dev), H, "nvfp4", "optimal", 16)
        torch.cuda.synchronize(dev)
        return
    fmt, bs, meth = spec.split(",")
    fmt = {"nvfp4": 0, "mxfp4": 1, "nvint4": 3, "int8": 4}[fmt]
    bs, meth = int(bs), {"naive": 0, "optimal": 1, "hoptimal": 2}[meth]
    dev = torch.device("cuda", 0)
    L = _lib.load()
    W = make_weight_device(M, K, 0, dev)
    if meth == 2:  # Hessian search: H blocks from 65,536 config-2 tokens
        from qwantize_b200.hessian import gram
        from qwantize_b200.synthetic import make_activations
        Hb = gram(make_activations(65536, K, seed=1, device=dev), "blockdiag", bs)
        codes = torch.empty(WEIGHTS // bs, dtype=torch.uint8, device=dev)
        packed = torch.empty(WEIGHTS, dtype=torch.uint8, device=dev)
        sp = torch.cuda.current_stream(dev).cuda_stream
        for _ in range(3):
            _lib.check(L.qz_quantize(W.data_ptr(), 1, WEIGHTS // bs, bs, fmt, meth, Hb.data_ptr(), K // bs, None,
                                     None, None, codes.data_ptr(), packed.data_ptr(), None, sp), "qz_quantize")
        torch.cuda.synchronize(dev)
        return
    codes = torch.empty(WEIGHTS // bs, dtype=torch.uint8, device=dev)
    packed = torch.empty(WEIGHTS, dtype=torch.uint8, device=dev)
    dq = torch.empty(WEIGHTS, dtype=torch.bfloat16, device=dev)
    sp = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(3):
        _lib.check(L.qz_quantize(W.data_ptr(), 1, WEIGHTS // bs, bs, fmt, meth, None, 0, None, None, None,
                                 codes.data_ptr(), packed.data_ptr(), dq.data_ptr(), sp), "qz_quantize")
    torch.cuda.synchronize(dev)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip configs 2, 3 and 4")
    ap.add_argument("--gram-tokens", type=int, default=1048576,
                    help="tokens for the config-2 extras (smaller for profiling runs)")
    ap.add_argument("--stack-layers", type=int, default=36,
                    help="layers of the config-3 stack (smaller for profiling runs)")
    ap.add_argument("--config4-layers", type=int, default=80,
                    help="layers of the config-4 Llama-3-70B stack (0 skips it)")
    ap.add_argument("--config4-tokens", type=int, default=262144,
                    help="tokens for config 4's full 28672^2 Gram (0 skips it)")
    ap.add_argument("--profile-call", default=None,
                    help='only launch one quantization three times (ncu captures), e.g. "int8,32,optimal"; '
                         '"nvfp4,16,hoptimal" the Hessian search, "gram" three full Grams of 65,536 tokens, "gptq" one GPTQ of the config weight')
    args = ap.parse_args()
    if args.profile_call:
        profile_call(args.profile_call)
    elif args.impl == "reference":
        bench_reference(args)
    else:
        bench_ours(args)


if __name__ == "__main__":
    main()
