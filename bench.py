#!/usr/bin/env python3
"""Benchmark of the Enigma hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-ops]

Headline (BASELINE metric, config 2 at its largest size): bf16 RMSNorm over
x [262144, 8192] (fp32 accumulate, eps 1e-6), HBM GB/s, one kernel launch per
step.  Bytes per step are the algorithmic ones: read x once, write y once,
read w once (4*rows*hidden + 2*hidden).  Inputs (4 GiB each way) are larger
than the 126 MB L2, so no flush is needed between steps.

With N > 1 (launched under torchrun, one rank per GPU) the 262144 rows are
split across the ranks (strong scaling, no collective on the data path); the
timed region is bracketed by a barrier and cuda synchronize, the elapsed time
is the max over ranks, and the NCCL all-gather of y is timed on its own.

`ops` in the JSON line adds the other hot-path operators at their BASELINE
headline sizes, sharded the same way across the ranks (GEMM bf16 8192^3 by
M-blocks, SDPA bf16 [8,32,8192,128] by batch, the decode step by sequences),
with the all-gather of each output timed separately.

--impl reference times the reference's own CPU formulation of the same
operator (the fp32 numpy check of examples/benchmark_rmsnorm.py:115-116) on
all the host's cores, on a bounded row sample per step.
"""
from __future__ import annotations

import argparse
import ctypes
import functools
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "enigma-dsl_b200"))

ROWS, HIDDEN, EPS = 262144, 8192, 1e-6
METRIC = "RMSNorm HBM GB/s (bf16 262144x8192, fp32 accumulate)"
BYTES_PER_STEP = 4 * ROWS * HIDDEN + 2 * HIDDEN
# DRAM bytes (read + write) per algorithmic byte of one rmsnorm launch, from an ncu capture
# (dram__bytes_read.sum 4.30 GB + dram__bytes_write.sum 4.25 GB, one pass) of the full
# 262144 x 8192 launch; scaled by bytes for the smaller row shards of N > 1.  Writes still
# held in L2 when the kernel ends are not in the capture, so it reads slightly below 1.
NCU_TRAFFIC_PER_BYTE = 8.55e9 / 8_589_950_976
NCU_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the full 262144 x "
                      "8192 launch (3 significant digits), scaled by bytes for smaller shards")


def _set_rows(rows: int) -> None:
    global ROWS, BYTES_PER_STEP, METRIC
    ROWS = rows
    BYTES_PER_STEP = 4 * ROWS * HIDDEN + 2 * HIDDEN
    METRIC = f"RMSNorm HBM GB/s (bf16 {ROWS}x{HIDDEN}, fp32 accumulate)"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and throttle-reason sampling during the timed region (read-only).

    The GPU is found by its UUID (the torch device index differs from the physical one
    under CUDA_VISIBLE_DEVICES).  NVML is polled every 10 ms; without NVML, nvidia-smi
    every 200 ms."""

    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    # NVML clocks-event-reason bits, in the order of Q's reason columns.
    BITS = (0x8, 0x40, 0x20, 0x4)

    def __init__(self, index: int):
        self.index = index
        self.uuid = None
        try:
            import torch
            u = str(torch.cuda.get_device_properties(index).uuid)
            self.uuid = u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            pass
        self.samples = []
        self._stop = threading.Event()
        self._ready = threading.Event()   # set once the first sample is in
        self._t = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        if self.uuid:
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(self.uuid.encode())
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _run(self):
        try:
            nv, h = self._nvml_handle()
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self._stop.is_set():
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = reasons(h)
                self.samples.append([str(sm), str(mx)] +
                                    ["Active" if r & bit else "Not Active" for bit in self.BITS])
                self._ready.set()
                self._stop.wait(0.01)
            return
        except Exception:
            pass
        dev = self.uuid or str(self.index)
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", "-i", dev, f"--query-gpu={self.Q}",
                     "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5
                ).stdout.strip()
                if out:
                    self.samples.append([s.strip() for s in out.split(",")])
                    self._ready.set()
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        # NVML start-up can outlast a short timed region: begin it once sampling runs.
        self._ready.wait(timeout=3.0)
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit())
        mx = max((float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()),
                 default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 2 + i and s[2 + i].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------------------- dist plumbing
def _dist_init(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _time_device(fn, steps, stream):
    """Average device ms of fn() over `steps` launches, CUDA events on `stream`."""
    import torch
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(steps):
        fn()
    e.record(stream)
    e.synchronize()
    return s.elapsed_time(e) / steps


def _time_device_flushed(fn, steps, stream):
    """Average device ms of fn() with L2 flushed before every launch: a 256 MB buffer
    (twice the 126 MB L2) is read between steps, outside the events, so each step reads
    its inputs from HBM.  The flush reads rather than writes: a written buffer would leave
    L2 full of dirty lines whose write-back the timed step would pay for."""
    import torch
    flush = torch.ones(64 << 20, dtype=torch.int32, device="cuda")
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for s, e in evs:
        flush.max()
        s.record(stream)
        fn()
        e.record(stream)
    evs[-1][1].synchronize()
    return sum(s.elapsed_time(e) for s, e in evs) / steps


# ----------------------------------------------------------------------------- CPU baseline
def _host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


@functools.lru_cache(maxsize=2)
def _cpu_inputs(sample_rows: int):
    """Seeded bf16-rounded x [sample_rows, HIDDEN] and w, made once per size."""
    import numpy as np
    from oracle import numerics as orc
    rng = np.random.default_rng(0)
    x = orc.bf16_round(rng.standard_normal((sample_rows, HIDDEN), dtype=np.float32))
    w = orc.bf16_round((1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32))
    return x, w


def _cpu_rmsnorm_rate(sample_rows: int, threads: int, min_seconds: float, passes: int = 0):
    """Time the reference's own RMSNorm formula (examples/benchmark_rmsnorm.py:115-116, fp32
    numpy, as oracle/numerics.py:rmsnorm_fp32 writes it) over a `sample_rows`-row sample of
    the workload, rows split across `threads` Python threads (numpy releases the GIL in its
    kernels).  Repeats whole passes until `min_seconds` have elapsed (or `passes` passes).
    Returns (seconds, rows processed)."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle import numerics as orc
    x, w = _cpu_inputs(sample_rows)
    chunks = [c for c in np.array_split(np.arange(sample_rows), threads * 4) if len(c)]

    def work(idx):
        orc.rmsnorm_fp32(x[idx[0]:idx[-1] + 1], w, EPS)

    done, t0 = 0, time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            list(ex.map(work, chunks))
            done += sample_rows
            el = time.perf_counter() - t0
            if (passes and done >= passes * sample_rows) or (not passes and el >= min_seconds):
                return el, done


def _cpu_sample_text(rows_done, dt, threads, sample_rows):
    return (f"{rows_done} rows x {HIDDEN} in {dt:.1f} s ({threads} threads): repeated passes "
            f"over a seeded {sample_rows}-row sample of the {ROWS}-row workload, the reference's fp32 "
            f"numpy formula (examples/benchmark_rmsnorm.py:115-116) on bf16-rounded values; "
            f"GB/s counts the workload's bf16 bytes (4 per element + w)")


def _cpu_baseline(sample_rows=16384, min_seconds=10.0):
    threads = _host_threads()
    dt, rows = _cpu_rmsnorm_rate(sample_rows, threads, min_seconds)
    gbs = (4 * rows * HIDDEN) / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": _cpu_sample_text(rows, dt, threads, sample_rows)}


def _config(world: int) -> dict:
    """The workload description both arms print (the same dict)."""
    return {"workload": f"rmsnorm bf16 rows={ROWS} hidden={HIDDEN} eps={EPS}, rows sharded "
                        f"across {world} GPU(s)",
            "rows_total": ROWS, "hidden": HIDDEN, "parallelism": f"row-shard x{world}",
            "l2": "inputs larger than L2 (126 MB) at every N; no flush",
            "bytes_per_step_total": BYTES_PER_STEP}


# ----------------------------------------------------------------------------- our arm
def _timed_max(fn, steps, world, stream, flushed=False):
    """Device ms per step of fn() on this rank (CUDA events on `stream`), bracketed by a
    barrier and synchronize, and the max of that over ranks."""
    import torch
    torch.cuda.synchronize()
    _barrier(world)
    ms = (_time_device_flushed if flushed else _time_device)(fn, steps, stream)
    torch.cuda.synchronize()
    _barrier(world)
    return ms, _max_over_ranks(ms, world)


def _allgather_ms(local, world, reps=3):
    """NCCL all-gather of this rank's output shard into the full tensor on every rank,
    timed alone (max over ranks); the only collective of the sharded path."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return None
    full = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                       device=local.device)
    dist.all_gather_into_tensor(full, local)
    ms, ms_max = _timed_max(lambda: dist.all_gather_into_tensor(full, local), reps, world,
                            torch.cuda.current_stream())
    nbytes = full.numel() * full.element_size()
    del full
    # bus bandwidth convention of nccl-tests: (world-1)/world of the gathered bytes cross links
    return {"ms": round(ms_max, 4), "bytes_gathered": nbytes,
            "busbw_gbs": round(nbytes * (world - 1) / world / (ms_max * 1e-3) / 1e9, 1)}


def _settle(seconds=2.0):
    """Idle the GPU before an operator's timed region, so each one starts from the power
    state it has when run on its own: right after the seconds-long GEMM and SDPA loops at
    the 1 kW cap, the next operator measured ~10 % slower with the sampled SM clock still
    at its maximum (SDPA causal 8192: 1028 against 1118-1147 TFLOP/s alone, same box)."""
    import torch
    torch.cuda.synchronize()
    time.sleep(seconds)


def _ops_side(world, rank, hbm_peak, tc_peak, peak_kind):
    """GEMM, SDPA and the decode step at their BASELINE headline sizes, sharded the way
    BASELINE configs 3-5 shard them: GEMM 8192^3 by M-blocks (B replicated, placed before
    timing), SDPA [8,32,8192,128] by batch (whole (b, h) slices), decode batch 64 by
    sequences (weights replicated).  Every rank runs its shard; the time is the max over
    ranks and the value is the whole problem's work over that time.  At N = 1 these are
    the single-GPU figures."""
    import torch
    from enigma import cuda_ops, shard
    res = {}
    stream = torch.cuda.current_stream()
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    lo, hi = shard.shard_range(n, world, rank)
    a = (torch.randn(n, n, device="cuda", generator=g)[lo:hi] / math.sqrt(n)).bfloat16()
    b = torch.randn(n, n, device="cuda", generator=g).bfloat16()
    c = torch.empty(hi - lo, n, dtype=torch.bfloat16, device="cuda")
    fn = lambda: cuda_ops.gemm(a, b, out=c)  # noqa: E731
    _settle()
    for _ in range(3):
        fn()
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms, ms_max = _timed_max(fn, 20, world, stream)
    tf = 2 * n ** 3 / (ms_max * 1e-3) / 1e12
    res["gemm_bf16_8192"] = {
        "tflops": round(tf, 1), "ms": round(ms_max, 4), "n_gpus": world,
        "rows_per_gpu": hi - lo, "frac": round(tf / world / tc_peak, 4), "peak": tc_peak,
        "peak_kind": peak_kind + " burst, per GPU", "clocks": clk.summary(),
        "allgather_C": _allgather_ms(c, world)}
    # cuBLAS (torch.matmul) on the same shard, timed the same way: the library reference point.
    ref = lambda: torch.matmul(a, b, out=c)  # noqa: E731
    _settle()
    for _ in range(3):
        ref()
    _, ms_ref = _timed_max(ref, 20, world, stream)
    res["gemm_bf16_8192"]["cublas_same_loop_tflops"] = round(2 * n ** 3 / (ms_ref * 1e-3) / 1e12, 1)
    res["gemm_bf16_8192"]["vs_cublas_same_loop"] = round(ms_ref / ms_max, 4)
    del a, b, c
    B, H, S, D = 8, 32, 8192, 128
    blo, bhi = shard.shard_range(B, world, rank)
    q, k, v = (torch.randn(bhi - blo, H, S, D, device="cuda", generator=g).bfloat16()
               for _ in range(3))
    o = torch.empty_like(q)
    for causal in (True, False):
        fn = lambda: cuda_ops.sdpa(q, k, v, causal=causal, out=o)  # noqa: E731
        _settle()
        for _ in range(3):
            fn()
        with ClockSampler(torch.cuda.current_device()) as clk:
            ms, ms_max = _timed_max(fn, 10, world, stream)
        fl = (2 if causal else 4) * B * H * S * S * D
        tf = fl / (ms_max * 1e-3) / 1e12
        res[f"sdpa_bf16_{'causal' if causal else 'noncausal'}_8x32x8192x128"] = {
            "tflops": round(tf, 1), "ms": round(ms_max, 3), "n_gpus": world,
            "batch_per_gpu": bhi - blo, "frac": round(tf / world / tc_peak, 4),
            "flops_convention": "causal 2*B*H*S^2*D, non-causal 4*B*H*S^2*D",
            "clocks": clk.summary(),
            "allgather_O": _allgather_ms(o, world) if not causal else None}
        # cuDNN fused attention on the same shard (torch SDPA, cuDNN backend), timed the same way.
        _settle()
        ref_ms = _cudnn_sdpa_ms(q, k, v, causal, 3, 10, stream)
        # every rank joins the max (1e30 stands for "backend refused"), so none waits alone
        ref_ms = _max_over_ranks(1e30 if ref_ms is None else ref_ms, world)
        if ref_ms < 1e29:
            key = f"sdpa_bf16_{'causal' if causal else 'noncausal'}_8x32x8192x128"
            res[key]["cudnn_same_loop_tflops"] = round(fl / (ref_ms * 1e-3) / 1e12, 1)
            res[key]["vs_cudnn_same_loop"] = round(ref_ms / ms_max, 4)
    del q, k, v, o
    _settle()
    res["decode_layer_config5"] = _decode_side(hbm_peak, world, rank)
    return res


def _decode_side(hbm_peak, world=1, rank=0):
    """one decode step, batch 64 (split by sequences across ranks),
    2048-token KV cache (HBM-bound)."""
    import torch
    from enigma.decode_layer import DecodeConfig, DecodeLayer
    full = DecodeConfig()
    if world > 1:
        from enigma import shard
        cfg = shard.decode_shard_config(full)
    else:
        cfg = full
    layer = DecodeLayer.random(cfg, seed=0)
    x = torch.randn(cfg.batch, cfg.hidden, device="cuda").bfloat16()
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    fn = layer.capture(x, out)
    for _ in range(5):
        fn()
    _, ms = _timed_max(fn, 50, world, stream, flushed=True)
    _, ms_warm = _timed_max(fn, 50, world, stream)
    kv = 2 * cfg.batch * cfg.heads_kv * (cfg.cache_len + 1) * cfg.head_dim * 2
    byts = layer.weight_bytes() + kv   # this rank's bytes per step
    del layer
    stack = _decode_stack(cfg, world, stream)
    return {"ms": round(ms, 4), "tokens_per_s": round(full.batch / (ms * 1e-3), 1),
            "n_gpus": world, "batch_per_gpu": cfg.batch,
            "algorithmic_bytes_per_gpu": byts, "gbs_per_gpu": round(byts / (ms * 1e-3) / 1e9, 1),
            "frac_hbm": round(byts / (ms * 1e-3) / 1e9 / hbm_peak, 4),
            "l2": "flushed (256 MB read) before every step",
            "ms_back_to_back": round(ms_warm, 4),
            "note": "weights (replicated) + this rank's KV read once per step; back to back, "
                    "L2 (126 MB) can hold part of the 97 MB working set",
            "stack": stack | {"gbs_per_gpu": round(byts / (stack["ms_per_layer"] * 1e-3) / 1e9, 1),
                              "frac_hbm": round(byts / (stack["ms_per_layer"] * 1e-3) / 1e9
                                                / hbm_peak, 4)}}


def _decode_stack(cfg, world, stream, n_layers=8):
    """The same step as one layer of a model: n_layers distinct layers (own weights and KV
    caches, ~0.78 GB together, six times the 126 MB L2, so no flush is needed) chained
    out -> x in one CUDA graph, the way a serving step runs a layer stack; time per layer =
    graph time / n_layers.  The single-layer figure above pays the graph launch and the
    event pair once per layer; here they are paid once per stack."""
    import torch
    from enigma.decode_layer import DecodeLayer
    layers = [DecodeLayer.random(cfg, seed=100 + i) for i in range(n_layers)]
    xs = [torch.randn(cfg.batch, cfg.hidden, device="cuda").bfloat16()]
    xs += [torch.empty_like(xs[0]) for _ in range(n_layers)]

    def chain():
        for i, lyr in enumerate(layers):
            lyr.step(xs[i], out=xs[i + 1])

    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        chain()                      # first launches (per-device setup) outside capture
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    for _ in range(5):
        graph.replay()
    _, ms = _timed_max(graph.replay, 30, world, stream)
    del graph, layers, xs
    return {"layers": n_layers, "ms_per_layer": round(ms / n_layers, 4),
            "l2": f"{n_layers} distinct layers per graph (~{n_layers * 97} MB), larger than L2; "
                  "no flush"}


def _cudnn_sdpa_ms(q, k, v, causal, warm, steps, stream):
    """Device ms of torch's scaled_dot_product_attention restricted to the cuDNN fused
    attention backend on the same tensors (a library reference point, as cuBLAS is for the
    GEMM), or None when that backend refuses the case."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    try:
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            fn = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal)  # noqa: E731
            for _ in range(warm):
                fn()
            return _time_device(fn, steps, stream)
    except RuntimeError:
        return None


def _sdpa_tc_available() -> bool:
    from enigma import _native
    return hasattr(_native.lib(), "enigma_sdpa_bf16")


def _rmsnorm_line(rows, hidden, dtype, steps, warmup, stream, hbm_peak):
    """One RMSNorm configuration (BASELINE configs 1 and 2): HBM GB/s of one read of x and
    one write of y (+ w), L2 flushed by a read before every step (small sizes fit in L2)."""
    import torch
    from enigma import cuda_ops
    g = torch.Generator(device="cuda").manual_seed(0)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    x = torch.randn(rows, hidden, device="cuda", generator=g).to(tdt)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(tdt)
    y = torch.empty_like(x)
    fn = lambda: cuda_ops.rmsnorm(x, w, EPS, out=y)  # noqa: E731
    for _ in range(warmup):
        fn()
    ms = _time_device_flushed(fn, steps, stream)
    es = x.element_size()
    byts = 2 * rows * hidden * es + hidden * es
    gbs = byts / (ms * 1e-3) / 1e9
    return {"op": "rmsnorm", "dtype": dtype, "rows": rows, "hidden": hidden, "ms": round(ms, 4),
            "value": round(gbs, 1), "unit": "GB/s", "frac_hbm": round(gbs / hbm_peak, 4),
            "timing": "L2 flushed (256 MB read) before every step"}


def run_sweep(args):
    """Every BASELINE configuration on one GPU, one JSON line each (the headline and its
    contract fields are the default run's; these lines are the per-config table)."""
    import torch
    from enigma import cuda_ops
    cuda_ops.ensure_device(0)
    stream = torch.cuda.current_stream()
    hbm_peak, tc_peak, _ = _peaks()
    steps, warm = max(5, min(args.steps, 30)), max(3, args.warmup)
    print(json.dumps(_rmsnorm_line(4096, 4096, "f32", steps, warm, stream, hbm_peak) |
                     {"config": 1}), flush=True)
    for rows in (16384, 65536, 262144):
        for hidden in (2048, 4096, 8192):
            print(json.dumps(_rmsnorm_line(rows, hidden, "bf16", steps, warm, stream, hbm_peak) |
                             {"config": 2}), flush=True)
    g = torch.Generator(device="cuda").manual_seed(0)
    for n in (1024, 4096, 8192):
        a = (torch.randn(n, n, device="cuda", generator=g) / math.sqrt(n)).bfloat16()
        b = torch.randn(n, n, device="cuda", generator=g).bfloat16()
        c = torch.empty_like(a)
        fn = lambda: cuda_ops.gemm(a, b, out=c)  # noqa: E731
        for _ in range(warm):
            fn()
        ms = _time_device(fn, steps, stream)
        tf = 2 * n ** 3 / (ms * 1e-3) / 1e12
        # cuBLAS (torch.matmul) timed the same way, for a like-for-like reference under the
        # same clocks and power state (a comparison line, not the product path).
        ref = lambda: torch.matmul(a, b, out=c)  # noqa: E731
        for _ in range(warm):
            ref()
        ms_ref = _time_device(ref, steps, stream)
        tf_ref = 2 * n ** 3 / (ms_ref * 1e-3) / 1e12
        print(json.dumps({"config": 3, "op": "gemm_bf16", "n": n, "ms": round(ms, 4),
                          "value": round(tf, 1), "unit": "TFLOP/s",
                          "frac_tensor": round(tf / tc_peak, 4), "timing": "back to back",
                          "cublas_same_loop_tflops": round(tf_ref, 1),
                          "vs_cublas_same_loop": round(tf / tf_ref, 4)}), flush=True)
        del a, b, c
    for S in (1024, 4096, 8192):
        B, H, D = 8, 32, 128
        q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16() for _ in range(3))
        o = torch.empty_like(q)
        for causal in (True, False):
            fn = lambda: cuda_ops.sdpa(q, k, v, causal=causal, out=o)  # noqa: E731
            for _ in range(warm):
                fn()
            ms = _time_device(fn, steps, stream)
            fl = (2 if causal else 4) * B * H * S * S * D
            tf = fl / (ms * 1e-3) / 1e12
            ref = _cudnn_sdpa_ms(q, k, v, causal, warm, steps, stream)
            print(json.dumps({"config": 4, "op": "sdpa_bf16", "S": S, "causal": causal,
                              "ms": round(ms, 4), "value": round(tf, 1), "unit": "TFLOP/s",
                              "frac_tensor": round(tf / tc_peak, 4), "timing": "back to back",
                              "flops": "causal 2BHS^2D, non-causal 4BHS^2D",
                              "cudnn_same_loop_tflops": None if ref is None else
                              round(fl / (ref * 1e-3) / 1e12, 1),
                              "vs_cudnn_same_loop": None if ref is None else
                              round(ref / ms, 4)}), flush=True)
        del q, k, v, o
    print(json.dumps({"config": 5, "op": "decode_layer"} | _decode_side(hbm_peak)), flush=True)


def run_ours(args):
    import torch
    from enigma import _native, cuda_ops, shard
    rank, world, local = _dist_init(args.gpus)
    cuda_ops.ensure_device(torch.cuda.current_device())
    hbm_peak, tc_peak, peak_kind = _peaks()
    stream = torch.cuda.current_stream()

    # Config 2's rows sharded across the ranks: each GPU normalises its own row range.
    lo, hi = shard.shard_range(ROWS, world, rank)
    rows_local = hi - lo
    local_bytes = 4 * rows_local * HIDDEN + 2 * HIDDEN
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    x = torch.randn(rows_local, HIDDEN, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(HIDDEN, device="cuda", generator=g)).bfloat16()
    y = torch.empty_like(x)
    step = lambda: cuda_ops.rmsnorm(x, w, EPS, out=y)  # noqa: E731

    for _ in range(args.warmup):
        step()
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms, ms_max = _timed_max(step, args.steps, world, stream)
    cuda_ops.synchronize(torch.cuda.current_device())
    value = BYTES_PER_STEP / (ms_max * 1e-3) / 1e9
    achieved = local_bytes / (ms * 1e-3) / 1e9  # one launch per step on this rank
    gather_y = _allgather_ms(y, world) if world > 1 else None

    # e2e through the C ABI with host buffers: enigma_rmsnorm_host takes pinned host x and w
    # and writes host y, moving every row of this rank's shard host -> device -> host each
    # step in chunks whose uploads, kernels and downloads overlap on two streams.
    lib = _native.lib()
    nbytes = rows_local * HIDDEN * 2
    chunk = 8192
    hx = torch.empty((rows_local, HIDDEN), dtype=torch.bfloat16, pin_memory=True)
    hy = torch.empty((rows_local, HIDDEN), dtype=torch.bfloat16, pin_memory=True)
    hw = torch.empty((HIDDEN,), dtype=torch.bfloat16, pin_memory=True)
    hx.copy_(x)
    hw.copy_(w)
    wsb = ctypes.c_size_t()
    _native.check(lib.enigma_rmsnorm_host_workspace_bytes(_native.DTYPE_BF16, HIDDEN, chunk,
                                                          ctypes.byref(wsb)), "ws bytes")
    ws = torch.empty(wsb.value, dtype=torch.uint8, device="cuda")
    sp = stream.cuda_stream

    def e2e_step():
        _native.check(lib.enigma_rmsnorm_host(_native.DTYPE_BF16, hx.data_ptr(), hw.data_ptr(),
                                              hy.data_ptr(), rows_local, HIDDEN, EPS,
                                              ws.data_ptr(), wsb.value, chunk, sp), "rmsnorm_host")

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    _, e2e_ms = _timed_max(e2e_step, e2e_steps, world, stream)
    e2e_value = BYTES_PER_STEP / (e2e_ms * 1e-3) / 1e9
    del hx, hy, hw, ws, x, y

    ops = None if args.no_ops else _ops_side(world, rank, hbm_peak, tc_peak, peak_kind)
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (x ~ N(0,1), w ~ 1 + 0.1 N(0,1), torch generator seeded per rank)",
        "config": _config(world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "peak_kind": f"{peak_kind} (copy bandwidth, MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": round(NCU_TRAFFIC_PER_BYTE * local_bytes),
                     "traffic_source": NCU_TRAFFIC_SOURCE,
                     "algorithmic_bytes_per_launch": local_bytes,
                     "rows_per_launch": rows_local},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": nbytes + HIDDEN * 2, "d2h_bytes_per_step": nbytes,
                "ms_per_step": round(e2e_ms, 3),
                "path": "C ABI enigma_rmsnorm_host per rank: pinned host in / out, 8192-row "
                        "chunks, uploads / kernels / downloads overlapped on two streams; "
                        "value = all ranks' algorithmic bytes / max e2e time; bytes per step "
                        "are rank 0's"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if gather_y is not None:
        line["allgather_y"] = gather_y
    if ops is not None:
        line["ops"] = ops
    # The CPU baseline is a one-host figure: taken at N = 1 only.
    if not args.no_cpu and world == 1:
        line["cpu_baseline"] = _cpu_baseline(sample_rows=args.cpu_rows)
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's CPU implementation of the path, timed on this host's cores: its fp32
    numpy RMSNorm (examples/benchmark_rmsnorm.py:115-116; the reference's kernels are
    Apple-Metal only).  Rank 0 alone runs under torchrun; the host is one machine at every
    N, so the value does not grow with n_gpus."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = _host_threads()
    sample = args.cpu_rows
    _cpu_rmsnorm_rate(sample, threads, 0.0, passes=args.warmup)
    times, rows = [], 0
    for _ in range(args.steps):
        dt, r = _cpu_rmsnorm_rate(sample, threads, 0.0, passes=1)
        times.append(dt)
        rows += r
    total = sum(times)
    gbs = 4 * rows * HIDDEN / total / 1e9
    cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": _cpu_sample_text(rows, total, threads, sample)}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / len(times) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(world),
        "host_note": "one host's cores at every n_gpus (the reference has no multi-device path)",
        "cpu_baseline": cpu,
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_single_op(args):
    """One operator alone at a chosen size (profiling cases for ncu; not the headline)."""
    import torch
    from enigma import cuda_ops
    cuda_ops.ensure_device(0)
    stream = torch.cuda.current_stream()
    g = torch.Generator(device="cuda").manual_seed(0)
    n = args.size
    if args.only == "decode":
        from enigma.decode_layer import DecodeConfig, DecodeLayer
        layer = DecodeLayer.random(DecodeConfig(), seed=0)
        x = torch.randn(64, 896, device="cuda", generator=g).bfloat16()
        out = torch.empty_like(x)
        fn = layer.capture(x, out) if args.graph else (lambda: layer.step(x, out=out))
        for _ in range(args.warmup):
            fn()
        ms = _time_device_flushed(fn, args.steps, stream)
        ms_warm = _time_device(fn, args.steps, stream)
        cuda_ops.synchronize(0)
        print(json.dumps({"op": "decode", "ms": round(ms, 4), "ms_back_to_back": round(ms_warm, 4),
                          "gbs": round((layer.weight_bytes() + 2 * 64 * 2 * 2049 * 64 * 2)
                                       / (ms * 1e-3) / 1e9, 1)}), flush=True)
        return
    if args.only == "rmsnorm":
        hbm_peak = _peaks()[0]
        print(json.dumps(_rmsnorm_line(args.rows, args.hidden, args.dtype, args.steps,
                                       args.warmup, stream, hbm_peak)), flush=True)
        return
    if args.only == "gemm":
        a = (torch.randn(n, n, device="cuda", generator=g) / math.sqrt(n)).bfloat16()
        b = torch.randn(n, n, device="cuda", generator=g).bfloat16()
        c = torch.empty_like(a)
        fn, work, unit = (lambda: cuda_ops.gemm(a, b, out=c)), 2 * n ** 3, "TFLOP/s"
    else:
        B, H, D = 8, 32, 128
        q, k, v = (torch.randn(B, H, n, D, device="cuda", generator=g).bfloat16()
                   for _ in range(3))
        o = torch.empty_like(q)
        causal = args.only == "sdpa_causal"
        fn = lambda: cuda_ops.sdpa(q, k, v, causal=causal, out=o)  # noqa: E731
        if args.cudnn:   # the library reference point instead: cuDNN fused attention
            import torch.nn.functional as F
            from torch.nn.attention import SDPBackend, sdpa_kernel
            ctx = sdpa_kernel(SDPBackend.CUDNN_ATTENTION)
            ctx.__enter__()
            fn = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal)  # noqa: E731
        work, unit = (2 if causal else 4) * B * H * n * n * D, "TFLOP/s"
    for _ in range(args.warmup):
        fn()
    ms = _time_device(fn, args.steps, stream)
    cuda_ops.synchronize(0)
    print(json.dumps({"op": args.only, "size": n, "ms": round(ms, 4),
                      "value": round(work / (ms * 1e-3) / 1e12, 1), "unit": unit,
                      "impl": "cudnn" if args.cudnn else "enigma"}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-ops", action="store_true", help="skip the GEMM/SDPA side numbers")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--cpu-rows", type=int, default=16384)
    ap.add_argument("--rows", type=int, default=ROWS,
                    help="rows per GPU (smaller cases are for profiling only)")
    ap.add_argument("--only", choices=["gemm", "sdpa", "sdpa_causal", "decode", "rmsnorm"],
                    default=None,
                    help="time one operator alone (profiling case)")
    ap.add_argument("--graph", action="store_true", help="--only decode: replay a CUDA graph")
    ap.add_argument("--cudnn", action="store_true",
                    help="--only sdpa|sdpa_causal: time cuDNN's fused attention (torch SDPA) instead")
    ap.add_argument("--size", type=int, default=4096, help="--only: n for GEMM n^3, S for SDPA")
    ap.add_argument("--hidden", type=int, default=HIDDEN, help="--only rmsnorm: row width")
    ap.add_argument("--dtype", choices=["bf16", "f32"], default="bf16", help="--only rmsnorm")
    ap.add_argument("--sweep", action="store_true",
                    help="every BASELINE configuration on one GPU, one JSON line each")
    args = ap.parse_args()
    _set_rows(args.rows)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.sweep:
        run_sweep(args)
        return
    if args.only:
        run_single_op(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and args.impl == "ours":
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
