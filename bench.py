#!/usr/bin/env python3
"""Benchmark of the Enigma hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-ops]

Headline (BASELINE metric, config 2 at its largest size): bf16 RMSNorm over
x [262144, 8192] (fp32 accumulate, eps 1e-6), HBM GB/s, one kernel launch per
step.  Bytes per step are the algorithmic ones: read x once, write y once,
read w once (4*rows*hidden + 2*hidden).  Inputs (4 GiB each way) are larger
than the 126 MB L2, so no flush is needed between steps.

With N > 1 (launched under torchrun, one rank per GPU) each rank processes
its own full-size row shard (weak scaling, no collective on the data path);
the timed region is bracketed by a barrier and cuda synchronize, and the
elapsed time is the max over ranks.

`ops` in the JSON line adds the other hot-path operators at their BASELINE
headline sizes on rank 0 (GEMM bf16 8192^3, SDPA bf16 [8,32,8192,128]),
TFLOP/s against the measured bf16 peak.

--impl reference times the reference's own CPU formulation of the same
operator (the numpy check of examples/benchmark_rmsnorm.py:117-118, restated
in oracle/numerics.py) on the host cores, on a bounded row sample per step.
"""
from __future__ import annotations

import argparse
import ctypes
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
# DRAM bytes (read + write) of one rmsnorm launch at this size, from the ncu
# capture summarised in profiles/rmsnorm_bf16_262144x8192.md (small case scaled x8).
NCU_TRAFFIC_PER_LAUNCH = 8_192_407_552


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
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
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
def _cpu_rmsnorm_sample(sample_rows: int, threads: int):
    """Time the oracle's numpy RMSNorm on `sample_rows` rows of the workload.

    Returns (seconds, rows).  Rows are split across `threads` Python threads
    (numpy releases the GIL inside its kernels).
    """
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle import numerics as orc
    rng = np.random.default_rng(0)
    x = orc.bf16_round(rng.standard_normal((sample_rows, HIDDEN), dtype=np.float32))
    w = orc.bf16_round((1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32))
    chunks = np.array_split(np.arange(sample_rows), threads)

    def work(idx):
        if len(idx):
            orc.rmsnorm(x[idx[0]:idx[-1] + 1], w, EPS)

    t0 = time.perf_counter()
    if threads == 1:
        work(chunks[0])
    else:
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(work, chunks))
    return time.perf_counter() - t0, sample_rows


def _cpu_baseline(threads=1, sample_rows=16384):
    dt, rows = _cpu_rmsnorm_sample(sample_rows, threads)
    gbs = (4 * rows * HIDDEN + 2 * HIDDEN) / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {ROWS} rows x {HIDDEN} (bf16-rounded inputs, fp64 numpy "
                      f"oracle, oracle/numerics.py:rmsnorm), {dt:.2f} s"}


# ----------------------------------------------------------------------------- our arm
def _ops_side(hbm_peak, tc_peak, peak_kind):
    """GEMM / SDPA at their BASELINE headline sizes on this GPU (rank 0 only)."""
    import torch
    from enigma import cuda_ops
    res = {}
    stream = torch.cuda.current_stream()
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    a = (torch.randn(n, n, device="cuda", generator=g) / math.sqrt(n)).bfloat16()
    b = torch.randn(n, n, device="cuda", generator=g).bfloat16()
    c = torch.empty_like(a)
    for _ in range(3):
        cuda_ops.gemm(a, b, out=c)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = _time_device(lambda: cuda_ops.gemm(a, b, out=c), 20, stream)
    tf = 2 * n ** 3 / (ms * 1e-3) / 1e12
    res["gemm_bf16_8192"] = {"tflops": round(tf, 1), "ms": round(ms, 4),
                             "frac": round(tf / tc_peak, 4), "peak": tc_peak,
                             "peak_kind": peak_kind + " burst", "clocks": clk.summary()}
    del a, b, c
    if os.environ.get("ENIGMA_BENCH_SDPA", "1") == "1" and _sdpa_tc_available():
        B, H, S, D = 8, 32, 8192, 128
        q = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
        k = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
        v = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
        o = torch.empty_like(q)
        for causal in (True, False):
            fn = lambda: cuda_ops.sdpa(q, k, v, causal=causal, out=o)  # noqa: E731
            for _ in range(3):
                fn()
            with ClockSampler(torch.cuda.current_device()) as clk:
                ms = _time_device(fn, 10, stream)
            fl = (2 if causal else 4) * B * H * S * S * D
            tf = fl / (ms * 1e-3) / 1e12
            res[f"sdpa_bf16_{'causal' if causal else 'noncausal'}_8x32x8192x128"] = {
                "tflops": round(tf, 1), "ms": round(ms, 3), "frac": round(tf / tc_peak, 4),
                "flops_convention": "causal 2*B*H*S^2*D, non-causal 4*B*H*S^2*D",
                "clocks": clk.summary()}
    res["decode_layer_config5"] = _decode_side(hbm_peak)
    return res


def _decode_side(hbm_peak):
    """one decode step, batch 64, 2048-token KV cache (HBM-bound)."""
    import torch
    from enigma.decode_layer import DecodeConfig, DecodeLayer
    cfg = DecodeConfig()
    layer = DecodeLayer.random(cfg, seed=0)
    x = torch.randn(cfg.batch, cfg.hidden, device="cuda").bfloat16()
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    fn = layer.capture(x, out)
    for _ in range(5):
        fn()
    ms = _time_device_flushed(fn, 50, stream)
    ms_warm = _time_device(fn, 50, stream)
    kv = 2 * cfg.batch * cfg.heads_kv * (cfg.cache_len + 1) * cfg.head_dim * 2
    byts = layer.weight_bytes() + kv
    return {"ms": round(ms, 4), "tokens_per_s": round(cfg.batch / (ms * 1e-3), 1),
            "algorithmic_bytes": byts, "gbs": round(byts / (ms * 1e-3) / 1e9, 1),
            "frac_hbm": round(byts / (ms * 1e-3) / 1e9 / hbm_peak, 4),
            "l2": "flushed (256 MB read) before every step",
            "ms_back_to_back": round(ms_warm, 4),
            "note": "weights + KV read once per step; back to back, L2 (126 MB) can hold "
                    "part of the 97 MB working set"}


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
            tf = (2 if causal else 4) * B * H * S * S * D / (ms * 1e-3) / 1e12
            print(json.dumps({"config": 4, "op": "sdpa_bf16", "S": S, "causal": causal,
                              "ms": round(ms, 4), "value": round(tf, 1), "unit": "TFLOP/s",
                              "frac_tensor": round(tf / tc_peak, 4), "timing": "back to back",
                              "flops": "causal 2BHS^2D, non-causal 4BHS^2D"}), flush=True)
        del q, k, v, o
    print(json.dumps({"config": 5, "op": "decode_layer"} | _decode_side(hbm_peak)), flush=True)


def run_ours(args):
    import torch
    from enigma import _native, cuda_ops
    rank, world, local = _dist_init(args.gpus)
    cuda_ops.ensure_device(torch.cuda.current_device())
    hbm_peak, tc_peak, peak_kind = _peaks()
    stream = torch.cuda.current_stream()

    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    x = torch.randn(ROWS, HIDDEN, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(HIDDEN, device="cuda", generator=g)).bfloat16()
    y = torch.empty_like(x)
    step = lambda: cuda_ops.rmsnorm(x, w, EPS, out=y)  # noqa: E731

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = _time_device(step, args.steps, stream)
        torch.cuda.synchronize()
    _barrier(world)
    cuda_ops.synchronize(torch.cuda.current_device())
    ms_max = _max_over_ranks(ms, world)
    value = world * BYTES_PER_STEP / (ms_max * 1e-3) / 1e9
    achieved = BYTES_PER_STEP / (ms * 1e-3) / 1e9  # one launch per step on this rank

    # e2e through the C ABI with host buffers: enigma_rmsnorm_host takes pinned host x and w
    # and writes host y, moving every row host -> device -> host each step in chunks whose
    # uploads, kernels and downloads overlap on two streams.
    lib = _native.lib()
    nbytes = ROWS * HIDDEN * 2
    chunk = 8192
    hx = torch.empty((ROWS, HIDDEN), dtype=torch.bfloat16, pin_memory=True)
    hy = torch.empty((ROWS, HIDDEN), dtype=torch.bfloat16, pin_memory=True)
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
                                              hy.data_ptr(), ROWS, HIDDEN, EPS, ws.data_ptr(),
                                              wsb.value, chunk, sp), "rmsnorm_host")

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    _barrier(world)
    e2e_ms = _max_over_ranks(_time_device(e2e_step, e2e_steps, stream), world)
    e2e_value = world * BYTES_PER_STEP / (e2e_ms * 1e-3) / 1e9
    del hx, hy, hw, ws

    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (x ~ N(0,1), w ~ 1 + 0.1 N(0,1), torch generator seeded per rank)",
        "config": {"workload": f"rmsnorm bf16 rows={ROWS} hidden={HIDDEN} eps={EPS} per GPU",
                   "rows_per_gpu": ROWS, "hidden": HIDDEN, "parallelism": f"row-shard x{world}",
                   "l2": "inputs (4 GiB) larger than L2; no flush",
                   "bytes_per_step_per_gpu": BYTES_PER_STEP},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "peak_kind": f"{peak_kind} (copy bandwidth, MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": NCU_TRAFFIC_PER_LAUNCH,
                     "algorithmic_bytes_per_launch": BYTES_PER_STEP},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s (algorithmic bytes / e2e time)",
                "h2d_bytes_per_step": nbytes + HIDDEN * 2, "d2h_bytes_per_step": nbytes,
                "ms_per_step": round(e2e_ms, 3),
                "path": "C ABI enigma_rmsnorm_host: pinned host in / out, 8192-row chunks, "
                        "uploads / kernels / downloads overlapped on two streams"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    # The per-operator lines and the CPU baseline are one-GPU figures: taken at N = 1 only
    # (under torchrun the other GPUs would sit held while rank 0 measured them).
    if not args.no_ops and world == 1:
        line["ops"] = _ops_side(hbm_peak, tc_peak, peak_kind)
    if not args.no_cpu and world == 1:
        line["cpu_baseline"] = _cpu_baseline(threads=1, sample_rows=args.cpu_rows)
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    sample = args.cpu_rows
    for _ in range(args.warmup):
        _cpu_rmsnorm_sample(min(sample, 1024), threads)
    times = []
    for _ in range(args.steps):
        dt, rows = _cpu_rmsnorm_sample(sample, threads)
        times.append(dt)
    dt = sum(times) / len(times)
    gbs = (4 * sample * HIDDEN + 2 * HIDDEN) / dt / 1e9
    cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": f"{sample} of {ROWS} rows x {HIDDEN} per step (numpy restatement of "
                     "examples/benchmark_rmsnorm.py:117-118 in oracle/numerics.py)"}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"rmsnorm bf16 rows={ROWS} hidden={HIDDEN} eps={EPS} per GPU",
                   "note": "reference is Apple-Metal only; its CPU numpy formulation is timed"},
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
        work, unit = (2 if causal else 4) * B * H * n * n * D, "TFLOP/s"
    for _ in range(args.warmup):
        fn()
    ms = _time_device(fn, args.steps, stream)
    cuda_ops.synchronize(0)
    print(json.dumps({"op": args.only, "size": n, "ms": round(ms, 4),
                      "value": round(work / (ms * 1e-3) / 1e12, 1), "unit": unit}), flush=True)


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
