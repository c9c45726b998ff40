"""Timing helpers (API of the reference's enigma/benchmark.py).

bench() times a Python callable by wall clock; bench_gpu() times a
PreparedKernel with CUDA events on the runtime's stream (dispatch_timed).
"""
from __future__ import annotations

import statistics
import time
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple


@dataclass
class BenchResult:
    label: str
    samples_us: Sequence[float]
    warmup: int

    n = property(lambda self: len(self.samples_us))
    min_us = property(lambda self: min(self.samples_us))
    max_us = property(lambda self: max(self.samples_us))
    median_us = property(lambda self: statistics.median(self.samples_us))
    mean_us = property(lambda self: statistics.fmean(self.samples_us))

    @property
    def stdev_us(self) -> float:
        return statistics.stdev(self.samples_us) if len(self.samples_us) > 1 else 0.0

    def __repr__(self) -> str:
        return (f"BenchResult({self.label!r}, n={self.n}, median={self.median_us:.2f}us, "
                f"min={self.min_us:.2f}us, max={self.max_us:.2f}us)")


def _validate(repeat: int, warmup: int) -> None:
    if repeat < 1:
        raise ValueError("repeat must be >= 1")
    if warmup < 0:
        raise ValueError("warmup must be >= 0")


def _samples(one: Callable[[], float], repeat: int, warmup: int) -> List[float]:
    for _ in range(warmup):
        one()
    return [one() for _ in range(repeat)]


def bench(fn: Callable, *args, repeat: int = 50, warmup: int = 5, label: Optional[str] = None,
          **kwargs) -> BenchResult:
    _validate(repeat, warmup)

    def one() -> float:
        t0 = time.perf_counter_ns()
        fn(*args, **kwargs)
        return (time.perf_counter_ns() - t0) / 1000.0

    return BenchResult(label or getattr(fn, "__name__", "fn"), _samples(one, repeat, warmup),
                       warmup)


def bench_gpu(prepared, grid: Tuple[int, int, int], threads: Tuple[int, int, int], *,
              repeat: int = 50, warmup: int = 5, label: Optional[str] = None) -> BenchResult:
    _validate(repeat, warmup)
    name = label or getattr(getattr(prepared, "_compiled", None), "kernel_name", "prepared")
    return BenchResult(name, _samples(lambda: float(prepared.dispatch_timed(grid, threads)),
                                      repeat, warmup), warmup)


def format_bench_result(r: BenchResult, *, throughput_gbps: Optional[float] = None) -> str:
    parts = [r.label, f"n={r.n}", f"median={r.median_us:.2f}us", f"min={r.min_us:.2f}us",
             f"max={r.max_us:.2f}us"]
    if throughput_gbps is not None:
        parts.append(f"BW={throughput_gbps:.2f}GB/s")
    return "  ".join(parts)
