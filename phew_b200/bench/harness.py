"""Benchmark harness on CUDA events (phew ``bench/harness.py:28-112``).

Same contract as the reference: ``n_warmup`` untimed calls, then batches of
``n_bench`` timed calls until the coefficient of variation of the batch means
drops below ``cv_target`` or ``max_n_bench`` calls have been timed; ``compare``
reports a speedup as significant only outside the 3% noise band.

What changes is the clock: each call is bracketed by CUDA events recorded on
the current stream (device time, no host ``perf_counter``), and by default an
L2 flush (a write over a buffer larger than the L2) runs between timed calls,
outside the events, so every call starts with a cold L2.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Any, Callable

import torch


@dataclass
class BenchResult:
    mean_ms: float
    std_ms: float
    cv: float  # coefficient of variation = std/mean
    n_bench: int
    converged: bool  # σ/μ < cv_target
    samples_ms: list[float]


class L2Flusher:
    """Owns a device buffer twice the L2 size and overwrites it on demand."""

    def __init__(self) -> None:
        from .. import _native
        from ..mx.core import device

        dev = device()
        info = _native.DeviceInfo()
        _native.call("phew_device_query", dev.index, ctypes.byref(info))
        self.nbytes = max(int(info.l2_bytes) * 2, 64 << 20)
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=dev)
        self._native = _native

    def __call__(self) -> None:
        self._native.call(
            "phew_l2_flush",
            ctypes.c_void_p(self.buf.data_ptr()),
            ctypes.c_size_t(self.nbytes),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
        )


_flusher: L2Flusher | None = None


def l2_flush() -> None:
    global _flusher
    if _flusher is None:
        _flusher = L2Flusher()
    _flusher()


def benchmark(
    fn: Callable[..., Any],
    *args: Any,
    n_warmup: int = 5,
    n_bench: int = 20,
    max_n_bench: int = 100,
    cv_target: float = 0.05,
    flush_l2: bool = True,
    **kwargs: Any,
) -> BenchResult:
    """Mean device latency (ms) of fn(*args, **kwargs) per call."""
    stream = torch.cuda.current_stream()
    for _ in range(n_warmup):
        fn(*args, **kwargs)
    stream.synchronize()

    samples: list[float] = []
    while True:
        evs = []
        for _ in range(n_bench):
            if flush_l2:
                l2_flush()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn(*args, **kwargs)
            e.record(stream)
            evs.append((s, e))
        stream.synchronize()
        samples.append(sum(s.elapsed_time(e) for s, e in evs) / n_bench)

        mean = sum(samples) / len(samples)
        if len(samples) > 1:
            var = sum((x - mean) ** 2 for x in samples) / (len(samples) - 1)
            std = math.sqrt(var)
            cv = std / mean if mean > 0 else 0.0
            if cv < cv_target or n_bench * len(samples) >= max_n_bench:
                return BenchResult(mean, std, cv, n_bench * len(samples), cv < cv_target, samples)
        else:
            std, cv = 0.0, 0.0
        if n_bench * len(samples) >= max_n_bench:
            return BenchResult(mean, std, cv, n_bench * len(samples), False, samples)


def compare(baseline: BenchResult, optimized: BenchResult) -> dict[str, float]:
    """Speedup and significance (±3% noise band), as the reference reports."""
    speedup = baseline.mean_ms / optimized.mean_ms if optimized.mean_ms > 0 else float("inf")
    noise_band = 0.03
    return {
        "speedup": speedup,
        "baseline_ms": baseline.mean_ms,
        "baseline_std_ms": baseline.std_ms,
        "optimized_ms": optimized.mean_ms,
        "optimized_std_ms": optimized.std_ms,
        "is_significant": float(abs(speedup - 1.0) > noise_band),
        "baseline_converged": float(baseline.converged),
        "optimized_converged": float(optimized.converged),
    }
