"""Profile data and bottleneck classification from B200 measurements.

Stands in for phew's ``trace`` package as ``Optimizer.run`` step 2 uses it
(``optimizer.py:128-146``: ``BottleneckClassifier().classify(ProfileData)``,
``trace/classifier.py:84-122``).  The reference fills ``ProfileData`` from a
Metal trace (and, in its own code, only from device info); here it comes
from the device:

* ``profile(fn, *args)`` -- per-kernel device times from CUPTI (through
  ``torch.profiler``): enough for the launch-overhead test (small-kernel
  fraction) and the Phase-2 trigger (hottest kernel > 30 % of the time);
* ``from_ncu_csv(path)`` -- per-kernel counters from an Nsight Compute CSV
  of the metrics in ``NCU_METRICS`` (``ncu_command`` gives the command line):
  SM throughput as the ALU utilisation, DRAM bytes / duration as the
  bandwidth, active warps as the occupancy -- the quantities the
  reference's thresholds are written in.

The dataclasses have the reference's field names; when phew is importable
its own ``ProfileData`` / ``KernelStat`` / ``BottleneckClassifier`` are used,
so the optimizer consumes the result unchanged.
"""

from __future__ import annotations

import csv
import io
from dataclasses import dataclass, field
from enum import Enum
from pathlib import Path
from typing import Any, Callable

NCU_METRICS = (
    "gpu__time_duration.sum",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
)
SMALL_KERNEL_MS = 0.1  # the reference's "is_small" heuristic


class BottleneckClass(Enum):
    memory_bound = "memory_bound"
    compute_bound = "compute_bound"
    occupancy_limited = "occupancy_limited"
    launch_overhead = "launch_overhead"
    unknown = "unknown"


@dataclass
class KernelStat:
    name: str
    duration_ms: float
    alu_utilization: float = 0.0
    memory_bandwidth_gb: float = 0.0
    occupancy: float = 1.0
    is_small: bool = False


@dataclass
class ProfileData:
    kernels: list = field(default_factory=list)
    total_ms: float = 0.0
    device_info: dict = field(default_factory=dict)

    @property
    def n_kernels(self) -> int:
        return len(self.kernels)

    @property
    def small_kernel_fraction(self) -> float:
        return sum(1 for k in self.kernels if k.is_small) / len(self.kernels) if self.kernels else 0.0

    @property
    def mean_alu_util(self) -> float:
        return sum(k.alu_utilization for k in self.kernels) / len(self.kernels) if self.kernels else 0.0

    @property
    def mean_occupancy(self) -> float:
        return sum(k.occupancy for k in self.kernels) / len(self.kernels) if self.kernels else 1.0

    @property
    def hottest_kernel(self):
        return max(self.kernels, key=lambda k: k.duration_ms) if self.kernels else None

    @property
    def hottest_kernel_fraction(self) -> float:
        if not self.kernels or self.total_ms <= 0:
            return 0.0
        return self.hottest_kernel.duration_ms / self.total_ms


class BottleneckClassifier:
    """The reference's thresholds (trace/classifier.py:84-122)."""

    ALU_LOW, ALU_HIGH, OCC_LOW, SMALL_FRAC, PHASE2_TRIGGER = 0.40, 0.70, 0.50, 0.50, 0.30

    def classify(self, data) -> BottleneckClass:
        if data.small_kernel_fraction > self.SMALL_FRAC:
            return BottleneckClass.launch_overhead
        if data.mean_occupancy < self.OCC_LOW:
            return BottleneckClass.occupancy_limited
        if data.mean_alu_util > self.ALU_HIGH:
            return BottleneckClass.compute_bound
        if data.mean_alu_util < self.ALU_LOW:
            return BottleneckClass.memory_bound
        return BottleneckClass.unknown

    def needs_phase2(self, data) -> bool:
        return data.hottest_kernel_fraction > self.PHASE2_TRIGGER


def _classes():
    """phew's own classes when phew is importable, else this module's."""
    try:
        from phew.trace.classifier import KernelStat as K
        from phew.trace.classifier import ProfileData as P

        return K, P
    except ImportError:
        return KernelStat, ProfileData


def device_info() -> dict:
    try:
        from .mx.core import device_info as di

        return di()
    except Exception:  # noqa: BLE001  (no device: empty info, as the reference does off-Metal)
        return {}


def profile(fn: Callable, *args: Any, warmup: int = 2, **kwargs: Any):
    """Per-kernel device times of one call of `fn` (after `warmup` calls),
    from CUPTI activity records.  Counters need Nsight Compute
    (``from_ncu_csv``); here ALU utilisation and bandwidth stay 0 and
    occupancy 1, so only the launch-overhead test and the Phase-2 trigger
    read this profile."""
    import torch
    from torch.profiler import ProfilerActivity
    from torch.profiler import profile as tprofile

    K, P = _classes()
    for _ in range(warmup):
        fn(*args, **kwargs)
    torch.cuda.synchronize()
    with tprofile(activities=[ProfilerActivity.CUDA]) as prof:
        fn(*args, **kwargs)
        torch.cuda.synchronize()
    stats = []
    for ev in prof.events():
        dev_us = getattr(ev, "device_time", None)
        if dev_us is None:
            dev_us = getattr(ev, "cuda_time", 0.0)
        if getattr(ev, "device_type", None) is not None and "CUDA" in str(ev.device_type) and dev_us > 0:
            ms = dev_us / 1e3
            stats.append(K(name=ev.name, duration_ms=ms, is_small=ms < SMALL_KERNEL_MS))
    return P(kernels=stats, total_ms=sum(k.duration_ms for k in stats), device_info=device_info())


def ncu_command(cmd: str, out_csv: str = "ncu_metrics.csv", kernel_regex: str | None = None,
                launch_count: int | None = None) -> str:
    """The Nsight Compute command whose CSV ``from_ncu_csv`` reads (clocks
    left alone: ``--clock-control none``)."""
    parts = ["ncu", "--clock-control none", "--metrics", ",".join(NCU_METRICS), "--csv",
             f"--log-file {out_csv}"]
    if kernel_regex:
        parts.append(f"-k regex:{kernel_regex}")
    if launch_count:
        parts.append(f"-c {int(launch_count)}")
    return " ".join(parts + [cmd])


def _num(v: str) -> float:
    try:
        return float(str(v).replace(",", ""))
    except ValueError:
        return 0.0


def _scale(unit: str) -> float:
    """Factor to bytes / ms / fraction for the units Nsight Compute prints."""
    u = (unit or "").strip().lower()
    return {"byte": 1.0, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "tbyte": 1e12,
            "nsecond": 1e-6, "ns": 1e-6, "usecond": 1e-3, "us": 1e-3, "msecond": 1.0, "ms": 1.0,
            "second": 1e3, "s": 1e3, "%": 0.01}.get(u, 1.0)


def from_ncu_csv(source) -> Any:
    """ProfileData from an Nsight Compute CSV: either the per-metric rows of
    ``ncu --csv --metrics ...`` ("Metric Name" / "Metric Unit" / "Metric
    Value" columns) or the wide table of ``ncu -i rep --page raw --csv``
    (a header row, a units row, one row per kernel)."""
    K, P = _classes()
    text = Path(source).read_text() if not isinstance(source, str) or "\n" not in source else source
    lines = [ln for ln in text.splitlines() if ln.startswith('"')]
    rows = list(csv.reader(io.StringIO("\n".join(lines))))
    if not rows:
        return P(device_info=device_info())
    header = rows[0]
    per: dict[tuple, dict] = {}
    if "Metric Name" in header:
        ix = {h: i for i, h in enumerate(header)}
        for r in rows[1:]:
            key = (r[ix["ID"]], r[ix["Kernel Name"]])
            per.setdefault(key, {})[r[ix["Metric Name"]]] = _num(r[ix["Metric Value"]]) * _scale(r[ix["Metric Unit"]])
    else:
        units = rows[1] if len(rows) > 1 else []
        ix = {h: i for i, h in enumerate(header)}
        for r in rows[2:]:
            key = (r[ix.get("ID", 0)], r[ix.get("Kernel Name", 0)])
            d = per.setdefault(key, {})
            for m in NCU_METRICS:
                if m in ix:
                    d[m] = _num(r[ix[m]]) * _scale(units[ix[m]] if ix[m] < len(units) else "")
    stats = []
    for (_, name), m in per.items():
        ms = m.get("gpu__time_duration.sum", 0.0)
        byts = m.get("dram__bytes_read.sum", 0.0) + m.get("dram__bytes_write.sum", 0.0)
        stats.append(K(
            name=name, duration_ms=ms,
            alu_utilization=m.get("sm__throughput.avg.pct_of_peak_sustained_elapsed", 0.0),
            memory_bandwidth_gb=(byts / 1e9) / (ms / 1e3) if ms > 0 else 0.0,
            occupancy=m.get("sm__warps_active.avg.pct_of_peak_sustained_active", 1.0),
            is_small=ms < SMALL_KERNEL_MS,
        ))
    return P(kernels=stats, total_ms=sum(k.duration_ms for k in stats), device_info=device_info())


def classify(data) -> Any:
    """phew's BottleneckClassifier when importable, else the same rules here."""
    try:
        from phew.trace.classifier import BottleneckClassifier as C
    except ImportError:
        C = BottleneckClassifier
    return C().classify(data)
