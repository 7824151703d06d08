"""Profile data / bottleneck classification from Nsight Compute CSVs, and
the phase-2 search's enumeration, filtering and pruning (no GPU)."""

from __future__ import annotations

import types
from pathlib import Path

import pytest

GOLDEN = Path(__file__).parent / "golden"

LONG_CSV = '''"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","python","h","gelu_chain_fused","1","7","(256, 1, 1)","(9472, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","usecond","301.4"
"0","1","python","h","gelu_chain_fused","1","7","(256, 1, 1)","(9472, 1, 1)","0","10.0","Command line profiler metrics","sm__throughput.avg.pct_of_peak_sustained_elapsed","%","31.5"
"0","1","python","h","gelu_chain_fused","1","7","(256, 1, 1)","(9472, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_read.sum","Mbyte","134.28"
"0","1","python","h","gelu_chain_fused","1","7","(256, 1, 1)","(9472, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_write.sum","Mbyte","38.52"
"0","1","python","h","gelu_chain_fused","1","7","(256, 1, 1)","(9472, 1, 1)","0","10.0","Command line profiler metrics","sm__warps_active.avg.pct_of_peak_sustained_active","%","83.5"
'''


def test_ncu_long_format_memory_bound():
    """(A single kernel under 0.1 ms would count as launch overhead by the
    reference's small-kernel rule, so the sample is 0.3 ms long.)"""
    from phew_b200 import trace

    d = trace.from_ncu_csv(LONG_CSV)
    assert d.n_kernels == 1
    k = d.kernels[0]
    assert k.name == "gelu_chain_fused" and k.duration_ms == pytest.approx(0.3014)
    assert k.memory_bandwidth_gb == pytest.approx((134.28e6 + 38.52e6) / 1e9 / 301.4e-6, rel=1e-6)
    assert k.alu_utilization == pytest.approx(0.315) and k.occupancy == pytest.approx(0.835)
    assert trace.classify(d).value == "memory_bound"


def test_ncu_raw_page_of_the_tcgen05_kernels():
    """Real counters of the GEMM and attention kernels (ncu --page raw):
    one warp group per SM keeps the warp occupancy low by design, which the
    reference's thresholds call occupancy-limited."""
    from phew_b200 import trace

    d = trace.from_ncu_csv(GOLDEN / "ncu_raw_sample.csv")
    names = sorted(k.name.split("<")[0].split()[-1] for k in d.kernels)
    assert names == ["gemm_tc_kernel", "sdpa_fwd_kernel"]
    gemm = next(k for k in d.kernels if "gemm" in k.name)
    assert gemm.duration_ms == pytest.approx(0.231456)
    assert 700 < gemm.memory_bandwidth_gb < 800
    assert trace.classify(d).value == "occupancy_limited"
    assert trace.BottleneckClassifier().needs_phase2(d)


def test_launch_overhead_and_phase2_trigger():
    from phew_b200 import trace

    ks = [trace.KernelStat(f"k{i}", 0.01, is_small=True) for i in range(6)] + [trace.KernelStat("big", 1.0)]
    d = trace.ProfileData(kernels=ks, total_ms=1.06)
    assert trace.BottleneckClassifier().classify(d).value == "launch_overhead"
    assert trace.BottleneckClassifier().needs_phase2(d)


def test_ncu_command_keeps_clocks():
    from phew_b200 import trace

    cmd = trace.ncu_command("python bench.py", kernel_regex="gemm", launch_count=3)
    assert "--clock-control none" in cmd and "-k regex:gemm" in cmd and "-c 3" in cmd
    assert all(m in cmd for m in trace.NCU_METRICS)


def _node(source, grid=None):
    return types.SimpleNamespace(source=source, input_names=["x"], output_names=["y"],
                                 output_shapes=[(8,)], output_dtypes=["float32"], grid=grid, attrs={},
                                 header="", name="k")


def test_search_space_grid_stride_and_templates():
    from phew_b200.emit.autotune import KernelParamSearch

    s = KernelParamSearch()
    emitted = _node("for (...; elem += phew_nthreads) {}")
    assert KernelParamSearch.grid_stride(emitted)
    c = s._enumerate(emitted)
    assert len(c) == 5 * 5 and {x.waves for x in c} == {1, 2, 4, 8, 16}
    user = _node("y[i] = x[i] * VW; // UNROLL", grid=(8, 1, 1))
    c = s._enumerate(user)
    assert not KernelParamSearch.grid_stride(user)
    assert len(c) == 5 * 4 * 4 and {x.waves for x in c} == {0}
    assert s._grid(user, c[0], []) == (8, 1, 1)  # a user kernel keeps its grid


@pytest.mark.parametrize("bn,check", [
    ("memory_bound", lambda c: c.threadgroup[0] >= 128 and c.vector_width >= 2),
    ("occupancy_limited", lambda c: c.threadgroup[0] <= 128),
    ("launch_overhead", lambda c: c.threadgroup[0] >= 256 and c.loop_unroll >= 4),
])
def test_bottleneck_filters(bn, check):
    from phew_b200.emit.autotune import KernelParamSearch

    c = KernelParamSearch(bottleneck=bn)._enumerate(_node("VW UNROLL"))
    assert c and all(check(x) for x in c)


def test_prune_limits():
    from phew_b200.emit.autotune import KernelCandidate, KernelParamSearch

    s = KernelParamSearch()
    big = KernelCandidate((2048,), None, 1, 1, False, False)
    assert s._prune(_node(""), big)[0]
    n = _node("")
    n.attrs = {"threadgroup_mem_bytes": 300 * 1024}
    assert s._prune(n, KernelCandidate((256,), None, 1, 1, False, False))[0]
