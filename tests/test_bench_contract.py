"""bench.py's reference arm runs on the CPU: its JSON line keeps the
contract the driver reads (one line, the metric of the workload, the
reference's CPU timing, e2e with no host<->device bytes).  The default
workload is the verification sweep; the per-kernel workloads keep the same
contract."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _reference_line(*extra):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1", *extra], capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "dtype", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 1
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    return d


def test_reference_arm_sweep_line():
    """The default workload (reduced decoder dimensions here, to keep the
    CPU suite short): verified candidates/s, strong scaling."""
    d = _reference_line("--tiny")
    assert d["metric"] == "verified_candidates_per_s" and d["unit"] == "candidates/s"
    assert d["scaling"] == "strong" and d["units_per_s_subset"] > 0


def test_reference_arm_kernel_line():
    d = _reference_line("--workload", "gelu_chain")
    assert d["metric"] == "fused_kernel_hbm_gbs" and d["unit"] == "GB/s"


def test_reference_arm_sweep_internal_kernel_is_unavailable():
    """A sweep-internal kernel timed on its own has no CPU path of its own:
    the reference arm says so in one line and exits 0."""
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload",
                          "qk_scores", "--steps", "2", "--warmup", "1"],
                         capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and "unavailable" in d


def test_peaks_and_traffic_helpers():
    sys.path.insert(0, str(ROOT))
    import bench

    peaks = bench.load_peaks()
    assert peaks["hbm_gbs"] > 1000 and peaks["bf16_tflops"] > 100 and peaks["source"] in ("measured", "fallback")
    assert peaks["bf16_tflops_sustained"] > 100
    assert bench.load_traffic("gelu_chain_fused_fp16_4096x8192") > 0
    assert bench.load_traffic(None) is None


def test_small_rms_norm_inputs_rotate_past_l2():
    sys.path.insert(0, str(ROOT))
    import bench

    for n in (256, 1024, 4096):
        w = bench.RmsNorm(n)
        assert w.R * w.work_per_step() > 2 * bench.L2_BYTES
        assert w.min_steps >= w.R
