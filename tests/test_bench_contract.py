"""bench.py's reference arm runs on the CPU: its JSON line keeps the
contract the driver reads (one line, the metric of the default workload, the
reference's CPU timing, e2e with no host<->device bytes)."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "dtype", "config", "impl", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["metric"] == "fused_kernel_hbm_gbs" and d["unit"] == "GB/s"
    assert d["steps"] == 1 and d["warmup"] == 1 and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1


def test_peaks_and_traffic_helpers():
    sys.path.insert(0, str(ROOT))
    import bench

    peaks = bench.load_peaks()
    assert peaks["hbm_gbs"] > 1000 and peaks["bf16_tflops"] > 100 and peaks["source"] in ("measured", "fallback")
    assert bench.load_traffic("gelu_chain_fused_fp16_4096x8192") > 0
    assert bench.load_traffic(None) is None
