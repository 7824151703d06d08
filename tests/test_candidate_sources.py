"""The candidate sources the GPU tests run are what the reference's own
``Optimizer.run`` emits (CPU only).

``tests/golden/optimizer_runs.json`` holds the output of the reference's
``Optimizer(fn, input_factory).run()`` (optimizer.py:90-353) on the
rms_norm and gelu_chain harnesses, run with the oracle serving mlx.core
(``make_golden.py --part optimizer``).  Re-targeted the way
``integration.install()`` re-targets ``MLXCodegen`` (the two import lines),
each equals the committed source that ``tests/test_gpu_optimizer.py``
evaluates on the GPU."""

from __future__ import annotations

import json
from pathlib import Path

import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def _retarget(src: str) -> str:
    src = src.replace("import mlx.core as mx\n", "import phew_b200.mx as mx\n", 1)
    return src.replace("import mlx.core.fast as fast\n", "from phew_b200.mx import fast\n", 1)


@pytest.mark.parametrize("key", ["rms_norm__fusion0", "gelu_chain__fusion0"])
def test_optimizer_output_source_is_the_committed_candidate(key):
    run = json.loads((GOLDEN / "optimizer_runs.json").read_text())[key]
    assert _retarget(run["output_source"]) == (GOLDEN / "sources" / f"{key}.py").read_text()
    # the reference verified it and ran every step up to 7
    assert run["verification_passed"] is True and run["verification_details"] == []
    assert run["steps"][-2:] == ["Step 6: Benchmark candidate", "Step 7: Equivalence verification"]


def test_optimizer_applied_the_rms_norm_substitution():
    runs = json.loads((GOLDEN / "optimizer_runs.json").read_text())
    assert "primitive_subst" in runs["rms_norm__fusion0"]["applied_rules"]
    assert "mx.fast.rms_norm(" in runs["rms_norm__fusion0"]["output_source"]
    assert runs["gelu_chain__fusion0"]["applied_rules"] == ["compile_boundary"]
