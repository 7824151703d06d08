"""Steps 1, 6 and 7 of the reference's ``Optimizer.run`` on this backend
(``phew_b200.candidate.evaluate_candidate``, after optimizer.py:116-126 and
:290-353): the candidates the reference's passes emit for the rms_norm
(config 0) and elementwise-chain (config 1) harnesses are built, benchmarked
with CUDA events at the three sizes, verified with the equivalence protocol
and summarised.

Verdicts are checked against the reference: for the unfused candidates,
against the Step-7 verdict of the reference's own Optimizer run on the same
inputs (``tests/golden/optimizer_runs.json``, row counts reduced so the
oracle could run it); for the fused ones, against the oracle's restatement
of the checker (``oracle/verdict.py``) evaluating the chain each fused
kernel was emitted from."""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from oracle import mlx_cpu, verdict
from phew_b200.workloads import WORKLOADS, gelu_chain_inputs, rms_norm_inputs

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
SOURCES = GOLDEN / "sources"
RUNS = json.loads((GOLDEN / "optimizer_runs.json").read_text())


def _reduced_inputs(name, rows, size, seed):
    if name == "rms_norm":
        return rms_norm_inputs(size, seed, rows=rows[size])
    return gelu_chain_inputs(size, seed, rows=rows[size])


def _factory(mod, name, rows):
    def factory(size, seed):
        return [mod.array(a) for a in _reduced_inputs(name, rows, size, seed)], {}

    return factory


@pytest.mark.parametrize("name", ["rms_norm", "gelu_chain"])
def test_unfused_candidate_verdict_matches_reference_optimizer(mx, name):
    from phew_b200.candidate import evaluate_candidate

    key = f"{name}__fusion0"
    run = RUNS[key]
    src = (SOURCES / f"{key}.py").read_text()
    res = evaluate_candidate(WORKLOADS[name].make_fn(mx), _factory(mx, name, run["rows"]), src)
    assert res.verification_passed == run["verification_passed"]
    assert res.verification_details == run["verification_details"]
    assert res.output_source == src
    assert [ln for ln in res.search_trace if ln.startswith("Step")] == [
        "Step 1: Baseline benchmark", "Step 6: Benchmark candidate", "Step 7: Equivalence verification"]
    assert set(res.size_speedups) == {"small", "typical", "large"}


@pytest.mark.parametrize("name", ["rms_norm", "gelu_chain"])
def test_fused_candidate_verdict_matches_oracle(mx, name):
    """With elementwise fusion on, the reference emits a fused kernel
    (rms_norm: the tail after the mean; the chain: all 14 ops)."""
    from phew_b200.candidate import evaluate_candidate

    key = f"{name}__fusion1"
    src = (SOURCES / f"{key}.py").read_text()
    assert "mx.fast.cuda_kernel(" in src
    rows = RUNS[f"{name}__fusion0"]["rows"]
    res = evaluate_candidate(WORKLOADS[name].make_fn(mx), _factory(mx, name, rows), src)
    mlx_cpu.CUDA_CHAINS.update(json.loads((SOURCES / "cuda_chains.json").read_text()))
    osrc = src.replace("import phew_b200.mx as mx", "import oracle.mlx_cpu as mx").replace(
        "from phew_b200.mx import fast", "from oracle.mlx_cpu import fast")
    ns: dict = {}
    exec(compile(osrc, key, "exec"), ns)
    passed, failures = verdict.check(WORKLOADS[name].make_fn(mlx_cpu), ns["optimized"],
                                     _factory(mlx_cpu, name, rows), mlx_cpu, {"fp32_to_fp32"})
    assert res.verification_passed == passed, (res.verification_details, failures)
    assert res.verification_details == failures


@pytest.mark.parametrize("name", ["rms_norm", "gelu_chain"])
def test_fused_candidate_at_benchmark_sizes(mx, name):
    """At the benchmark shapes the fused candidate is verified, keeps its
    source, and beats the op-by-op baseline at every size by CUDA-event
    timing (the reference's significance rule: > 3 % at all sizes)."""
    from phew_b200.candidate import evaluate_candidate

    key = f"{name}__fusion1"
    src = (SOURCES / f"{key}.py").read_text()
    w = WORKLOADS[name]
    res = evaluate_candidate(w.make_fn(mx), w.input_factory(mx), src)
    assert res.verification_passed, res.verification_details
    assert res.output_source == src
    assert res.speedup > 1.03 and res.is_significant, (res.speedup, res.size_speedups)


def test_failed_verification_drops_the_candidate(mx):
    """A candidate that is not equivalent is dropped (optimizer.py:318-327):
    here the rms_norm harness against a source that doubles the weight."""
    from phew_b200.candidate import DROPPED_SOURCE, evaluate_candidate

    src = (SOURCES / "rms_norm__fusion0.py").read_text().replace(
        "mx.fast.rms_norm(x0, x1, eps=1e-05)", "mx.fast.rms_norm(x0, x1 * 2.0, eps=1e-05)")
    rows = RUNS["rms_norm__fusion0"]["rows"]
    res = evaluate_candidate(WORKLOADS["rms_norm"].make_fn(mx), _factory(mx, "rms_norm", rows), src)
    assert not res.verification_passed and res.verification_details
    assert res.output_source == DROPPED_SOURCE and not res.is_significant
    assert "Verification FAILED — candidate dropped" in res.warnings
